"""The Lisp bindings (lisp/b200-dit.lisp, b200-vae.lisp, b200-encoder.lisp) against the C header they bind.

SBCL is not installed here, so the binding cannot run; these checks read it as
text: the file is balanced s-expressions, every sb-alien routine names a
function that include/exn_b200.h declares, with the same number of arguments
and the same kind of each argument and result, the two structs list the
header's fields in the header's order, and the drivers keep the reference's
function names and lambda lists (src/cuda-dit.lisp:52, 99, 137; src/cuda-vae.lisp:15, 29, 94;
src/encoder.lisp:26, 41, 143)."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LISP = os.path.join(ROOT, "lisp", "b200-dit.lisp")
LISP_VAE = os.path.join(ROOT, "lisp", "b200-vae.lisp")
LISP_ENC = os.path.join(ROOT, "lisp", "b200-encoder.lisp")
HEADER = os.path.join(ROOT, "include", "exn_b200.h")


# --------------------------------------------------------------------------- a small reader

def read_forms(text):
    """Top-level forms of Lisp source as nested lists of atoms (strings keep their quotes)."""
    toks = re.findall(r'"(?:[^"\\]|\\.)*"|;[^\n]*|[()]|\'|`|,@|,|[^\s()\'`,";]+', text)
    stack, top = [[]], None
    for t in toks:
        if t.startswith(";") or t in ("'", "`", ",", ",@"):
            continue
        if t == "(":
            stack.append([])
        elif t == ")":
            assert len(stack) > 1, "unbalanced ')'"
            top = stack.pop()
            stack[-1].append(top)
        else:
            stack[-1].append(t.lower() if not t.startswith('"') else t)
    assert len(stack) == 1, "unbalanced '(': %d open" % (len(stack) - 1)
    return stack[0]


# --------------------------------------------------------------------------- kinds of C and Lisp types

def c_kind(decl):
    d = decl.replace("const", " ").strip()
    if "*" in d:
        return "ptr"
    d = re.sub(r"\s+\w+$", "", d) if len(d.split()) > 1 else d
    return {"int": "i32", "double": "f64", "uint64_t": "u64", "size_t": "u64", "int64_t": "i64",
            "long long": "i64", "void": "void"}[d.strip()]


def lisp_kind(t):
    if isinstance(t, list):
        if t[0] == "*":
            return "ptr"
        if t[0] in ("sb-alien:unsigned", "unsigned") and t[1] == "64":
            return "u64"
        raise AssertionError(t)
    return {"sb-alien:int": "i32", "double-float": "f64", "sb-alien:unsigned-long": "u64",
            "sb-alien:long-long": "i64", "sb-alien:c-string": "ptr", "sb-sys:system-area-pointer": "ptr",
            "sb-alien:void": "void"}[t]


def header_functions():
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for ret, name, args in re.findall(r"\b((?:const\s+)?\w+\s*\**)\s*\b(exn_\w+)\s*\(([^)]*)\)\s*;", src):
        kinds = [] if args.strip() in ("", "void") else [c_kind(a) for a in args.split(",")]
        out[name] = ("ptr" if "*" in ret else c_kind(ret), kinds)
    return out


def header_struct(name):
    """(field, kind) of a typedef'd struct of the header, in order; "int rh, rw" gives two fields."""
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    body = re.search(r"typedef struct %s \{(.*?)\}" % name, src, flags=re.S).group(1)
    fields = []
    for decl in body.split(";"):
        decl = decl.replace("const", " ").strip()
        if not decl:
            continue
        base, rest = re.match(r"(\w+)\s*(.*)$", decl).groups()
        for n in rest.split(","):
            kind = "ptr" if "*" in n else c_kind(base)
            fields.append((n.replace("*", "").strip().replace("_", "-"), kind))
    return fields


def forms(path=LISP):
    return read_forms(open(path).read())


# --------------------------------------------------------------------------- tests

def test_the_file_reads():
    fs = forms()
    assert fs[0] == ["in-package", "#:ex-nihilo"]
    assert any(f[0] == "sb-alien:load-shared-object" and f[1] == '"libexn_b200.so"' for f in fs)


def test_alien_routines_match_the_header():
    decl = header_functions()
    routines = [f for path in (LISP, LISP_VAE, LISP_ENC) for f in forms(path)
                if f[0] == "sb-alien:define-alien-routine"]
    assert len(routines) >= 21
    for f in routines:
        cname = f[1][0].strip('"')
        assert cname in decl, cname
        ret, kinds = decl[cname]
        assert lisp_kind(f[2]) == ret, (cname, f[2], ret)
        args = f[3:]
        assert len(args) == len(kinds), (cname, len(args), len(kinds))
        for (argname, t), k in zip(args, kinds):
            assert lisp_kind(t) == k, (cname, argname, t, k)
    bound = {f[1][0].strip('"') for f in routines}
    for needed in ("exn_open", "exn_close", "exn_last_error", "exn_load_gguf", "exn_velocity", "exn_generate",
                   "exn_release", "exn_default_config", "exn_vae_open", "exn_vae_close", "exn_vae_last_error",
                   "exn_vae_load_safetensors", "exn_vae_decode", "exn_vae_release", "exn_enc_default_config",
                   "exn_enc_open", "exn_enc_close", "exn_enc_last_error", "exn_enc_load_gguf", "exn_enc_states",
                   "exn_enc_release"):
        assert needed in bound, needed


def test_structs_match_the_header():
    types = {}
    for f in forms() + forms(LISP_ENC):
        if f[0] == "sb-alien:define-alien-type" and isinstance(f[2], list) and f[2][0] == "sb-alien:struct":
            types[f[2][1]] = [(fld[0], lisp_kind(fld[1])) for fld in f[2][2:]]
    assert types["exn-config"] == header_struct("exn_config")
    assert types["exn-ref"] == header_struct("exn_ref")
    assert types["exn-enc-config"] == header_struct("exn_enc_config")


def test_driver_keeps_the_reference_lambda_lists():
    defuns = {f[1]: f[2] for f in forms() if f[0] == "defun"}
    # src/cuda-dit.lisp:52, 137, 99
    assert defuns["upload-dit"] == ["path", "&key", ["device", "0"]]
    assert defuns["dit-velocity"] == ["d", "context", "p", "latent", "h", "w", "sigma", "&key",
                                      ["prefix-key", "nil"], "ref"]
    assert defuns["dit-release"] == ["d"]
    assert "dit-euler" in defuns


def test_vae_driver_keeps_the_reference_lambda_lists():
    fs = forms(LISP_VAE)
    assert fs[0] == ["in-package", "#:ex-nihilo"]
    defuns = {f[1]: f[2] for f in fs if f[0] == "defun"}
    # src/cuda-vae.lisp:15, 94, 29
    assert defuns["upload-vae"] == ["path", "&key", ["device", "0"]]
    assert defuns["vae-decode"] == ["v", "latent", "h", "w"]
    assert defuns["vae-release"] == ["v"]


def test_encoder_driver_keeps_the_reference_lambda_lists():
    fs = forms(LISP_ENC)
    assert fs[0] == ["in-package", "#:ex-nihilo"]
    defuns = {f[1]: f[2] for f in fs if f[0] == "defun"}
    # src/encoder.lisp:41, 143, 26, 50
    assert defuns["load-encoder"] == ["path", "&key", "device", "threads"]
    assert defuns["encoder-states"] == ["model", "ids", "&key", "rope"]
    assert defuns["mrope-table"] == ["positions", "rd", "base"]
    assert defuns["encoder-gpu-p"] == ["model"]
