;;;; b200-dit.lisp -- ex-nihilo's DiT driver on libexn_b200.so (sm_100a).
;;;;
;;;; It takes the place of src/cuda-dit.lisp in ex-nihilo.asd on Linux and keeps
;;;; that file's exported functions and calling conventions, so load-engine,
;;;; generate, edit and decode-latent (src/generate.lisp) are unchanged:
;;;;
;;;;   (upload-dit path &key (device 0))                       src/cuda-dit.lisp:52-86
;;;;   (dit-velocity d context p latent h w sigma
;;;;                 &key prefix-key ref)                        src/cuda-dit.lisp:137-243
;;;;   (dit-release d)                                          src/cuda-dit.lisp:99-108
;;;;
;;;; plus (dit-euler d context p z h w sigmas &key prefix-key ref), which runs
;;;; the step loop of generate / edit (src/generate.lisp:133-135, 95-97) with
;;;; the latent kept on the device and the update z += (s' - s) v fused into the
;;;; last GEMM.  The alien routines below mirror include/exn_b200.h one for one;
;;;; the repository's tests check their names, argument counts and argument
;;;; types against that header (SBCL itself is not needed for that check).
;;;;
;;;; Every entry point returns an int status, 0 for success; a failure becomes
;;;; a Lisp error carrying exn_last_error's text, as the reference signals its
;;;; own errors (open-dit's list of bad tensors included).

(in-package #:ex-nihilo)

(sb-alien:load-shared-object "libexn_b200.so")

;;; --- the C ABI (include/exn_b200.h) ---------------------------------------------------

(sb-alien:define-alien-type nil
  (sb-alien:struct exn-config
    (width sb-alien:int) (layers sb-alien:int) (ffn sb-alien:int) (latent sb-alien:int)
    (context sb-alien:int) (freq sb-alien:int) (head-dim sb-alien:int) (device sb-alien:int)))

(sb-alien:define-alien-type nil
  (sb-alien:struct exn-ref
    (a sb-alien:int) (latent (* single-float)) (rh sb-alien:int) (rw sb-alien:int)))

(sb-alien:define-alien-routine ("exn_abi_version" %abi-version) sb-alien:int)

(sb-alien:define-alien-routine ("exn_default_config" %default-config) sb-alien:void
  (cfg (* (sb-alien:struct exn-config))))

(sb-alien:define-alien-routine ("exn_open" %open) sb-alien:int
  (cfg (* (sb-alien:struct exn-config)))
  (out (* sb-sys:system-area-pointer)))

(sb-alien:define-alien-routine ("exn_close" %close) sb-alien:void
  (h sb-sys:system-area-pointer))

(sb-alien:define-alien-routine ("exn_last_error" %last-error) sb-alien:c-string
  (h sb-sys:system-area-pointer))

(sb-alien:define-alien-routine ("exn_load_gguf" %load-gguf) sb-alien:int
  (h sb-sys:system-area-pointer)
  (path sb-alien:c-string))

(sb-alien:define-alien-routine ("exn_velocity" %velocity) sb-alien:int
  (h sb-sys:system-area-pointer)
  (context sb-sys:system-area-pointer)
  (p sb-alien:int)
  (latent sb-sys:system-area-pointer)
  (hh sb-alien:int)
  (ww sb-alien:int)
  (sigma double-float)
  (prefix-key sb-alien:unsigned-long)
  (ref (* (sb-alien:struct exn-ref)))
  (v-out sb-sys:system-area-pointer))

(sb-alien:define-alien-routine ("exn_generate" %generate) sb-alien:int
  (h sb-sys:system-area-pointer)
  (context sb-sys:system-area-pointer)
  (p sb-alien:int)
  (z sb-sys:system-area-pointer)
  (hh sb-alien:int)
  (ww sb-alien:int)
  (sigmas sb-sys:system-area-pointer)
  (nsig sb-alien:int)
  (prefix-key sb-alien:unsigned-long)
  (ref (* (sb-alien:struct exn-ref))))

(sb-alien:define-alien-routine ("exn_release" %release) sb-alien:int
  (h sb-sys:system-area-pointer))

;;; --- the reference's functions on top of it ------------------------------------------

(defstruct (gdit (:constructor %make-gdit (handle)))
  handle
  ;; the prefix keys the reference compares with EQUAL, as nonzero 64-bit ids for the ABI
  (key nil) (key-id 0))

(defun exn-check (d status)
  (unless (zerop status)
    (error "libexn_b200: ~A" (%last-error (if d (gdit-handle d) (sb-sys:int-sap 0))))))

(defun upload-dit (path &key (device 0))
  "The DiT in the GGUF at PATH on CUDA device DEVICE, after open-dit's checks of its
   architecture, tensor names and dims."
  (sb-alien:with-alien ((cfg (sb-alien:struct exn-config))
                        (h sb-sys:system-area-pointer))
    (%default-config (sb-alien:addr cfg))
    (setf (sb-alien:slot cfg 'device) device)
    (exn-check nil (%open (sb-alien:addr cfg) (sb-alien:addr h)))
    (let ((d (%make-gdit h)))
      (handler-bind ((error (lambda (c) (declare (ignore c)) (%close h))))
        (exn-check d (%load-gguf h (namestring path))))
      d)))

(defun prefix-id (d key)
  "EQUAL keys give the same nonzero id; NIL gives 0 (nothing kept)."
  (cond ((null key) 0)
        ((equal key (gdit-key d)) (gdit-key-id d))
        (t (setf (gdit-key d) key) (incf (gdit-key-id d)))))

(defmacro with-ref ((var ref) &body body)
  "VAR: an exn_ref pointer for REF = (A LATENT RH RW), or a null pointer for NIL."
  (let ((r (gensym "REF")) (alien (gensym "ALIEN")))
    `(let ((,r ,ref))
       (sb-alien:with-alien ((,alien (sb-alien:struct exn-ref)))
         (when ,r
           (setf (sb-alien:slot ,alien 'a) (first ,r)
                 (sb-alien:slot ,alien 'latent)
                 (sb-sys:sap-alien (sb-sys:vector-sap (second ,r)) (* single-float))
                 (sb-alien:slot ,alien 'rh) (third ,r)
                 (sb-alien:slot ,alien 'rw) (fourth ,r)))
         (let ((,var (if ,r
                         (sb-alien:addr ,alien)
                         (sb-sys:sap-alien (sb-sys:int-sap 0) (* (sb-alien:struct exn-ref))))))
           ,@body)))))

(defun dit-velocity (d context p latent h w sigma &key (prefix-key nil) ref)
  "The DiT's velocity at noise level SIGMA: LATENT (64 x H x W floats, channel-major)
   in, the same shape out.  CONTEXT: the encoder's P x 4096 states.  With PREFIX-KEY
   the prompt's keys and values are kept after the first call and reused by the next
   calls with an EQUAL key.  REF = (A LATENT RH RW): a picture to edit, put in the
   prefix after the first A states."
  (let ((v (make-array (* 64 h w) :element-type 'single-float))
        (id (prefix-id d prefix-key)))
    (sb-sys:with-pinned-objects (context latent v (and ref (second ref)))
      (with-ref (r ref)
        (exn-check d (%velocity (gdit-handle d) (sb-sys:vector-sap context) p
                                (sb-sys:vector-sap latent) h w (coerce sigma 'double-float) id r
                                (sb-sys:vector-sap v)))))
    v))

(defun dit-euler (d context p z h w sigmas &key (prefix-key nil) ref)
  "generate's loop (loop for (s s2) on sigmas while s2 do z += (s2 - s) v) in one
   call: Z (64 x H x W floats) is updated in place and returned."
  (let ((s (make-array (length sigmas) :element-type 'double-float
                                       :initial-contents (mapcar (lambda (x) (coerce x 'double-float))
                                                                 sigmas)))
        (id (prefix-id d prefix-key)))
    (sb-sys:with-pinned-objects (context z s (and ref (second ref)))
      (with-ref (r ref)
        (exn-check d (%generate (gdit-handle d) (sb-sys:vector-sap context) p (sb-sys:vector-sap z) h w
                                (sb-sys:vector-sap s) (length sigmas) id r))))
    z))

(defun dit-release (d)
  "Free the step buffers and the kept prompt keys and values (the weights stay)."
  (exn-check d (%release (gdit-handle d))))
