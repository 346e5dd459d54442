;;;; b200-encoder.lisp -- ex-nihilo's prompt encoder on libexn_b200.so (sm_100a).
;;;;
;;;; Loaded after b200-dit.lisp (which loads the library).  It replaces the
;;;; text model's forward of src/encoder.lisp (illatio's qwen3 forward, on a
;;;; second GPU or the CPU) by the library's, on the DiT's own B200, and keeps
;;;; that file's functions and lambda lists:
;;;;
;;;;   (load-encoder path &key device threads)     src/encoder.lisp:41-48
;;;;   (encoder-gpu-p model)                       src/encoder.lisp:50-53
;;;;   (encoder-states model ids &key rope)        src/encoder.lisp:143-183
;;;;   (mrope-table positions rd base)             src/encoder.lisp:26-39
;;;;
;;;; The library builds the M-RoPE rows itself from the (t h w) positions, so
;;;; mrope-table here keeps the positions and encoder-states hands them to
;;;; exn_enc_states; encode-edit-prompt's call (encoder-states model ids :rope
;;;; (mrope-table positions ...)) is unchanged.  Tokenising stays with illatio's
;;;; tokenizer of the same GGUF (il::tokenize), which encode-prompt calls on
;;;; the model's TOKENIZER slot.  The alien routines mirror include/exn_b200.h;
;;;; the repository's tests check their names, argument counts and argument
;;;; types against that header.

(in-package #:ex-nihilo)

;;; --- the C ABI (include/exn_b200.h, the prompt encoder's section) -----------------------

(sb-alien:define-alien-type nil
  (sb-alien:struct exn-enc-config
    (width sb-alien:int) (layers sb-alien:int) (heads sb-alien:int) (kv-heads sb-alien:int)
    (ffn sb-alien:int) (vocab sb-alien:int) (theta double-float) (device sb-alien:int)))

(sb-alien:define-alien-routine ("exn_enc_default_config" %enc-default-config) sb-alien:void
  (cfg (* (sb-alien:struct exn-enc-config))))

(sb-alien:define-alien-routine ("exn_enc_open" %enc-open) sb-alien:int
  (cfg (* (sb-alien:struct exn-enc-config)))
  (out (* sb-sys:system-area-pointer)))

(sb-alien:define-alien-routine ("exn_enc_close" %enc-close) sb-alien:void
  (e sb-sys:system-area-pointer))

(sb-alien:define-alien-routine ("exn_enc_last_error" %enc-last-error) sb-alien:c-string
  (e sb-sys:system-area-pointer))

(sb-alien:define-alien-routine ("exn_enc_load_gguf" %enc-load-gguf) sb-alien:int
  (e sb-sys:system-area-pointer)
  (path sb-alien:c-string))

(sb-alien:define-alien-routine ("exn_enc_states" %enc-states) sb-alien:int
  (e sb-sys:system-area-pointer)
  (ids sb-sys:system-area-pointer)
  (n sb-alien:int)
  (positions sb-sys:system-area-pointer)
  (states sb-sys:system-area-pointer))

(sb-alien:define-alien-routine ("exn_enc_release" %enc-release) sb-alien:int
  (e sb-sys:system-area-pointer))

;;; --- the reference's functions -----------------------------------------------------------

(defstruct (genc (:constructor %make-genc (handle width tokenizer)))
  handle width
  ;; illatio's model of the same GGUF, for il::tokenize (or NIL)
  tokenizer)

(defun enc-check (e status)
  (unless (zerop status)
    (error "libexn_b200: ~A" (%enc-last-error (if e (genc-handle e) (sb-sys:int-sap 0))))))

(defun load-encoder (path &key device threads)
  "The prompt encoder: the qwen3vl GGUF at PATH, its text model on CUDA device DEVICE
   (0 when NIL), next to the DiT."
  (declare (ignore threads))
  (sb-alien:with-alien ((cfg (sb-alien:struct exn-enc-config))
                        (h sb-sys:system-area-pointer))
    (%enc-default-config (sb-alien:addr cfg))
    (setf (sb-alien:slot cfg 'device) (if (integerp device) device 0))
    (enc-check nil (%enc-open (sb-alien:addr cfg) (sb-alien:addr h)))
    (let ((e (%make-genc h (sb-alien:slot cfg 'width) nil)))
      (handler-bind ((error (lambda (c) (declare (ignore c)) (%enc-close h))))
        (enc-check e (%enc-load-gguf h (namestring path))))
      e)))

(defun encoder-gpu-p (model)
  "The library's encoder always runs on a GPU."
  (genc-p model))

(defun mrope-table (positions rd base)
  "POSITIONS, a list of (t h w), kept for encoder-states: the library turns them into
   Qwen3-VL's interleaved M-RoPE rows itself (RD 128, BASE the model's 5e6)."
  (declare (ignore rd base))
  (list :positions positions))

(defun encoder-states (model ids &key rope)
  "Every token's state after the text model's last block, before its final norm:
   (length IDS) x 4096 floats.  ROPE: mrope-table's positions, or NIL for a text
   prompt's (i i i)."
  (let* ((n (length ids)) (d (genc-width model))
         (all (make-array (* n d) :element-type 'single-float))
         (idv (make-array n :element-type '(signed-byte 32) :initial-contents (coerce ids 'list)))
         (pos (and rope (make-array (* 3 n) :element-type '(signed-byte 32)
                                            :initial-contents (loop for p in (second rope) append p)))))
    (sb-sys:with-pinned-objects (all idv pos)
      (enc-check model (%enc-states (genc-handle model) (sb-sys:vector-sap idv) n
                                    (if pos (sb-sys:vector-sap pos) (sb-sys:int-sap 0))
                                    (sb-sys:vector-sap all))))
    all))

(defun encoder-release (model)
  "The encoder's scratch freed (the weights stay)."
  (enc-check model (%enc-release (genc-handle model))))
