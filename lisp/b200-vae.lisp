;;;; b200-vae.lisp -- ex-nihilo's VAE decoder on libexn_b200.so (sm_100a).
;;;;
;;;; Loaded after b200-dit.lisp (which loads the library).  It replaces the
;;;; decoder half of src/cuda-vae.lisp and keeps that file's functions and
;;;; lambda lists, so decode-latent (src/generate.lisp) is unchanged:
;;;;
;;;;   (upload-vae path &key (device 0))      src/cuda-vae.lisp:15-27
;;;;   (vae-decode v latent h w)              src/cuda-vae.lisp:94-136
;;;;   (vae-release v)                        src/cuda-vae.lisp:29-33
;;;;
;;;; The encoder (vae-encode, src/cuda-vae.lisp:138-) is not in the library:
;;;; an edit's input picture still goes through the reference's own encoder.
;;;; The alien routines mirror include/exn_b200.h; the repository's tests check
;;;; their names, argument counts and argument types against that header.

(in-package #:ex-nihilo)

;;; --- the C ABI (include/exn_b200.h, the VAE section) ---------------------------------

(sb-alien:define-alien-routine ("exn_vae_open" %vae-open) sb-alien:int
  (device sb-alien:int)
  (out (* sb-sys:system-area-pointer)))

(sb-alien:define-alien-routine ("exn_vae_close" %vae-close) sb-alien:void
  (v sb-sys:system-area-pointer))

(sb-alien:define-alien-routine ("exn_vae_last_error" %vae-last-error) sb-alien:c-string
  (v sb-sys:system-area-pointer))

(sb-alien:define-alien-routine ("exn_vae_load_safetensors" %vae-load-safetensors) sb-alien:int
  (v sb-sys:system-area-pointer)
  (path sb-alien:c-string))

(sb-alien:define-alien-routine ("exn_vae_decode" %vae-decode) sb-alien:int
  (v sb-sys:system-area-pointer)
  (latent sb-sys:system-area-pointer)
  (h sb-alien:int)
  (w sb-alien:int)
  (rgba sb-sys:system-area-pointer))

(sb-alien:define-alien-routine ("exn_vae_release" %vae-release) sb-alien:int
  (v sb-sys:system-area-pointer))

;;; --- the reference's functions -----------------------------------------------------------

(defstruct (gvae (:constructor %make-gvae (handle)))
  handle)

(defun vae-check (v status)
  (unless (zerop status)
    (error "libexn_b200: ~A" (%vae-last-error (if v (gvae-handle v) (sb-sys:int-sap 0))))))

(defun upload-vae (path &key (device 0))
  "The decoder in the safetensors at PATH on CUDA device DEVICE, after open-vae's
   checks of every decoder tensor's name and shape (the encoder's are ignored)."
  (sb-alien:with-alien ((h sb-sys:system-area-pointer))
    (vae-check nil (%vae-open device (sb-alien:addr h)))
    (let ((v (%make-gvae h)))
      (handler-bind ((error (lambda (c) (declare (ignore c)) (%vae-close h))))
        (vae-check v (%vae-load-safetensors h (namestring path))))
      v)))

(defun vae-decode (v latent h w)
  "LATENT (64 x H x W floats, channel-major, denormalized) decoded: the picture as
   16H x 16W x 4 floats (RGBA, -1 .. 1), row-major, channels last, and its height
   and width.  H x W must be a multiple of 64."
  (let ((px (make-array (* 16 h 16 w 4) :element-type 'single-float)))
    (sb-sys:with-pinned-objects (latent px)
      (vae-check v (%vae-decode (gvae-handle v) (sb-sys:vector-sap latent) h w (sb-sys:vector-sap px))))
    (values px (* 16 h) (* 16 w))))

(defun vae-release (v)
  "V's scratch freed (the weights stay), for the DiT's next picture."
  (vae-check v (%vae-release (gvae-handle v))))
