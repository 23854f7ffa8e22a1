;;;; The B200 CUDA accelerator backend for llambda, as a system of its own.
;;;;
;;;; It loads after llambda (whose accelerator.lisp defines the descriptor
;;;; protocol) and registers the :cuda descriptor, so llambda's own system and
;;;; its test asserting the registered backends are (:gpu :npu) stay as they are.
;;;; libllambda_cuda.so (include/llambda_cuda.h) must be on the foreign library
;;;; search path, or named by LLAMBDA_CUDA_LIBRARY.

(asdf:defsystem #:llambda-cuda
  :description "B200 (sm_100a) backend for llambda's quantized feed-forward path"
  :version "0.2.0"
  :license "MIT"
  :serial t
  :depends-on (#:llambda #:cffi)
  :components ((:module "accelerators"
                :serial t
                :components ((:file "cuda")))))
