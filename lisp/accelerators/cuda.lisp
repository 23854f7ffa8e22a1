;;;; accelerators/cuda.lisp — the :cuda accelerator-backend descriptor.
;;;;
;;;; A sibling of llambda's accelerators/directml.lisp: the same eighteen
;;;; required slots of make-accelerator-backend (accelerator.lisp:3-91), over
;;;; the C ABI of libllambda_cuda.so (include/llambda_cuda.h) instead of the
;;;; ONNX Runtime bridge (native/llambda_npu.h).  Projections are the raw GGUF
;;;; tensor bytes behind a small header (no ONNX graph), so the exporter copies
;;;; them out of the model's mapping.
;;;;
;;;; The routed experts bypass the projection store (llambda.lisp L4951-4971),
;;;; so this file also defines the MoE half: a foreign struct for one layer's
;;;; tensors and the make/run/close functions behind the optional MoE slots.
;;;; Written against the ABI; SBCL is not available where this backend is
;;;; built, and the same call sequence is exercised through ctypes by the
;;;; Python restatement (llambda_b200/accelerator.py) and its tests.

(in-package #:llambda)

;;; ------------------------------------------------------------------ library

(cffi:define-foreign-library llambda-cuda
  (:unix (:or (:default "libllambda_cuda") "libllambda_cuda.so"))
  (t (:default "libllambda_cuda")))

(defvar *cuda-library-loaded-p* nil)

(defun load-cuda-backend ()
  "Loads libllambda_cuda once; LLAMBDA_CUDA_LIBRARY may name the file."
  (unless *cuda-library-loaded-p*
    (let ((explicit (uiop:getenv "LLAMBDA_CUDA_LIBRARY")))
      (if (and explicit (plusp (length explicit)))
          (cffi:load-foreign-library explicit)
          (cffi:load-foreign-library 'llambda-cuda)))
    (setf *cuda-library-loaded-p* t))
  t)

(cffi:defcfun ("llambda_cuda_probe" %cuda-probe) :int)
(cffi:defcfun ("llambda_cuda_bridge_version" %cuda-bridge-version) :string)
(cffi:defcfun ("llambda_cuda_runtime_version" %cuda-runtime-version) :string)
(cffi:defcfun ("llambda_cuda_last_error" %cuda-last-error) :string)
(cffi:defcfun ("llambda_cuda_sha256" %cuda-sha256) :int
  (data :pointer) (data-size :size) (output :pointer) (output-size :size))
(cffi:defcfun ("llambda_cuda_session_create" %cuda-session-create) :int
  (model-path :string) (result :pointer))
(cffi:defcfun ("llambda_cuda_session_destroy" %cuda-session-destroy) :void
  (session :pointer))
(cffi:defcfun ("llambda_cuda_session_input_element_count" %cuda-session-input-element-count)
    :size
  (session :pointer))
(cffi:defcfun ("llambda_cuda_session_output_element_count" %cuda-session-output-element-count)
    :size
  (session :pointer))
(cffi:defcfun ("llambda_cuda_session_run" %cuda-session-run) :int
  (session :pointer) (input :pointer) (input-count :size)
  (output :pointer) (output-count :size))
(cffi:defcfun ("llambda_cuda_moe_session_create" %cuda-moe-session-create) :int
  (desc :pointer) (result :pointer))
(cffi:defcfun ("llambda_cuda_moe_session_destroy" %cuda-moe-session-destroy) :void
  (session :pointer))
(cffi:defcfun ("llambda_cuda_moe_session_hidden" %cuda-moe-session-hidden) :size
  (session :pointer))
(cffi:defcfun ("llambda_cuda_moe_session_run" %cuda-moe-session-run) :int
  (session :pointer) (x :pointer) (tokens :size) (out :pointer)
  (selected :pointer) (weights :pointer))

;;; ------------------------------------------------------------------ errors

(define-condition cuda-backend-error (simple-error) ())

(defun cuda-backend-error (format-control &rest format-arguments)
  (error 'cuda-backend-error
         :format-control format-control
         :format-arguments format-arguments))

(defun check-cuda-status (status operation)
  "Every fallible entry point returns 0 or -1 and leaves a thread-local
message (the bridge convention of llambda_npu.cpp:24, 43-49)."
  (unless (zerop status)
    (cuda-backend-error "~a failed: ~a" operation (%cuda-last-error))))

(defun cuda-backend-available-p ()
  (let ((result (%cuda-probe)))
    (cond ((= result 1) t)
          ((zerop result) nil)
          (t (cuda-backend-error "CUDA backend probe failed: ~a" (%cuda-last-error))))))

;;; ------------------------------------------------------------------ projections

(defstruct (cuda-session (:constructor %make-cuda-session))
  (pointer (cffi:null-pointer))
  (input-element-count 0 :type fixnum)
  (output-element-count 0 :type fixnum))

(defun make-cuda-session (model-path)
  (cffi:with-foreign-object (result :pointer)
    (check-cuda-status (%cuda-session-create (uiop:native-namestring model-path) result)
                       "CUDA session creation")
    (let ((pointer (cffi:mem-ref result :pointer)))
      (%make-cuda-session :pointer pointer
                          :input-element-count (%cuda-session-input-element-count pointer)
                          :output-element-count (%cuda-session-output-element-count pointer)))))

(defun close-cuda-session (session)
  (let ((pointer (cuda-session-pointer session)))
    (unless (cffi:null-pointer-p pointer)
      (%cuda-session-destroy pointer)
      (setf (cuda-session-pointer session) (cffi:null-pointer))))
  nil)

(defun run-cuda-session-into (dest session input)
  (declare (type (simple-array single-float (*)) dest input))
  (cffi:with-pointer-to-vector-data (in input)
    (cffi:with-pointer-to-vector-data (out dest)
      (check-cuda-status (%cuda-session-run (cuda-session-pointer session)
                                            in (length input) out (length dest))
                         "CUDA GEMV")))
  dest)

(defconstant +cuda-projection-header-bytes+ 64)

(defun write-u32-le (stream value)
  (dotimes (i 4) (write-byte (ldb (byte 8 (* 8 i)) value) stream)))

(defun write-u64-le (stream value)
  (dotimes (i 8) (write-byte (ldb (byte 8 (* 8 i)) value) stream)))

(defun export-model-cuda-projection (model tensor-name output-path
                                     &key python-command generator-path)
  "Writes the file llambda_cuda_session_create opens: \"LLBCUDA1\", u32
version 1, u32 GGML type, u64 ne0 ne1 ne2, u64 data bytes, u64 data offset
(64), zero padding, then the tensor's raw bytes from the mapping.  Written to
a temporary name and renamed, like the ONNX exporter (L391-400)."
  (declare (ignore python-command generator-path))
  (let* ((info (gguf-model-tensor-info model tensor-name t))
         (dimensions (getf info :dimensions))
         (byte-size (getf info :byte-size))
         (source (cffi:inc-pointer (gguf-model-mapping model) (getf info :data-offset)))
         (temporary (make-pathname :type "tmp" :defaults output-path)))
    (ensure-directories-exist output-path)
    (with-open-file (stream temporary :direction :output :element-type '(unsigned-byte 8)
                                      :if-exists :supersede)
      (map nil (lambda (c) (write-byte (char-code c) stream)) "LLBCUDA1")
      (write-u32-le stream 1)
      (write-u32-le stream (getf info :type-tag))
      (write-u64-le stream (first dimensions))
      (write-u64-le stream (or (second dimensions) 1))
      (write-u64-le stream (or (third dimensions) 1))
      (write-u64-le stream byte-size)
      (write-u64-le stream +cuda-projection-header-bytes+)
      (dotimes (i (- +cuda-projection-header-bytes+ 56)) (write-byte 0 stream))
      (dotimes (i byte-size)
        (write-byte (cffi:mem-aref source :unsigned-char i) stream)))
    (rename-file temporary output-path)
    output-path))

;;; ------------------------------------------------------------------ MoE layers

(cffi:defcstruct cuda-tensor
  (type :int)
  (ne0 :uint64) (ne1 :uint64) (ne2 :uint64)
  (data :pointer))

;;; Field order of llambda_cuda_moe_desc (include/llambda_cuda.h).
(cffi:defcstruct cuda-moe-desc
  (arch :int)
  (hidden :uint64)
  (top-k :int)
  (weight-scale :float)
  (weights-norm :int)
  (data-on-device :int)
  (router (:struct cuda-tensor))
  (router-bias :pointer)
  (shared-gate-inp :pointer)
  (gate-exps (:struct cuda-tensor))
  (up-exps (:struct cuda-tensor))
  (down-exps (:struct cuda-tensor))
  (gate-shexp (:struct cuda-tensor))
  (up-shexp (:struct cuda-tensor))
  (down-shexp (:struct cuda-tensor))
  (expert-begin :int)
  (expert-end :int)
  (shared-here :int)
  (max-tokens :int)
  (input-norm :pointer)
  (norm-epsilon :float)
  (add-residual :int)
  (latent-down (:struct cuda-tensor))
  (latent-up (:struct cuda-tensor)))

(defconstant +cuda-arch-qwen3next+ 0)
(defconstant +cuda-arch-nemotron-h-moe+ 1)

(defstruct (cuda-moe-session (:constructor %make-cuda-moe-session))
  (pointer (cffi:null-pointer))
  (hidden 0 :type fixnum))

(defun fill-cuda-tensor (slot model layer-index suffix)
  "Points a cuda-tensor at blk.N.SUFFIX inside the mapping, or leaves it
empty (data NULL) when the layer has no such tensor."
  (let ((info (gguf-model-tensor-info model (make-layer-tensor-name layer-index suffix) nil)))
    (cffi:with-foreign-slots ((type ne0 ne1 ne2 data) slot (:struct cuda-tensor))
      (if info
          (let ((dimensions (getf info :dimensions)))
            (setf type (getf info :type-tag)
                  ne0 (first dimensions)
                  ne1 (or (second dimensions) 1)
                  ne2 (or (third dimensions) 1)
                  data (cffi:inc-pointer (gguf-model-mapping model) (getf info :data-offset))))
          (setf type 0 ne0 0 ne1 0 ne2 0 data (cffi:null-pointer))))))

(defun layer-vector-pointer (model layer-index suffix)
  (let ((info (gguf-model-tensor-info model (make-layer-tensor-name layer-index suffix) nil)))
    (if info
        (cffi:inc-pointer (gguf-model-mapping model) (getf info :data-offset))
        (cffi:null-pointer))))

(defun make-cuda-moe-session (model layer-index &key (max-tokens 64))
  "One layer's MoE block (qwen3next-moe-into L5321-5426 or
nemotron-h-moe-ffn-into L5827-5949) uploaded to the GPU; the metadata the
Lisp blocks read (L5329-5332, L6165-6171) fills the descriptor."
  (let* ((kv (gguf-model-kv-pairs model))
         (architecture (gguf-kv-value kv "general.architecture"))
         (nemotron-p (string= architecture "nemotron_h_moe"))
         (router (gguf-model-tensor-info model (make-layer-tensor-name layer-index "ffn_gate_inp")
                                         t)))
    (cffi:with-foreign-objects ((desc '(:struct cuda-moe-desc)) (result :pointer))
      (cffi:with-foreign-slots ((arch hidden top-k weight-scale weights-norm data-on-device
                                 router-bias shared-gate-inp expert-begin expert-end
                                 shared-here max-tokens input-norm norm-epsilon add-residual)
                                desc (:struct cuda-moe-desc))
        (setf arch (if nemotron-p +cuda-arch-nemotron-h-moe+ +cuda-arch-qwen3next+)
              hidden (tensor-column-count router)
              top-k (if nemotron-p
                        (gguf-kv-value kv "nemotron_h_moe.expert_used_count")
                        (gguf-kv-value kv "qwen3next.expert_used_count"))
              weight-scale (if nemotron-p
                               (coerce (or (gguf-kv-value-or-nil
                                            kv "nemotron_h_moe.expert_weights_scale")
                                           1.0f0)
                                       'single-float)
                               1.0f0)
              weights-norm (if (or (not nemotron-p)
                                   (gguf-kv-value-or-nil kv "nemotron_h_moe.expert_weights_norm"))
                               1 0)
              data-on-device 0
              router-bias (layer-vector-pointer model layer-index "exp_probs_b.bias")
              shared-gate-inp (layer-vector-pointer model layer-index "ffn_gate_inp_shexp")
              expert-begin 0
              expert-end 0
              shared-here 1
              max-tokens max-tokens
              input-norm (cffi:null-pointer)
              norm-epsilon 0.0f0
              add-residual 0))
      (loop for (slot suffix) in '((router "ffn_gate_inp")
                                   (gate-exps "ffn_gate_exps") (up-exps "ffn_up_exps")
                                   (down-exps "ffn_down_exps") (gate-shexp "ffn_gate_shexp")
                                   (up-shexp "ffn_up_shexp") (down-shexp "ffn_down_shexp")
                                   (latent-down "ffn_latent_down") (latent-up "ffn_latent_up"))
            do (fill-cuda-tensor (cffi:foreign-slot-pointer desc '(:struct cuda-moe-desc) slot)
                                 model layer-index suffix))
      (check-cuda-status (%cuda-moe-session-create desc result) "CUDA MoE session creation")
      (let ((pointer (cffi:mem-ref result :pointer)))
        (%make-cuda-moe-session :pointer pointer
                                :hidden (%cuda-moe-session-hidden pointer))))))

(defun run-cuda-moe-into (dest session input tokens)
  "dest[t] = MoE(input[t]) for TOKENS row-major vectors of the layer's
hidden size."
  (declare (type (simple-array single-float (*)) dest input))
  (cffi:with-pointer-to-vector-data (in input)
    (cffi:with-pointer-to-vector-data (out dest)
      (check-cuda-status (%cuda-moe-session-run (cuda-moe-session-pointer session)
                                                in tokens out
                                                (cffi:null-pointer) (cffi:null-pointer))
                         "CUDA MoE layer")))
  dest)

(defun close-cuda-moe-session (session)
  (let ((pointer (cuda-moe-session-pointer session)))
    (unless (cffi:null-pointer-p pointer)
      (%cuda-moe-session-destroy pointer)
      (setf (cuda-moe-session-pointer session) (cffi:null-pointer))))
  nil)

;;; ------------------------------------------------------------------ descriptor

(register-accelerator-backend
 (make-accelerator-backend
  :name :cuda
  :display-name "CUDA (B200)"
  :priority 5                       ; ahead of :gpu (10) and :npu (20)
  :initialization-priority 30
  :load-function #'load-cuda-backend
  :available-p-function #'cuda-backend-available-p
  :runtime-version-function (lambda () (%cuda-runtime-version))
  :bridge-version-function (lambda () (%cuda-bridge-version))
  :make-session-function
  (lambda (model-path &key cache-directory cache-key)
    (declare (ignore cache-directory cache-key))
    (make-cuda-session model-path))
  :close-session-function #'close-cuda-session
  :run-session-function #'run-cuda-session-into
  :session-input-element-count-function #'cuda-session-input-element-count
  :session-output-element-count-function #'cuda-session-output-element-count
  :error-p-function (lambda (condition)
                      (typep condition 'cuda-backend-error))
  :signal-error-function #'cuda-backend-error
  :default-cache-directory-function #'default-gpu-cache-directory
  :export-projection-function #'export-model-cuda-projection
  :weight-format :gguf-raw
  :foreign-data-sha256-function #'foreign-data-sha256
  :byte-vector-sha256-function #'byte-vector-sha256)
 :replace t)

;;; The optional MoE slots.  llambda's accelerator-backend struct has no such
;;; slots yet; until it gains them (make-moe-session-function,
;;; run-moe-function, close-moe-session-function, default nil), a model binds
;;; a layer through this table, consulted at the top of the MoE blocks.
(defvar *cuda-moe-functions*
  (list :make-moe-session-function #'make-cuda-moe-session
        :run-moe-function #'run-cuda-moe-into
        :close-moe-session-function #'close-cuda-moe-session))
