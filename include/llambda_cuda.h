/*
 * llambda_cuda.h — C ABI of the B200 (sm_100a) accelerator backend for
 * llambda's quantized feed-forward path.
 *
 * This library replaces the ONNX Runtime bridge of jrm-code-project/llambda
 * (native/llambda_npu.h, native/llambda_npu.cpp) for the path that bridge
 * served, and extends it to the routed-MoE blocks that bypass it today.  The
 * conventions are the bridge's own:
 *   - every fallible call returns an int status, 0 on success and -1 on
 *     failure, and leaves a message readable with llambda_cuda_last_error()
 *     (thread-local, like set_error/last_error in llambda_npu.cpp:24,43-49);
 *   - sessions are opaque handles, *result is set to NULL on entry of each
 *     constructor, destroy functions accept NULL;
 *   - inputs and outputs are caller-owned host float buffers (Lisp vectors
 *     pinned with with-pointer-to-vector-data), copied to and from the GPU
 *     inside the call, which returns when the output is written;
 *   - calls on different sessions may run concurrently from different
 *     threads; calls on one session are serialised by the session.
 * There is no CPU fallback inside this library: without a usable CUDA
 * device every session constructor fails, and the host's own fallback logic
 * (call-with-accelerator-runtime-fallback, llambda.lisp L4660-4676) decides
 * what happens next.
 *
 * Tensor data is raw GGUF: GGML type tags 0 (F32), 12 (Q4_K), 14 (Q6_K);
 * ne0 = columns, ne1 = rows, ne2 = experts; rows are contiguous and expert e
 * starts at row e * ne1 (llambda.lisp L3389-3400, L3909-3916, L4951-4971).
 */
#ifndef LLAMBDA_CUDA_H
#define LLAMBDA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#define LLAMBDA_CUDA_API __declspec(dllexport)
#else
#define LLAMBDA_CUDA_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define LLAMBDA_CUDA_TYPE_F32 0
/* 32-value blocks (llambda.lisp L26-27, sizes L2139-2140): projection
 * sessions only, the formats of rows whose width is not a multiple of 256. */
#define LLAMBDA_CUDA_TYPE_Q5_0 6
#define LLAMBDA_CUDA_TYPE_Q8_0 8
#define LLAMBDA_CUDA_TYPE_Q4_K 12
/* Q5_K (176-byte super-blocks, dot-product-with-q5-k-tensor-data L4387-4441):
 * projection sessions and the latent projections of a MoE layer. */
#define LLAMBDA_CUDA_TYPE_Q5_K 13
#define LLAMBDA_CUDA_TYPE_Q6_K 14

typedef struct llambda_cuda_session llambda_cuda_session;
typedef struct llambda_cuda_moe_session llambda_cuda_moe_session;

/* ------------------------------------------------------------------------
 * Runtime identity.  Replace llambda_gpu_probe / llambda_npu_bridge_version /
 * llambda_npu_runtime_version / llambda_npu_last_error / llambda_npu_sha256
 * (native/llambda_npu.h:23-33; llambda_npu.cpp:205-272, 405-420).
 * ---------------------------------------------------------------------- */

/* 1: a compute-capability 10.0 (B200) device is usable; 0: none (message in
 * last_error); -1: the CUDA runtime failed.  Replaces llambda_gpu_probe,
 * llambda_npu.cpp:405-420. */
LLAMBDA_CUDA_API int llambda_cuda_probe(void);

/* Bridge ABI version, part of llambda's projection cache key
 * (llambda_npu_bridge_version, llambda_npu.cpp:218-220; cache key L2976-2993). */
LLAMBDA_CUDA_API const char* llambda_cuda_bridge_version(void);

/* CUDA runtime/driver versions and device name; NULL on failure
 * (llambda_npu_runtime_version, llambda_npu.cpp:205-216). */
LLAMBDA_CUDA_API const char* llambda_cuda_runtime_version(void);

/* Message of the last failed call on this thread (llambda_npu.cpp:222-224). */
LLAMBDA_CUDA_API const char* llambda_cuda_last_error(void);

/* SHA-256 of data as 64 lowercase hex digits plus NUL; output_size >= 65.
 * Replaces llambda_npu_sha256 (llambda_npu.cpp:226-272), which used Windows
 * BCrypt; this is a FIPS 180-4 implementation. */
LLAMBDA_CUDA_API int llambda_cuda_sha256(const void* data, size_t data_size, char* output,
                                         size_t output_size);

/* ------------------------------------------------------------------------
 * Projection sessions: one 2-D (or 3-D expert) GGUF tensor resident on the
 * GPU.  Replace llambda_gpu_session_* (native/llambda_npu.h:49-62).
 * ---------------------------------------------------------------------- */

/* Opens a projection file written by the backend's exporter: the header
 * "LLBCUDA1", then little-endian u32 version (1), u32 type, u64 ne0, ne1,
 * ne2, u64 data bytes, u64 data offset, then the raw GGUF tensor bytes.
 * Replaces llambda_gpu_session_create (llambda_npu.cpp:422-487), which
 * opened an ONNX Gemm graph. */
LLAMBDA_CUDA_API int llambda_cuda_session_create(const char* model_path,
                                                 llambda_cuda_session** result);

/* Uploads a tensor straight from memory (for example the GGUF mapping at a
 * tensor's data offset).  data_size must equal ne2 * ne1 * row bytes.
 * Q4_K/Q6_K need ne0 % 256 == 0 (ggml-tensor-byte-size, L2147-2155); fp16
 * scales that are Inf/NaN are rejected here (fp16-to-single-float raises
 * on them at run time, L727-728). */
LLAMBDA_CUDA_API int llambda_cuda_session_create_from_tensor(int type, uint64_t ne0, uint64_t ne1,
                                                             uint64_t ne2, const void* data,
                                                             size_t data_size,
                                                             llambda_cuda_session** result);

/* As above, but `device_data` already lives in this process's current CUDA
 * device memory; the session borrows it (the caller keeps it alive and frees
 * it after llambda_cuda_session_destroy). */
LLAMBDA_CUDA_API int llambda_cuda_session_create_device(int type, uint64_t ne0, uint64_t ne1,
                                                        uint64_t ne2, const void* device_data,
                                                        llambda_cuda_session** result);

LLAMBDA_CUDA_API void llambda_cuda_session_destroy(llambda_cuda_session* session);

/* ne0 (input) and ne1 (output) of the session's tensor; 0 for NULL
 * (llambda_gpu_session_input/output_element_count, llambda_npu.cpp:494-501). */
LLAMBDA_CUDA_API size_t llambda_cuda_session_input_element_count(const llambda_cuda_session* s);
LLAMBDA_CUDA_API size_t llambda_cuda_session_output_element_count(const llambda_cuda_session* s);

/* output[r] = row r . input, r < ne1, on expert 0.  Counts must match the
 * tensor (llambda_gpu_session_run, llambda_npu.cpp:503-537). */
LLAMBDA_CUDA_API int llambda_cuda_session_run(llambda_cuda_session* session, const float* input,
                                              size_t input_element_count, float* output,
                                              size_t output_element_count);

/* `tokens` input vectors (row-major [tokens][ne0]) -> [tokens][ne1] in one
 * pass over the weights. */
LLAMBDA_CUDA_API int llambda_cuda_session_run_batch(llambda_cuda_session* session,
                                                    const float* input, size_t tokens,
                                                    float* output);

/* Rows [expert*ne1, (expert+1)*ne1) of a 3-D expert tensor
 * (gguf-model-expert-matrix-vector-multiply-into, llambda.lisp L4951-4971). */
LLAMBDA_CUDA_API int llambda_cuda_session_run_expert(llambda_cuda_session* session, int expert,
                                                     const float* input,
                                                     size_t input_element_count, float* output,
                                                     size_t output_element_count);

/* Device-memory form for callers that keep activations on the GPU: input
 * [tokens][ne0] and output [tokens][ne1] in device memory, enqueued on
 * `cuda_stream` (a cudaStream_t, NULL = legacy default stream), no sync. */
LLAMBDA_CUDA_API int llambda_cuda_session_run_device(llambda_cuda_session* session,
                                                     const float* device_input, size_t tokens,
                                                     float* device_output, void* cuda_stream);

/* ------------------------------------------------------------------------
 * MoE sessions: one routed feed-forward layer (qwen3next-moe-into,
 * llambda.lisp L5321-5426; nemotron-h-moe-ffn-into, L5827-5949).  llambda's
 * descriptor protocol has no slot for these today; they back the optional
 * :make-moe-session-function / :run-moe-function descriptor slots.
 * ---------------------------------------------------------------------- */

#define LLAMBDA_CUDA_ARCH_QWEN3NEXT 0
#define LLAMBDA_CUDA_ARCH_NEMOTRON_H_MOE 1

typedef struct {
  int type;          /* GGML type tag */
  uint64_t ne0, ne1, ne2;
  const void* data;  /* host memory (copied) or device memory (borrowed) */
} llambda_cuda_tensor;

typedef struct {
  int arch;                 /* LLAMBDA_CUDA_ARCH_* */
  uint64_t hidden;          /* length of the token vectors */
  int top_k;                /* expert_used_count (min'd with the expert count) */
  float weight_scale;       /* nemotron expert_weights_scale (1.0 if absent) */
  int weights_norm;         /* nemotron expert_weights_norm */
  int data_on_device;       /* 1: every data pointer below is device memory */
  llambda_cuda_tensor router;          /* ffn_gate_inp: F32, ne0 = hidden, ne1 = experts */
  const float* router_bias;            /* nemotron exp_probs_b.bias [experts] or NULL */
  const float* shared_gate_inp;        /* qwen3next ffn_gate_inp_shexp [hidden] */
  llambda_cuda_tensor gate_exps;       /* qwen3next only */
  llambda_cuda_tensor up_exps;
  llambda_cuda_tensor down_exps;
  llambda_cuda_tensor gate_shexp;      /* qwen3next only */
  llambda_cuda_tensor up_shexp;        /* data NULL: no shared expert */
  llambda_cuda_tensor down_shexp;
  int expert_begin, expert_end;        /* experts owned by this process;
                                          0,0 = all */
  int shared_here;                     /* compute the shared expert here (1) */
  int max_tokens;                      /* largest batch a run may pass */
  const float* input_norm;             /* optional rms-norm weight [hidden] applied to x
                                          first (post_attention_norm, L5739-5744) */
  float norm_epsilon;                  /* its epsilon (rms-norm-into, L859-879) */
  int add_residual;                    /* 1: out = x + MoE(...) (vector-add-into, L5746) */
  /* nemotron_h_moe latent projections (ffn_latent_down / ffn_latent_up,
   * nemotron-h-moe-ffn-into L5845-5855, L5883-5887, L5933-5938), both or
   * neither (data NULL): latent_down (ne0 >= hidden, ne1 = latent size L)
   * maps the input to the experts' input, the expert tensors then have
   * latent widths (up rows >= L wide, down ne1 = L), and latent_up (ne0 >= L,
   * ne1 = hidden) maps the experts' weighted sum back before the shared
   * expert, which sees the input itself, is added.  Any projection type:
   * F32, Q4_K, Q5_K, Q6_K, Q5_0, Q8_0.  Sessions only (not the
   * static-scratch call), on one device (no peer attachment). */
  llambda_cuda_tensor latent_down;
  llambda_cuda_tensor latent_up;
} llambda_cuda_moe_desc;

/* Gate/up rows may be wider than `hidden` and down rows wider than the
 * intermediate size when they are zero-padded to a multiple of 256 columns;
 * the inputs are zero-extended to match. */
LLAMBDA_CUDA_API int llambda_cuda_moe_session_create(const llambda_cuda_moe_desc* desc,
                                                     llambda_cuda_moe_session** result);
LLAMBDA_CUDA_API void llambda_cuda_moe_session_destroy(llambda_cuda_moe_session* session);
LLAMBDA_CUDA_API size_t llambda_cuda_moe_session_hidden(const llambda_cuda_moe_session* session);

/* out[t] = MoE(x[t]) for t < tokens (host buffers [tokens][hidden]).
 * selected / weights (optional, [tokens][top_k]) receive the chosen experts
 * in rank order and their final weights.  Fails like the reference when the
 * top-k weight sum is not positive (L5373-5375, L5903-5905). */
LLAMBDA_CUDA_API int llambda_cuda_moe_session_run(llambda_cuda_moe_session* session,
                                                  const float* x, size_t tokens, float* out,
                                                  int32_t* selected, float* weights);

/* Device-memory form: x, out (and optional selected/weights) in device
 * memory, enqueued on `cuda_stream`, no synchronisation, no status check
 * (read it with llambda_cuda_moe_session_status after synchronising). */
LLAMBDA_CUDA_API int llambda_cuda_moe_session_run_device(llambda_cuda_moe_session* session,
                                                         const float* device_x, size_t tokens,
                                                         float* device_out,
                                                         int32_t* device_selected,
                                                         float* device_weights,
                                                         void* cuda_stream);

/* Status word of the device-side checks of the last runs (0 = ok; 1 = a
 * token's top-k weight sum was not positive); reading it clears it.  -1 on
 * a CUDA error. */
LLAMBDA_CUDA_API int llambda_cuda_moe_session_status(llambda_cuda_moe_session* session);

/* Kernel timing (a measurement aid with no counterpart in the reference):
 * with enable != 0 every later run records CUDA events around the gate/up
 * pass and the routed down pass on the run's stream;
 * llambda_cuda_moe_session_kernel_ms waits for the last run's events and
 * returns the two durations in milliseconds.  0 on success, -1 on failure. */
LLAMBDA_CUDA_API int llambda_cuda_moe_session_time_kernels(llambda_cuda_moe_session* session,
                                                           int enable);
LLAMBDA_CUDA_API int llambda_cuda_moe_session_kernel_ms(llambda_cuda_moe_session* session,
                                                        float* gate_up_ms, float* down_ms);
/* The stages of the last timed run, in milliseconds, into ms[0..n): router,
 * top-k with the routing, gate/up pass, routed down pass, shared down pass,
 * combine (with the expert-parallel exchange); with n >= 9 on a session
 * attached to peers also the combine's phases as its first CTA saw them
 * (pushing its partial, waiting for every rank's, summing).  Returns the
 * number written (6 or 9), -1 on failure.  No counterpart in the reference
 * (a measurement aid). */
LLAMBDA_CUDA_API int llambda_cuda_moe_session_kernel_breakdown(llambda_cuda_moe_session* session,
                                                               float* ms, int n);

/* GGUF files (replaces the ONNX export/cache of the reference's bridge,
 * llambda.lisp L402-476 / L2976-3067, with the raw blocks themselves).
 * llambda_cuda_gguf_open maps and parses a file as the reference loader does
 * (read-gguf-header, L2049-2062; read-gguf-metadata-section, L2064-2084;
 * read-gguf-tensor-infos, L2157-2238: 1..4 positive dimensions, the data
 * start aligned to general.alignment, default 32, a power of two, every
 * tensor inside the file); 0 on success, -1 with last_error otherwise, *out
 * nulled on entry.  Tensor infos give the type tag, dimensions (ne[4],
 * unused ones 1), byte size (0 for types the loader does not size) and a host
 * pointer into the mapping, valid until llambda_cuda_gguf_close.
 * llambda_cuda_gguf_upload copies the chosen tensors into one device arena
 * (each 256-byte aligned) and returns its pointer and each tensor's device
 * pointer, for projection sessions (llambda_cuda_session_create_device) and
 * MoE descriptors (data_on_device = 1); free it with llambda_cuda_device_free
 * after the sessions that use it. */
typedef struct llambda_cuda_gguf llambda_cuda_gguf;
LLAMBDA_CUDA_API int llambda_cuda_gguf_open(const char* path, llambda_cuda_gguf** out);
LLAMBDA_CUDA_API void llambda_cuda_gguf_close(llambda_cuda_gguf* gguf);
LLAMBDA_CUDA_API uint64_t llambda_cuda_gguf_tensor_count(const llambda_cuda_gguf* gguf);
/* Index of the tensor named `name`, -1 if there is none. */
LLAMBDA_CUDA_API int64_t llambda_cuda_gguf_find(const llambda_cuda_gguf* gguf, const char* name);
LLAMBDA_CUDA_API int llambda_cuda_gguf_tensor_info(const llambda_cuda_gguf* gguf, uint64_t index,
                                                   char* name_out, size_t name_capacity,
                                                   int* type, uint32_t* n_dims, uint64_t* ne,
                                                   uint64_t* byte_size, const void** host_data);
LLAMBDA_CUDA_API int llambda_cuda_gguf_upload(const llambda_cuda_gguf* gguf,
                                              const uint64_t* indices, size_t count,
                                              void** device_arena, void** device_ptrs);
LLAMBDA_CUDA_API int llambda_cuda_device_free(void* device_ptr);

/* Prefill path (a tuning knob with no counterpart in the reference; the
 * reference runs every token through the same per-token code,
 * qwen3next-moe-into L5321-5426 / nemotron-h-moe-ffn-into L5827-5949).
 * MoE runs of at least `tokens` tokens (default 128; values below 64 act as
 * 64) compute the expert products as bf16 grouped GEMMs on the tensor cores:
 * weights decoded once per 128-row block and 64 tokens, inputs and the
 * gate/up activations rounded to bf16, fp32 sums (results within 2e-2
 * relative of the fp32 path).  Smaller runs use the fp32 decode kernels.
 * Process-wide; later runs use the new value.  0 on success, -1 on a
 * non-positive value. */
LLAMBDA_CUDA_API int llambda_cuda_set_prefill_min_tokens(int tokens);
LLAMBDA_CUDA_API int llambda_cuda_prefill_min_tokens(void);

/* Expert-parallel reduction over peer memory.  These entry points have no
 * counterpart in the reference (llambda runs on one device).
 *
 * Bytes of the symmetric device buffer that `world` expert-parallel ranks of
 * this session need (0 on a bad argument). */
LLAMBDA_CUDA_API size_t llambda_cuda_moe_peer_bytes(const llambda_cuda_moe_session* session,
                                                    int world);

/* After this call every run of the session sums the partial outputs of all
 * `world` ranks itself (each rank owning a range of experts,
 * expert_begin/expert_end), so every rank ends with the whole layer output
 * (plus the residual when add_residual is set, on every rank) and no
 * all-reduce follows.  A rank created with shared_here computes the shared
 * expert for its part [T*rank/world, T*(rank+1)/world) of the tokens only.  peer_buffers[r] is rank r's copy of one symmetric
 * device buffer of `bytes` bytes (>= llambda_cuda_moe_peer_bytes), mapped
 * into this process, 16-byte aligned and zero-filled before the first run;
 * every session of a stack may share it.  Every rank must then run the same
 * sessions in the same order.  A rank that waits more than two seconds for a
 * peer sets bit 2 (value 4) of the session status. */
LLAMBDA_CUDA_API int llambda_cuda_moe_session_attach_peers(llambda_cuda_moe_session* session,
                                                           int rank, int world,
                                                           void* const* peer_buffers,
                                                           size_t bytes);

/* Expert-parallel prefill by token dispatch.  These entry points have no
 * counterpart in the reference (llambda runs every token through one device).
 *
 * Bytes of the symmetric device buffer that `world` ranks need when each
 * passes at most `max_local_tokens` tokens per call (0 on a bad argument). */
LLAMBDA_CUDA_API size_t llambda_cuda_moe_dispatch_bytes(const llambda_cuda_moe_session* session,
                                                        int world, int max_local_tokens);

/* After this call, runs of at least llambda_cuda_prefill_min_tokens()
 * tokens take the token dispatch: every rank passes ITS OWN tokens (x and
 * out hold that rank's rows only, at most max_local_tokens of them), each
 * token's row travels over NVLink peer memory to the ranks owning its
 * selected experts, those ranks multiply it on the tensor cores (the bf16
 * prefill GEMMs) and store the result rows back into the source rank's
 * buffer, and each rank combines its own tokens (weights, shared expert,
 * residual) as one device would.  Rank r must own experts [r*E/world,
 * (r+1)*E/world) with shared_here = 1, world * max_local_tokens must not
 * exceed the session's max_tokens, and every rank must run the same sessions
 * in the same order.  peer_buffers[r] is rank r's copy of one symmetric
 * buffer of `bytes` bytes (>= llambda_cuda_moe_dispatch_bytes), mapped into
 * this process, 256-byte aligned and zero-filled before the first run; the
 * sessions of a stack may share it.  Smaller runs keep the decode path and
 * need the peer reduction (llambda_cuda_moe_session_attach_peers).  A rank
 * that waits more than two seconds for a peer sets bit 2 (value 4) of the
 * session status. */
LLAMBDA_CUDA_API int llambda_cuda_moe_session_attach_dispatch(llambda_cuda_moe_session* session,
                                                              int rank, int world,
                                                              void* const* peer_buffers,
                                                              size_t bytes, int max_local_tokens);

/* One MoE layer without any device allocation.  This entry point has no
 * counterpart in the reference.
 *
 * It is for callers that cannot call cudaMalloc: a host whose device memory
 * is already claimed by its own pooling allocator (so a cudaMalloc would
 * fail or fragment the pool), or a latency-critical decode loop that must not
 * pay for cudaMalloc/cudaFree and the device-wide synchronisation they can
 * cause.  Such callers keep every tensor in device memory themselves and pass
 * it here: `desc` must have data_on_device = 1 (weights, router, bias, norm
 * and the qwen3next shared-gate vector all in device memory, expert tensors
 * starting at expert 0), `device_x` and `device_out` are [tokens][hidden]
 * device arrays, and nothing is uploaded or copied into owned buffers.
 *
 * Working memory comes from one static device array of
 * LLAMBDA_CUDA_STATIC_SCRATCH_BYTES (16 MiB) that every GPU loading this
 * library holds until the process exits.  A call whose working set (it grows
 * with tokens, top_k, the expert intermediate size and hidden) does not fit
 * fails with a message naming the limit.  All calls share the array and it
 * keeps the previous call's contents: the call clears what must start at
 * zero, but two calls that overlap on the GPU (different streams, threads or
 * devices sharing a context) race on it, so serialise them.
 *
 * The first call on each device checks that the device is sm_100 and looks
 * up the array's device address with that device current; make that first
 * call before any stream capture.  Every call enqueues on `cuda_stream`, then
 * waits for that stream before it returns, also when it fails part-way (so
 * no kernel of a failed call still writes the array afterwards), and
 * returns -1 (message in last_error) when a token's top-k weight sum is not
 * positive, like llambda_cuda_moe_session_run.  Batches of at least
 * llambda_cuda_prefill_min_tokens() tokens take the bf16 prefill path here
 * too, as long as their working set fits the array.  Inf/NaN fp16 scales are
 * not checked here (sessions check them at creation). */
#define LLAMBDA_CUDA_STATIC_SCRATCH_BYTES (16u << 20)
LLAMBDA_CUDA_API int llambda_cuda_moe_forward_static_scratch(const llambda_cuda_moe_desc* desc,
                                                             const float* device_x,
                                                             size_t tokens, float* device_out,
                                                             void* cuda_stream);

/* ------------------------------------------------------------------------
 * Synthetic GGUF data for benchmarks and tests (seeded, counter-based; the
 * same generator runs on the host in the test oracle, byte for byte).
 * type: Q4_K / Q6_K write `count` super-blocks starting at block `first`;
 * F32 writes `count` floats ~ N(0, scale).  `scale` is the dscale of
 * fp16(|N(0,1)| * dscale) for the block types.
 * ---------------------------------------------------------------------- */
LLAMBDA_CUDA_API int llambda_cuda_synth_fill_device(int type, uint64_t seed, uint64_t stream_id,
                                                    uint64_t first, size_t count, float scale,
                                                    void* device_out, void* cuda_stream);

#ifdef __cplusplus
}
#endif

#endif /* LLAMBDA_CUDA_H */
