// Host-side launch interface of the CUDA kernels (internal to the library).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace lb {

// Dense GEMV / small-batch GEMM over a raw GGUF tensor:
//   y[t][r] = sum_k W[r][k] * x[t][k]   for r < rows, t < tokens
// x rows hold n_valid values (zero-padded to K); y rows have stride ldy.
cudaError_t launch_gemv(int type, const void* W, size_t row_bytes, int rows, int K,
                        const float* x, long ldx, int n_valid, int tokens, float* y, long ldy,
                        cudaStream_t stream);

// Checks every fp16 scale (d, dmin) of a Q4_K / Q6_K tensor for Inf/NaN,
// which llambda rejects (fp16-to-single-float, llambda.lisp L727-728).
// *bad_count receives the number of offending blocks.
cudaError_t check_fp16_scales(int type, const void* W, size_t blocks, unsigned* bad_count_dev,
                              cudaStream_t stream);

// Synthetic GGUF data straight into device memory (synth.h generator).
cudaError_t synth_fill(int type, uint64_t seed, uint64_t stream_id, uint64_t first,
                       size_t count, float scale, void* out, cudaStream_t stream);

// One MoE feed-forward layer on device-resident tensors.
struct MoeDevice {
  int arch;          // 0 qwen3next, 1 nemotron_h_moe
  int hidden;        // H
  int experts;       // E
  int top_k;
  int weights_norm;
  float weight_scale;
  int inter;         // routed intermediate rows (up_exps ne1)
  int inter_sh;      // shared intermediate rows (0: no shared expert)
  int k_in;          // gate/up row width (>= H, multiple of 256)
  int k_down;        // down row width (>= inter, multiple of 256)
  int k_down_sh;     // shared down row width
  int k_in_sh;       // shared gate/up row width
  int gate_type, up_type, down_type;
  int gate_sh_type, up_sh_type, down_sh_type;
  const float* router;      // [E (+1 for the qwen3next shared gate row)][H]
  const float* router_bias; // [E] or null
  const uint8_t* gate_exps; // null for nemotron
  const uint8_t* up_exps;
  const uint8_t* down_exps;
  const uint8_t* gate_sh;
  const uint8_t* up_sh;
  const uint8_t* down_sh;
  size_t gate_rb, up_rb, down_rb;           // row bytes
  size_t gate_sh_rb, up_sh_rb, down_sh_rb;
  int expert_begin, expert_end;             // experts computed on this device
  int shared_here;                          // compute the shared expert here
  const float* input_norm;                  // rms-norm weight applied to x first, or null
  float norm_epsilon;
  int add_residual;                         // out = x + moe(norm(x))
  // Shared-expert gate row kept apart from `router` (router then has E rows);
  // null when the row is appended to `router` as row E.
  const float* router_extra_row;
};

// Scratch for one layer call with up to max_tokens tokens.
struct MoeWork {
  int max_tokens;
  float* logits;      // [T][E+1]
  int* sel;           // [T][k]
  float* wts;         // [T][k]
  float* shw;         // [T] shared-expert weight
  int* counts;        // [E]
  int* offsets;       // [E+1]
  int* entries;       // [T*k] token*k + rank, grouped by expert
  int* active;        // [E+1] active experts, then count at [E]
  int* status;        // [1] device status word (0 ok; 1 non-positive weight sum)
  float* hbuf;        // [T*k + T][inter_max] expert intermediates
  float* partial;     // [T][k+1][H]
  float* xnorm;       // [T][H] normalised input (when input_norm is set)
  size_t bytes;
};

size_t moe_work_bytes(const MoeDevice& m, int max_tokens);
void moe_work_carve(const MoeDevice& m, int max_tokens, void* base, MoeWork* w);

// out[t][h] for t < tokens; sel/wts optional device outputs [T][k].
cudaError_t launch_moe(const MoeDevice& m, const MoeWork& w, const float* x, int tokens,
                       float* out, cudaStream_t stream);

}  // namespace lb
