// Host-side launch interface of the CUDA kernels (internal to the library).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace lb {

// ------------------------------------------------------------ dense GEMV
//
// Quantized GEMV runs in two launches: the activations are first prepared
// (permuted to the weight type's task layout, sub-block sums for Q4_K) into
// a scratch buffer of xprep_floats(K, tokens) floats, then the TMA-staged
// GEMV reads them.  y[t][r] = sum_k W[r][k] * x[t][k], x zero-padded from
// n_valid to K.

// Work decomposition of one pass over a matrix: units of rl * (32/lpr) rows
// (lpr lanes per row), staged through `stages` shared-memory stages per warp.
struct UnitPlan {
  int lpr;          // lanes per row: 8, 16 or 32
  int rl;           // rows per lane
  int stage_bytes;  // bytes of one shared-memory stage
  int stages;       // stages per warp
  int warps;        // warps per CTA
};

// `ranges` matrices (gate and up) share one stage.
UnitPlan plan_units(size_t row_bytes, int tasks, int ranges);
int sm_count();
size_t xprep_floats(int K, int tokens);
// rows: the matrix the prepared input is for (picks the layout).
cudaError_t launch_prep(int type, int rows, const float* x, long ldx, int n_valid, int K,
                        int tokens, const int* gather, float* xp, cudaStream_t stream);
// Q4_K rows times one or two raw input vectors in one launch (the prep fused
// in); false when the shape does not apply (then prep + launch_gemv_prepped).
bool launch_gemv_fused(int type, const void* W, size_t row_bytes, int rows, int K, const float* x,
                       long ldx, int tokens, float* y, long ldy, int* status, cudaStream_t stream,
                       cudaError_t* err);
cudaError_t launch_gemv_prepped(int type, const void* W, size_t row_bytes, int rows, int K,
                                const float* xp, int tokens, float* y, long ldy, int* status,
                                cudaStream_t stream);
// Q5_0 / Q8_0 rows (32-value blocks): x natural layout, no preparation;
// n_valid values per token (zero past them), -1: K.
cudaError_t launch_gemv_q32(int type, const void* W, size_t row_bytes, int rows, int K,
                            const float* x, long ldx, int tokens, float* y, long ldy,
                            cudaStream_t stream, int n_valid = -1);
// Q5_K rows (176-byte super-blocks): x natural layout, no preparation.
cudaError_t launch_gemv_q5k(const void* W, size_t row_bytes, int rows, int K, const float* x,
                            long ldx, int n_valid, int tokens, float* y, long ldy,
                            cudaStream_t stream);
// Any projection type (F32, Q4_K, Q5_K, Q6_K, Q5_0, Q8_0): y[t][r] = W[r] .
// x[t], x [tokens][ldx] with n_valid values per token, zero-extended to K
// (F32 rows need n_valid == K).  xp: scratch of xprep_floats(K, tokens)
// floats (Q4_K / Q6_K); status: the device status word of the staged kernels.
cudaError_t launch_projection(int type, const void* W, size_t row_bytes, int rows, int K,
                              const float* x, long ldx, int n_valid, int tokens, float* y,
                              long ldy, float* xp, int* status, cudaStream_t stream);
// F32 rows (router): x natural layout, no preparation.
cudaError_t launch_gemv_f32(const void* W, int rows, int K, const float* x, long ldx, int tokens,
                            float* y, long ldy, cudaStream_t stream);

// Checks every fp16 scale (d, dmin) of a Q4_K / Q6_K tensor for Inf/NaN,
// which llambda rejects (fp16-to-single-float, llambda.lisp L727-728).
// *bad_count receives the number of offending blocks.
cudaError_t check_fp16_scales(int type, const void* W, size_t blocks, unsigned* bad_count_dev,
                              cudaStream_t stream);

// Synthetic GGUF data straight into device memory (synth.h generator).
cudaError_t synth_fill(int type, uint64_t seed, uint64_t stream_id, uint64_t first,
                       size_t count, float scale, void* out, cudaStream_t stream);

// ------------------------------------------------------------ MoE layer

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
  const float* router;      // [router_rows][H]
  int router_rows;          // E, or E + 1 with the qwen3next shared-gate row appended
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
  // Expert-parallel reduction over peer memory (ep_world > 1): ep_peers is a
  // device array of every rank's copy of one symmetric buffer (ep_layout()),
  // and the combine step sums all ranks' partial outputs itself.
  void* const* ep_peers;
  int ep_rank, ep_world;
  int ep_max_tokens;  // tokens per slot of the buffer (the same on every rank)
  // With shared_here, the shared expert is computed for tokens
  // [T*sh_part/sh_parts, T*(sh_part+1)/sh_parts) only (sh_parts <= 1: all):
  // expert-parallel ranks split its tokens, and the rank sum reunites them.
  int sh_part, sh_parts;
  // Kernel timing only (null otherwise): the expert-parallel combine's CTA 0
  // writes %globaltimer stamps here: start, its pushes done, every peer
  // seen, end.
  unsigned long long* ep_stamps;
  // Nemotron latent projections (latent_dim > 0; ffn_latent_down and
  // ffn_latent_up, llambda.lisp L5845-5855, L5883-5887, L5933-5938): the
  // routed experts run on latent_down . x (latent_dim values; the expert
  // tensors' widths are latent ones), their weighted sum goes through
  // latent_up back to `hidden`, and then the shared expert (on x) is added.
  int latent_dim;
  int lat_down_type, lat_up_type;  // any projection type
  int k_lat_down, k_lat_up;        // row widths (>= hidden, >= latent_dim)
  const uint8_t* lat_down;         // [latent_dim][k_lat_down]
  const uint8_t* lat_up;           // [hidden][k_lat_up]
  size_t lat_down_rb, lat_up_rb;
  // The router logits are already in the workspace (the routed sub-layer of
  // a latent layer): no router stage.
  int logits_ready;
  // Token dispatch across expert-parallel ranks (dx_world > 1, prefill
  // batches): dx_peers is a device array of every rank's copy of one
  // symmetric buffer (dx_layout()), dx_partials a device array of their
  // partial regions, dx_partial_local this rank's (host-readable pointer);
  // each rank passes its own tokens (at most dx_cap per call).
  void* const* dx_peers;
  float* const* dx_partials;
  float* dx_partial_local;
  int dx_rank, dx_world, dx_cap;
};

// Per-rank copy of the token-dispatch buffer:
//   [0, 64)     local: u32 epoch, u32 arrival ticket, u32 entries sent to each rank [8]
//   [64, 128)   u64 dispatch flag per source rank: epoch << 32 | entries it sent here
//   [128, 192)  u64 done flag per rank: epoch << 32 once its rows for this rank landed
//   meta        int2 [world][cap * k]: {expert, the source's partial row}
//   rows        bf16 [world][cap * k][k_in]: the received input rows
//   partial     fp32 [cap][k + 1][hidden]: expert outputs for this rank's tokens
struct DxLayout {
  size_t meta, rows, partial, bytes;
};
__host__ __device__ inline size_t dx_align(size_t v) { return (v + 255) & ~size_t(255); }
__host__ __device__ inline DxLayout dx_layout(int world, int cap, int k, int k_in, int hidden) {
  DxLayout L;
  const size_t entries = (size_t)world * cap * k;
  L.meta = 256;
  L.rows = dx_align(L.meta + entries * 8);
  L.partial = dx_align(L.rows + entries * k_in * 2);
  L.bytes = dx_align(L.partial + (size_t)cap * (k + 1) * hidden * 4);
  return L;
}

// The routed experts of a latent layer as a layer of their own: hidden =
// latent_dim, no norm, residual or shared expert, logits computed before.
MoeDevice latent_routed_view(const MoeDevice& m);

// The tokens [t0, t1) of a T-token call the shared expert is computed for.
__host__ __device__ inline void shared_tokens(const MoeDevice& m, int T, int& t0, int& t1) {
  if (m.sh_parts <= 1) {
    t0 = 0;
    t1 = T;
  } else {
    t0 = (int)((long)T * m.sh_part / m.sh_parts);
    t1 = (int)((long)T * (m.sh_part + 1) / m.sh_parts);
  }
}

// Symmetric buffer of the peer-memory reduction, per rank copy:
//   [0, 512)        per-CTA epoch counters of this rank (local use)
//   [4096, 8192)    flags[rank q][CTA]: the last epoch rank q pushed for the CTA
//   [8192, ...)     slots[parity][rank q][ep_max_tokens][hidden] floats
constexpr int kEpGrid = 128;  // CTAs of the reduction (the same on every rank)
constexpr int kEpMaxWorld = 8;
inline size_t ep_buffer_bytes(int world, int max_tokens, int hidden) {
  return 8192 + (size_t)2 * world * max_tokens * hidden * sizeof(float);
}

// Scratch for one layer call with up to max_tokens tokens.
struct MoeWork {
  int max_tokens;
  float* logits;      // [T][E+1]
  int* sel;           // [T][k]
  float* wts;         // [T][k]
  float* shw;         // [T] shared-expert weight
  int* counts;        // [E]
  int* offsets;       // [E+1]
  int* entries;       // [2*T*k]: per-entry position, then entry ids grouped by expert
  int* active;        // [E+1] active experts, then count at [E]
  int* pass_off;      // [E+1] per active expert: token passes (of the up pass's
                      //  tokens per pass) before it; total at [active count]
  int* pass_off_dn;   // [E+1] the same for the down pass (4 entries per pass)
  int* status;        // [1] device status word (bit 0: non-positive weight sum,
                      //  bit 1: a TMA stage wait timed out)
  int* tickets;       // [1] arrival counter of the top-k launch (zero between
                      //  launches; right after the status word)
  float* xn;          // [T][H] normalised input (when input_norm is set)
  float* xp_up;       // [T] prepared gate/up inputs (stride xp_stride(k_in))
  float* xp_down;     // [T*k + T] prepared down inputs: routed entry ids, then
                      // shared token rows (stride xp_stride(max(k_down, k_down_sh)))
  float* partial;     // [T][k+1][H] unscaled down outputs per (token, rank)
  float* up_part;     // gate/up items split over K: each item's slices' row sums
  int* up_tickets;    // and its arrival ticket
  // Prefill path (carved when max_tokens >= 64, null otherwise):
  uint16_t* pf_xs;    // [T*k + T][k_in] bf16 inputs grouped by expert, then shared rows
  uint16_t* pf_hs;    // [T*k + T][max(k_down, k_down_sh)] bf16 intermediates, same rows
  int* pf_prow;       // [T*k + T] partial-output row of each grouped row
  int4* pf_tiles;     // gate/up tiles [pf_max_up], then down tiles
  int* pf_count;      // [2] tiles of the gate/up and the down pass
  float* pf_rlog;     // [slices][T][E+1] router logits per K slice
  long pf_max_up;
  // Latent layers (m.latent_dim > 0), carved after the routed sub-layer's
  // buffers (which are sized by latent_routed_view(m)):
  float* lat_xr;      // [T][H] rms-normed input (with input_norm)
  float* lat_x;       // [T][L] latent_down . x: the experts' input
  float* lat_y;       // [T][L] the experts' weighted sum
  float* lat_u;       // [T][H] latent_up . lat_y
  float* lat_s1;      // [T][inter_sh] shared up, relu^2 in place
  float* lat_s2;      // [T][H] shared down
  float* lat_xp;      // prepared inputs of the K-quant projections
  size_t bytes;
};

// 2-D tensor maps of the Q4_K gate/up matrices (routed rows this device owns,
// shared rows) for the tensor-core gate/up pass; built once per layer.
struct SlabMaps {
  CUtensorMap gate, up, gate_sh, up_sh;
  long row_base;  // global row (expert_begin * inter) of the routed maps' row 0
  int ready;      // 0: not a Q4_K layer, or nothing to compute here
};
cudaError_t moe_maps_build(const MoeDevice& m, SlabMaps* maps);

size_t moe_work_bytes(const MoeDevice& m, int max_tokens);
void moe_work_carve(const MoeDevice& m, int max_tokens, void* base, MoeWork* w);

// out[t][h] for t < tokens.  maps: from moe_maps_build for this layer, or
// null to build them for this call.
// marks (optional, seven events): [0] before the gate/up pass, [1] after it,
// [2] after the routed down pass, [3] at the start of the layer (before the
// router), [4] before the combine, [5] after it, [6] between the router and
// the top-k launch, for timing those stages.
cudaError_t launch_moe(const MoeDevice& m, const MoeWork& w, const float* x, int tokens,
                       float* out, const SlabMaps* maps, cudaStream_t stream,
                       const cudaEvent_t* marks = nullptr);

// Top-k and weights of T tokens (w.sel, w.wts, w.shw); grouped_ids 1: also
// group the entries by owned expert with their ids, 0: positions only (the
// prefill gather), -1: no grouping (the token dispatch groups what it
// receives).
cudaError_t launch_topk(const MoeDevice& m, const MoeWork& w, int T, int grouped_ids,
                        cudaStream_t stream);
// out = (x +) the rank-ordered weighted sum of w.partial, plus the shared
// expert's row, for T tokens (experts outside [expert_begin, expert_end) add
// nothing).
cudaError_t launch_combine(const MoeDevice& m, const MoeWork& w, int T, const float* x, float* out,
                           cudaStream_t stream);

// Prefill path (prefill.cu): the expert products of batches of at least
// prefill_min_tokens() tokens as tcgen05 bf16 grouped GEMMs.
void set_prefill_min_tokens(int n);
int prefill_min_tokens();
size_t prefill_work_bytes(const MoeDevice& m, int max_tokens, size_t* parts /* [6] */);
long prefill_max_up_tiles(const MoeDevice& m, int max_tokens);
bool prefill_applies(const MoeDevice& m, const MoeWork& w, int T);
// rms-norm (into w.xn) and the fp32 router GEMM of a prefill batch.
cudaError_t launch_prefill_router(const MoeDevice& m, const MoeWork& w, const float* x, int T,
                                  cudaStream_t stream);
// Gather, plan, gate/up and down passes; partial outputs land in w.partial
// as in the decode path.  marks as in launch_moe.
cudaError_t launch_prefill_passes(const MoeDevice& m, const MoeWork& w, const float* x, int T,
                                  cudaStream_t stream, const cudaEvent_t* marks);
// A whole layer call through the token dispatch (m.dx_world > 1): this
// rank's T tokens are routed here, their rows sent to the experts' owners,
// the received rows multiplied by this rank's experts (tcgen05 prefill
// GEMMs) with the results stored back into their source ranks' partial
// buffers, and this rank's tokens combined.
cudaError_t launch_moe_dispatch(const MoeDevice& m, const MoeWork& w, const float* x, int T,
                                float* out, cudaStream_t stream, const cudaEvent_t* marks);

}  // namespace lb
