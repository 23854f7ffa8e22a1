// Dense dequant-fused GEMV for raw GGUF Q4_K / Q6_K tensors (warp TMA
// pipeline, engine.cuh), the F32 GEMV of the MoE router, the activation
// preparation kernel, the fp16 scale validator and the synthetic-data fill.
//
// Replaces %gguf-model-matrix-vector-multiply-into (llambda.lisp L4542-4658),
// which splits rows over lparallel workers and runs an 8-lane AVX2 loop per
// row.
#include <algorithm>
#include <map>
#include <mutex>

#include "engine.cuh"
#include "kernels.h"
#include "mma.cuh"
#include "synth.h"

namespace lb {

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

int kernel_occupancy(const void* kernel, int threads, size_t smem) {
  static std::mutex mu;
  static std::map<std::pair<const void*, size_t>, int> cache;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(kernel, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  // opt in to what this launch needs (at least 200 KB; at most the 227 KB a
  // CTA may use)
  const int optin = (int)std::min<size_t>(std::max<size_t>(smem, 200 * 1024), 227 * 1024);
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin) !=
      cudaSuccess)
    return -1;
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, threads, smem) != cudaSuccess)
    return -1;
  cache[key] = occ;
  return occ;
}

UnitPlan plan_units(size_t rb, int tasks, int ranges) {
  UnitPlan p{};
  p.lpr = lanes_for(tasks);
  p.rl = 4;
  while (p.rl > 1 && (size_t)p.rl * (32 / p.lpr) * rb * ranges > 7 * 1024) p.rl /= 2;
  const size_t ru = (size_t)p.rl * (32 / p.lpr);
  p.stage_bytes = (int)(((size_t)ranges * (ru * rb + 32) + 127) & ~size_t(127));
  p.stages = std::max(2, std::min(4, (16 * 1024) / p.stage_bytes));
  p.warps = 4;
  return p;
}

namespace {

// ------------------------------------------------------------ preparation

// One block per (256-value super-block, token): 64 threads, one float4 each.
template <int TYPE>
__global__ void __launch_bounds__(64) prep_kernel(const float* __restrict__ x, long ldx,
                                                  int n_valid, int K, const int* __restrict__ gather,
                                                  float* __restrict__ xp) {
  const int sb = blockIdx.x, tok = blockIdx.y;
  const int tasks = K >> 6;
  const long row = gather ? gather[tok] : tok;
  const float* s = x + row * ldx;
  const int e = sb * 256 + threadIdx.x * 4;
  float4 v;
  if (e + 3 < n_valid && (reinterpret_cast<uintptr_t>(s + e) & 15u) == 0) {
    v = *reinterpret_cast<const float4*>(s + e);
  } else {
    v.x = e < n_valid ? s[e] : 0.f;
    v.y = e + 1 < n_valid ? s[e + 1] : 0.f;
    v.z = e + 2 < n_valid ? s[e + 2] : 0.f;
    v.w = e + 3 < n_valid ? s[e + 3] : 0.f;
  }
  if (TYPE == LB_TYPE_Q4_K) {  // tensor-core layout (mma.cuh)
    mx_store4(reinterpret_cast<uint8_t*>(xp) + (size_t)tok * mx_bytes(K), K, e, v);
  } else {
    float* out = xp + (long)tok * xp_stride(K);
    *reinterpret_cast<float4*>(out + xp_index<TYPE>(e, tasks)) = v;
  }
}

// The Q6_K tensor-core layouts (mma.cuh, "m6", or "i6" with SLOT) of token
// rows: one block per (super-block, token), two warps storing 8 of its 16
// sub-blocks each.
template <bool SLOT>
__global__ void __launch_bounds__(64) m6_prep_kernel(const float* __restrict__ x, long ldx,
                                                     int n_valid, int K,
                                                     const int* __restrict__ gather,
                                                     uint8_t* __restrict__ m6) {
  const int sb = blockIdx.x, tok = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  griddep_wait();  // x is the kernel before's output; m6 may still be its input
  griddep_launch();
  const long row = gather ? gather[tok] : tok;
  const float* s = x + row * ldx;
  uint8_t* dst = m6 + (size_t)tok * m6_bytes(K);
  const int g = lane >> 2;
  for (int j = 0; j < 8; ++j) {
    const int sub = warp * 8 + j;
    const int e0 = sb * 256 + sub * 16;
    float va = 0.f, vb = 0.f;
    if ((lane & 3) == 0) {
      va = e0 + g < n_valid ? s[e0 + g] : 0.f;
      vb = e0 + g + 8 < n_valid ? s[e0 + g + 8] : 0.f;
    }
    if (SLOT)
      i6_store_subblock(dst, sb * 16 + sub, va, vb, lane);
    else
      m6_store_subblock(dst, sb * 16 + sub, va, vb, lane);
  }
}

// ------------------------------------------------------------ dense GEMV

// Q6_K rows on the tensor cores (mma.cuh): a unit is a 16-row block with its
// whole K (16 rows x row bytes, one aligned bulk copy), staged by warp CW
// through full/empty mbarriers; consumer warp w takes super-blocks
// [w*nsb/CW, (w+1)*nsb/CW) of every block, and warp 0 adds the other warps'
// sums (in warp order) and writes the rows.  NG groups of 4 tokens share the
// decoded weights; the tokens' prepared inputs (m6) are read through L1.
// SLOT: one or two tokens (NG of them) in the sub-block slot form (i6).
struct DenseSync {
  uint64_t full[8], empty[8], red[8];
  int abort;
  int pad[3];
};

template <int NG, int CW, bool SLOT>
__global__ void __launch_bounds__((CW + 1) * 32, 1)
    gemv_q6k_slab_kernel(const uint8_t* __restrict__ W, size_t rb, int rows, int nsb,
                         const uint8_t* __restrict__ m6, int tokens, float* __restrict__ y,
                         long ldy, int stages, int stage_bytes, int* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  DenseSync* sync = reinterpret_cast<DenseSync*>(smem + (size_t)stages * stage_bytes);
  float2* red = reinterpret_cast<float2*>(sync + 1);  // [stages][CW][32][NG]
  volatile int* abort = &sync->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&sync->full[s], 1);
      mbar_init(&sync->empty[s], CW);
      mbar_init(&sync->red[s], CW - 1);
    }
    sync->abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const int units = rows / kTileRows;  // rows % 16 == 0
  const int u0 = (int)((long)blockIdx.x * units / gridDim.x);
  const int n_my = (int)((long)(blockIdx.x + 1) * units / gridDim.x) - u0;
  const uint32_t block_bytes = (uint32_t)(kTileRows * rb);
  if (warp == CW) {  // ---------------- producer
    if (lane == 0) {
      RingPos rp;
      int q = 0;
      for (int i = 0; i < n_my; ++i, ++q, rp.next(stages)) {
        if (q >= stages && !mbar_wait_or_abort(&sync->empty[rp.s], rp.phase ^ 1u, status, abort))
          break;
        mbar_expect_tx(&sync->full[rp.s], block_bytes);
        tma_load_1d(smem + (size_t)rp.s * stage_bytes, W + (size_t)(u0 + i) * block_bytes,
                    block_bytes, &sync->full[rp.s]);
      }
      for (int r = max(0, q - stages); r < q; ++r)
        mbar_wait(&sync->full[r % stages], (r / stages) & 1, nullptr);
    }
    return;
  }
  // consumers: the prepared input is the kernel before's output (the
  // producer's weight copies above need no wait)
  griddep_wait();
  griddep_launch();
  const int sb0 = warp * nsb / CW, sb1 = (warp + 1) * nsb / CW;
  const int g = lane >> 2, t = lane & 3;
  const size_t m6b = m6_bytes(nsb * 256);
  const uint8_t* m6p[4 * NG];
#pragma unroll
  for (int n = 0; n < 4 * NG; ++n) m6p[n] = m6 + (size_t)min(n, tokens - 1) * m6b;
  RingPos rp;
  for (int i = 0; i < n_my; ++i, rp.next(stages)) {
    const int s = rp.s;
    if (!mbar_wait_or_abort(&sync->full[s], rp.phase, status, abort)) break;
    const uint8_t* blk = smem + (size_t)s * stage_bytes;
    float2 acc[NG];
#pragma unroll
    for (int grp = 0; grp < NG; ++grp) acc[grp] = make_float2(0.f, 0.f);
    if (SLOT) {
      q6i_block<false, NG>(blk, rb, sb0, sb1, m6p, kZero32, lane, 0, acc[0]);
    } else {
      for (int sb = sb0; sb < sb1; ++sb)
        q6k_sb_mma<false, NG>(blk + g * rb + sb * LB_Q6K, blk + (g + 8) * rb + sb * LB_Q6K, sb,
                              m6p, tokens, lane, acc);
    }
    float2* rs = red + (size_t)s * CW * 32 * NG;
    if (warp != 0) {
#pragma unroll
      for (int grp = 0; grp < NG; ++grp) rs[(warp * 32 + lane) * NG + grp] = acc[grp];
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sync->red[s]);
        mbar_arrive(&sync->empty[s]);
      }
    } else {
      if (!mbar_wait_or_abort(&sync->red[s], rp.phase, status, abort)) break;
      for (int w2 = 1; w2 < CW; ++w2)
#pragma unroll
        for (int grp = 0; grp < NG; ++grp) {
          const float2 o = rs[(w2 * 32 + lane) * NG + grp];
          acc[grp].x += o.x;
          acc[grp].y += o.y;
        }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sync->empty[s]);
      const int row = (u0 + i) * kTileRows + g;
#pragma unroll
      for (int grp = 0; grp < (SLOT ? 1 : NG); ++grp) {
        const int n = 4 * grp + t;
        if (n < tokens) {
          y[(long)n * ldy + row] = acc[grp].x;
          y[(long)n * ldy + row + 8] = acc[grp].y;
        }
      }
    }
  }
}

// Q6_K rows times 3..8 tokens (m6 layout) with the tokens' inputs resident
// in shared memory.  K is cut into slices of 8 super-blocks (1680-byte row
// pieces, 16-byte aligned); CTA c keeps slice c % slices of every token's
// input (tokens x 9216 bytes, loaded once) and streams that slice of a run of
// 16-row blocks, one block per stage by 16 row copies.  Consumer warp w takes
// super-block w of the slice; warp 0 adds the others' sums (in warp order).
// With two slices the halves meet in y (zeroed first) by atomic adds, whose
// two-term sum is the same in either order.
constexpr int kSliceSb = 8;
struct SliceSync {
  uint64_t full[8], empty[8], red[8], act;
  int abort;
  int pad[3];
};

template <int NG>
__global__ void __launch_bounds__((kSliceSb + 1) * 32, 1)
    gemv_q6k_slice_kernel(const uint8_t* __restrict__ W, size_t rb, int rows, int slices,
                          const uint8_t* __restrict__ m6, int tokens, float* __restrict__ y,
                          long ldy, int stages, int* status) {
  constexpr int CW = kSliceSb;
  constexpr uint32_t kPiece = kSliceSb * LB_Q6K;  // 1680 bytes of a row
  constexpr uint32_t kStage = kTileRows * kPiece;
  constexpr uint32_t kActTok = kSliceSb * 1152;
  constexpr uint32_t kActPitch = kActTok + 16;  // tokens 4 banks apart (meta loads)
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* act = smem + (size_t)stages * kStage;  // [tokens][kActPitch]
  SliceSync* sync = reinterpret_cast<SliceSync*>(act + (size_t)4 * NG * kActPitch);
  float2* red = reinterpret_cast<float2*>(sync + 1);  // [stages][CW][32][NG]
  volatile int* abort = &sync->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&sync->full[s], 1);
      mbar_init(&sync->empty[s], CW);
      mbar_init(&sync->red[s], CW - 1);
    }
    mbar_init(&sync->act, 1);
    sync->abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const int slice = blockIdx.x % slices, ctas = gridDim.x / slices, cta = blockIdx.x / slices;
  const int units = rows / kTileRows;  // rows % 16 == 0
  const int u0 = (int)((long)cta * units / ctas);
  const int n_my = cta < ctas ? (int)((long)(cta + 1) * units / ctas) - u0 : 0;
  const size_t m6b = m6_bytes((int)(rb / LB_Q6K) * 256);
  if (warp == CW) {  // ---------------- producer
    if (lane == 0) {
      mbar_expect_tx(&sync->act, (uint32_t)tokens * kActTok);
      for (int n = 0; n < tokens; ++n)
        tma_load_1d(act + (size_t)n * kActPitch, m6 + n * m6b + (size_t)slice * kActTok, kActTok,
                    &sync->act);
    }
    RingPos rp;
    int q = 0;
    for (int i = 0; i < n_my; ++i, ++q, rp.next(stages)) {
      bool ok = true;
      if (lane == 0 && q >= stages)
        ok = mbar_wait_or_abort(&sync->empty[rp.s], rp.phase ^ 1u, status, abort);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      if (lane == 0) mbar_expect_tx(&sync->full[rp.s], kStage);
      __syncwarp();
      if (lane < kTileRows)  // one row piece per lane
        tma_load_1d(smem + (size_t)rp.s * kStage + lane * kPiece,
                    W + ((size_t)(u0 + i) * kTileRows + lane) * rb + (size_t)slice * kPiece,
                    kPiece, &sync->full[rp.s]);
    }
    if (lane == 0) {
      for (int r = max(0, q - stages); r < q; ++r)
        mbar_wait(&sync->full[r % stages], (r / stages) & 1, nullptr);
      mbar_wait(&sync->act, 0, nullptr);
    }
    return;
  }
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* m6p[4 * NG];
#pragma unroll
  for (int n = 0; n < 4 * NG; ++n) m6p[n] = act + (size_t)min(n, tokens - 1) * kActPitch;
  if (!mbar_wait_or_abort(&sync->act, 0, status, abort)) return;
  RingPos rp;
  for (int i = 0; i < n_my; ++i, rp.next(stages)) {
    const int s = rp.s;
    if (!mbar_wait_or_abort(&sync->full[s], rp.phase, status, abort)) break;
    const uint8_t* blk = smem + (size_t)s * kStage;
    float2 acc[NG];
#pragma unroll
    for (int grp = 0; grp < NG; ++grp) acc[grp] = make_float2(0.f, 0.f);
    q6k_sb_mma<true, NG>(blk + g * kPiece + warp * LB_Q6K, blk + (g + 8) * kPiece + warp * LB_Q6K,
                         warp, m6p, tokens, lane, acc);
    float2* rs = red + (size_t)s * CW * 32 * NG;
    if (warp != 0) {
#pragma unroll
      for (int grp = 0; grp < NG; ++grp) rs[(warp * 32 + lane) * NG + grp] = acc[grp];
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sync->red[s]);
        mbar_arrive(&sync->empty[s]);
      }
    } else {
      if (!mbar_wait_or_abort(&sync->red[s], rp.phase, status, abort)) break;
      for (int w2 = 1; w2 < CW; ++w2)
#pragma unroll
        for (int grp = 0; grp < NG; ++grp) {
          const float2 o = rs[(w2 * 32 + lane) * NG + grp];
          acc[grp].x += o.x;
          acc[grp].y += o.y;
        }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sync->empty[s]);
      const int row = (u0 + i) * kTileRows + g;
#pragma unroll
      for (int grp = 0; grp < NG; ++grp) {
        const int n = 4 * grp + t;
        if (n < tokens) {
          float* o = y + (long)n * ldy + row;
          if (slices > 1) {
            atomicAdd(o, acc[grp].x);
            atomicAdd(o + 8, acc[grp].y);
          } else {
            o[0] = acc[grp].x;
            o[8] = acc[grp].y;
          }
        }
      }
    }
  }
}

// Each warp owns a contiguous run of units (RU rows each), streams them
// through its TMA ring and computes every token against each staged unit.
template <int TYPE, int LPR, int RL>
__global__ void __launch_bounds__(128) gemv_kernel(const uint8_t* __restrict__ W, size_t rb,
                                                   int rows, int tasks,
                                                   const float* __restrict__ xp, int tokens,
                                                   float* __restrict__ y, long ldy, int stages,
                                                   int stage_bytes, int* status) {
  constexpr int RPP = 32 / LPR, RU = RL * RPP;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)nwarps * stages * stage_bytes);
  const WarpRing ring{smem + (size_t)warp * stages * stage_bytes, bars + warp * stages,
                      stage_bytes, stages};
  ring_init(ring, lane);
  const long xld = xp_stride(tasks * 64);
  const int units = (rows + RU - 1) / RU;
  const int gw = blockIdx.x * nwarps + warp, total = gridDim.x * nwarps;
  const int chunk = (units + total - 1) / total;
  const int u0 = gw * chunk;
  const int n_my = max(0, min(units, u0 + chunk) - u0);
  auto issue = [&](int idx) {
    const int row0 = (u0 + idx) * RU;
    ring_issue(ring, idx % stages, W + (size_t)row0 * rb, (size_t)min(RU, rows - row0) * rb,
               nullptr, 0);
  };
  int issued = 0;
  if (lane == 0)
    for (; issued < stages - 1 && issued < n_my; ++issued) issue(issued);
  issued = __shfl_sync(0xffffffffu, issued, 0);
  XCache xc;
  xc.key = -1;
  const int grp = lane / LPR, lt = lane % LPR;
  int i = 0;
  bool ok = true;
  for (; i < n_my; ++i) {
    if (issued < n_my && issued <= i + stages - 1) {
      if (lane == 0) issue(issued);
      ++issued;
    }
    ok = __all_sync(0xffffffffu, mbar_wait(&ring.bars[i % stages], (i / stages) & 1, status));
    if (!ok) break;
    const int row0 = (u0 + i) * RU, nrows = min(RU, rows - row0);
    const uint8_t* gsrc = W + (size_t)row0 * rb;
    const uint8_t* rowsp =
        ring.smem + (size_t)(i % stages) * stage_bytes + (reinterpret_cast<uintptr_t>(gsrc) & 15);
    for (int t = 0; t < tokens; ++t) {
      float a[RL], unused[RL];
      unit_rows<TYPE, LPR, RL, false>(rowsp, (int)rb, nullptr, 0, nrows, tasks, xp + t * xld, t,
                                      xc, lane, a, unused);
#pragma unroll
      for (int q = 0; q < RL; ++q) {
        const int r = grp + q * RPP;
        if (lt == q && r < nrows) y[(long)t * ldy + row0 + r] = a[q];
      }
    }
    __syncwarp();
  }
  if (!ok)  // drain copies still in flight before the warp exits
    for (int k = i + 1; k < issued; ++k) mbar_wait(&ring.bars[k % stages], (k / stages) & 1, nullptr);
}

// Q4_K rows on the tensor cores (mma.cuh): each CTA owns a contiguous run of
// 16-row tiles, stages them through its bulk-copy ring, and computes the
// tokens in groups of NT against each staged tile.
template <int NT, int NW>
__global__ void __launch_bounds__(NW * 32, 1)
    gemv_q4k_mma_kernel(const uint8_t* __restrict__ W, size_t rb, int rows, int nsb,
                        const uint8_t* __restrict__ mx, int tokens, float* __restrict__ y,
                        long ldy, TilePlan plan, int* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)plan.stages * plan.stage_bytes);
  float* red = reinterpret_cast<float*>(full + 8);
  if (threadIdx.x == 0) {
    for (int s = 0; s < plan.stages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const size_t mxb = mx_bytes(nsb * 256);
  const int tiles = (rows + kTileRows - 1) / kTileRows;
  const int u0 = (int)((long)blockIdx.x * tiles / gridDim.x);
  const int n_my = (int)((long)(blockIdx.x + 1) * tiles / gridDim.x) - u0;
  auto issue = [&](int idx) {
    const int row0 = (u0 + idx) * kTileRows, s = idx % plan.stages;
    tile_issue(smem + (size_t)s * plan.stage_bytes, &full[s], plan.pitch,
               min(kTileRows, rows - row0), rb, W + (size_t)row0 * rb, nullptr, lane);
  };
  int issued = 0;  // meaningful in warp 0 (the producer)
  if (warp == 0)
    for (; issued < plan.stages && issued < n_my; ++issued) issue(issued);
  int i = 0, buf = 0;
  bool stop = false;
  for (; i < n_my; ++i) {
    const int s = i % plan.stages;
    const bool ok = mbar_wait(&full[s], (i / plan.stages) & 1, status);
    const int row0 = (u0 + i) * kTileRows, nr = min(kTileRows, rows - row0);
    const uint8_t* st = smem + (size_t)s * plan.stage_bytes;
    int t0 = 0;
    do {
      const int nt = min(NT, tokens - t0);
      const uint8_t* mxp[NT];
#pragma unroll
      for (int n = 0; n < NT; ++n) mxp[n] = mx + (size_t)min(t0 + n, tokens - 1) * mxb;
      float2 acc[1][NT][2];
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int n = 0; n < NT; ++n) acc[0][n][r] = make_float2(0.f, 0.f);
      if (ok) tile_items<NT, 1, NW>(st, plan.pitch, nsb, warp, lane, mxp, nt, acc);
      float* rbuf = red + buf * (tile_red_floats<NT, 1, NW>() / 2);
      tile_partials_store<NT, 1>(rbuf, warp, lane, acc);
      stop = __syncthreads_or(!ok);  // also: every warp is done with this stage
      if (stop) break;
      const int r = threadIdx.x & 15, n = threadIdx.x >> 4;
      if (n < nt && r < nr) y[(long)(t0 + n) * ldy + row0 + r] = tile_row_sum<NT, 1, NW>(rbuf, 0, r, n);
      buf ^= 1;
      t0 += NT;
    } while (t0 < tokens);
    if (stop) break;
    if (warp == 0 && issued < n_my) {
      issue(issued);
      ++issued;
    }
  }
  if (stop && threadIdx.x == 0)  // drain copies still in flight before the CTA exits
    for (int q = i; q < issued; ++q) mbar_wait(&full[q % plan.stages], (q / plan.stages) & 1, nullptr);
}

// The same tile pipeline for up to NT tokens with the activation prep fused
// in: every CTA forms the tokens' mx layout of the raw input in shared memory
// while its first tiles stream in (the input is a few KB per token), so the
// call is one launch and the B fragments are shared-memory reads.
template <int NT, int NW>
__global__ void __launch_bounds__(NW * 32, 1)
    gemv_q4k_fused_kernel(const uint8_t* __restrict__ W, size_t rb, int rows, int nsb,
                          const float* __restrict__ x, long ldx, int tokens,
                          float* __restrict__ y, long ldy, TilePlan plan, int* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = nsb * 256;
  const size_t mxb = mx_bytes(K);
  uint8_t* act = smem + (size_t)plan.stages * plan.stage_bytes;  // [NT][mxb]
  uint8_t* bz = act + NT * mxb;                                  // 32 zero bytes
  uint64_t* full = reinterpret_cast<uint64_t*>(bz + 32);
  float* red = reinterpret_cast<float*>(full + 8);
  if (threadIdx.x == 0) {
    for (int s = 0; s < plan.stages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  if (threadIdx.x < 8) reinterpret_cast<uint32_t*>(bz)[threadIdx.x] = 0u;
  __syncthreads();
  const int tiles = (rows + kTileRows - 1) / kTileRows;
  const int u0 = (int)((long)blockIdx.x * tiles / gridDim.x);
  const int n_my = (int)((long)(blockIdx.x + 1) * tiles / gridDim.x) - u0;
  auto issue = [&](int idx) {
    const int row0 = (u0 + idx) * kTileRows, s = idx % plan.stages;
    tile_issue(smem + (size_t)s * plan.stage_bytes, &full[s], plan.pitch,
               min(kTileRows, rows - row0), rb, W + (size_t)row0 * rb, nullptr, lane);
  };
  // the tokens' prepared input, 128 values per warp item (mx_store4 wants the
  // 8 lanes of each 32-value sub-block together); a warp's next four items
  // are loaded before any is converted, so their latencies overlap.  The
  // kernel is launched with programmatic stream serialization: its first
  // tiles' copies (the weights depend on no kernel before it) are issued
  // while the kernel before it still runs, and the input is read after
  // griddepcontrol.wait (the input is that kernel's output; the output may
  // still be its input).
  constexpr int kPrepBatch = 4;
  const int items = tokens * (K >> 7);
  float4 v[kPrepBatch];
  auto load_batch = [&](int it0) {
#pragma unroll
    for (int b = 0; b < kPrepBatch; ++b) {
      const int it = min(it0 + b * NW, items - 1);  // clamped, not guarded
      const int tok = it / (K >> 7), e = (it - tok * (K >> 7)) * 128 + lane * 4;
      v[b] = __ldg(reinterpret_cast<const float4*>(x + (long)tok * ldx + e));
    }
  };
  int issued = 0;  // meaningful in warp 0 (the producer)
  if (warp == 0)
    for (; issued < plan.stages && issued < n_my; ++issued) issue(issued);
  griddep_wait();
  griddep_launch();
  for (int it0 = warp; it0 < items; it0 += NW * kPrepBatch) {
    load_batch(it0);
#pragma unroll
    for (int b = 0; b < kPrepBatch; ++b) {
      const int it = it0 + b * NW;  // warp-uniform
      if (it < items) {
        const int tok = it / (K >> 7), e = (it - tok * (K >> 7)) * 128 + lane * 4;
        mx_store4(act + tok * mxb, K, e, v[b]);
      }
    }
  }
  __syncthreads();
  const uint8_t* mxp[NT];
#pragma unroll
  for (int n = 0; n < NT; ++n) mxp[n] = act + (size_t)min(n, tokens - 1) * mxb;
  int i = 0;
  bool stop = false;
  for (; i < n_my; ++i) {
    const int s = i % plan.stages;
    const bool ok = mbar_wait(&full[s], (i / plan.stages) & 1, status);
    const int row0 = (u0 + i) * kTileRows, nr = min(kTileRows, rows - row0);
    const uint8_t* st = smem + (size_t)s * plan.stage_bytes;
    float2 acc[1][NT][2];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int n = 0; n < NT; ++n) acc[0][n][r] = make_float2(0.f, 0.f);
    if (ok) tile_items<NT, 1, NW, true>(st, plan.pitch, nsb, warp, lane, mxp, tokens, acc, bz);
    float* rbuf = red + (i & 1) * (tile_red_floats<NT, 1, NW>() / 2);
    tile_partials_store<NT, 1>(rbuf, warp, lane, acc);
    stop = __syncthreads_or(!ok);  // also: every warp is done with this stage
    if (stop) break;
    if (warp == 0 && issued < n_my) {  // the refill first, then the rows' sums
      issue(issued);
      ++issued;
    }
    const int r = threadIdx.x & 15, n = threadIdx.x >> 4;
    if (n < tokens && r < nr) y[(long)n * ldy + row0 + r] = tile_row_sum<NT, 1, NW>(rbuf, 0, r, n);
  }
  if (stop && threadIdx.x == 0)  // drain copies still in flight before the CTA exits
    for (int q = i; q < issued; ++q) mbar_wait(&full[q % plan.stages], (q / plan.stages) & 1, nullptr);
}

// F32 rows (the MoE router, ffn_gate_inp), tiled: a CTA of 4 warps takes 16
// rows (4 per warp) and up to kF32Tok tokens, whose activations it first
// copies into shared memory, so that each weight float4 read from global
// memory serves 8 tokens and each activation read serves 4 rows.  Lane l
// sums columns 4l.., 4(l+32).. of its 32 (row, token) products, and the 32
// sums meet in a 31-shuffle butterfly that leaves lane l with product l.
constexpr int kF32Rows = 4, kF32Tok = 8;
__global__ void __launch_bounds__(128) gemv_f32_tile_kernel(const float* __restrict__ W, int rows,
                                                            int K, const float* __restrict__ x,
                                                            long ldx, int tokens,
                                                            float* __restrict__ y, long ldy) {
  extern __shared__ float4 xs4[];  // [kF32Tok][K/4]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ __align__(8) uint64_t bar;
  const int t0 = blockIdx.y * kF32Tok, nt = min(kF32Tok, tokens - t0);
  const int K4 = K >> 2;
  const int crow0 = blockIdx.x * 4 * kF32Rows, crows = min(4 * kF32Rows, rows - crow0);
  float4* ws4 = xs4 + kF32Tok * K4;  // [16][K/4] this CTA's weight rows
  // one bulk copy of the token rows and one of the weight rows, so the loads
  // cost one round trip instead of one per loop iteration
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    const uint32_t xb = (uint32_t)K * 4u;
    mbar_expect_tx(&bar, xb * (uint32_t)(nt + crows));
    if (ldx == K) {
      tma_load_1d(xs4, x + (long)t0 * ldx, xb * nt, &bar);
    } else {
      for (int n = 0; n < nt; ++n) tma_load_1d(xs4 + n * K4, x + (long)(t0 + n) * ldx, xb, &bar);
    }
    tma_load_1d(ws4, W + (size_t)crow0 * K, xb * crows, &bar);
  }
  for (int i = nt * K4 + threadIdx.x; i < kF32Tok * K4; i += blockDim.x)
    xs4[i] = make_float4(0.f, 0.f, 0.f, 0.f);  // tokens past the end
  __syncthreads();
  mbar_wait(&bar, 0, nullptr);
  const int row0 = (blockIdx.x * 4 + warp) * kF32Rows;
  if (row0 >= rows) return;
  float2 acc[kF32Rows][kF32Tok / 2];  // (token 2p, token 2p+1)
#pragma unroll
  for (int r = 0; r < kF32Rows; ++r)
#pragma unroll
    for (int p = 0; p < kF32Tok / 2; ++p) acc[r][p] = make_float2(0.f, 0.f);
  const float4* wr[kF32Rows];
#pragma unroll
  for (int r = 0; r < kF32Rows; ++r)
    wr[r] = ws4 + (size_t)min(warp * kF32Rows + r, crows - 1) * K4;
  for (int c = lane; c < K4; c += 32) {
    float4 wv[kF32Rows];
#pragma unroll
    for (int r = 0; r < kF32Rows; ++r) wv[r] = wr[r][c];
#pragma unroll
    for (int p = 0; p < kF32Tok / 2; ++p) {
      const float4 xa = xs4[(2 * p) * K4 + c], xb = xs4[(2 * p + 1) * K4 + c];
#pragma unroll
      for (int r = 0; r < kF32Rows; ++r) {
        acc[r][p] = __ffma2_rn(make_float2(wv[r].x, wv[r].x), make_float2(xa.x, xb.x), acc[r][p]);
        acc[r][p] = __ffma2_rn(make_float2(wv[r].y, wv[r].y), make_float2(xa.y, xb.y), acc[r][p]);
        acc[r][p] = __ffma2_rn(make_float2(wv[r].z, wv[r].z), make_float2(xa.z, xb.z), acc[r][p]);
        acc[r][p] = __ffma2_rn(make_float2(wv[r].w, wv[r].w), make_float2(xa.w, xb.w), acc[r][p]);
      }
    }
  }
  // butterfly: value v[i], i = r * 8 + n, ends on lane i
  float v[32];
#pragma unroll
  for (int r = 0; r < kF32Rows; ++r)
#pragma unroll
    for (int p = 0; p < kF32Tok / 2; ++p) {
      v[r * 8 + 2 * p] = acc[r][p].x;
      v[r * 8 + 2 * p + 1] = acc[r][p].y;
    }
#pragma unroll
  for (int h = 16; h >= 1; h >>= 1) {
    const bool upper = (lane & h) != 0;
#pragma unroll
    for (int i = 0; i < h; ++i) {
      const float send = upper ? v[i] : v[i + h];
      const float keep = upper ? v[i + h] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, h);
    }
  }
  const int r = lane >> 3, n = lane & 7;
  if (row0 + r < rows && n < nt) y[(long)(t0 + n) * ldy + row0 + r] = v[0];
}

// F32 rows without the tile's shared memory (very wide rows or unaligned
// data): one warp per (row, group of up to
// 8 tokens); activations are read straight from global memory (they stay in
// L1/L2), so there is no staging and every SM takes part.
__global__ void __launch_bounds__(128) gemv_f32_kernel(const float* __restrict__ W, int rows,
                                                       int K, const float* __restrict__ x,
                                                       long ldx, int tokens,
                                                       float* __restrict__ y, long ldy) {
  const int lane = threadIdx.x & 31;
  const int groups = (tokens + 7) / 8;
  const long items = (long)rows * groups;
  const bool vec = (K & 3) == 0 && (ldx & 3) == 0 &&
                   (reinterpret_cast<uintptr_t>(W) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  for (long it = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); it < items;
       it += (long)gridDim.x * (blockDim.x >> 5)) {
    const int row = (int)(it / groups), t0 = (int)(it - (long)row * groups) * 8;
    const int nt = min(8, tokens - t0);
    const float* wr = W + (size_t)row * K;
    float acc[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) acc[t] = 0.f;
    if (vec) {
      const float4* w4 = reinterpret_cast<const float4*>(wr);
      for (int k4 = lane; k4 < (K >> 2); k4 += 32) {
        const float4 wv = __ldg(w4 + k4);
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          if (t < nt) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(x + (long)(t0 + t) * ldx) + k4);
            acc[t] = fmaf(wv.x, v.x, acc[t]);
            acc[t] = fmaf(wv.y, v.y, acc[t]);
            acc[t] = fmaf(wv.z, v.z, acc[t]);
            acc[t] = fmaf(wv.w, v.w, acc[t]);
          }
        }
      }
    } else {
      for (int k = lane; k < K; k += 32) {
        const float wv = __ldg(wr + k);
#pragma unroll
        for (int t = 0; t < 8; ++t)
          if (t < nt) acc[t] = fmaf(wv, __ldg(x + (long)(t0 + t) * ldx + k), acc[t]);
      }
    }
#pragma unroll
    for (int t = 0; t < 8; ++t) acc[t] = warp_sum(acc[t]);
#pragma unroll
    for (int t = 0; t < 8; ++t)
      if (lane == t && t < nt) y[(long)(t0 + t) * ldy + row] = acc[t];
  }
}

// Q5_0 / Q8_0 rows (32-value blocks; dot-product-with-q5-0-tensor-data,
// llambda.lisp L4037-4068, and -q8-0-, L4070-4094): one warp per row, 8
// blocks (256 values) per step, lane l taking values [8l, 8l + 8) of the step
// (block l/4, part l%4), so the weight loads of a step are one contiguous
// run and the activation reads are contiguous shared-memory reads; the
// tokens' inputs sit in shared memory, so a block's bytes are read once for
// all of them.  Per lane and block the exact integer values times x are
// summed in fp32 and scaled by d (the reference scales each product; only
// the rounding order differs).  Rows are 2-byte aligned (22- and 34-byte
// blocks): 16-bit loads.
template <int TYPE>
__global__ void __launch_bounds__(256) gemv_q32_kernel(const uint8_t* __restrict__ W, size_t rb,
                                                       int rows, int K,
                                                       const float* __restrict__ x, long ldx,
                                                       int n_valid, int tokens,
                                                       float* __restrict__ y, long ldy) {
  constexpr int kMaxTok = 8;
  constexpr int BB = TYPE == LB_TYPE_Q5_0 ? LB_Q5_0 : LB_Q8_0;
  extern __shared__ __align__(16) float xs[];  // [tokens][K], zero past n_valid
  for (int i = threadIdx.x; i < tokens * K; i += blockDim.x) {
    const int t = i / K, c = i - t * K;
    xs[i] = c < n_valid ? x[(long)t * ldx + c] : 0.f;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nblk = K >> 5, part = lane & 3;
  for (int row = blockIdx.x * 8 + warp; row < rows; row += gridDim.x * 8) {
    const uint8_t* wr = W + (size_t)row * rb;
    float acc[kMaxTok];
#pragma unroll
    for (int t = 0; t < kMaxTok; ++t) acc[t] = 0.f;
    constexpr int U = 4;  // steps whose loads are issued before any is used
    for (int b0 = 0; b0 < nblk; b0 += 8 * U) {
      // per step: d, this lane's 8 value bytes as two words (Q8_0: qs bytes
      // [8 part, +8); Q5_0: qs bytes [(8 part) % 16, +8)), Q5_0's qh
      uint32_t rd[U], ra[U], rb2[U], rh[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int b = min(b0 + 8 * u + (lane >> 2), nblk - 1);  // clamped: loads overlap
        const unsigned short* h = reinterpret_cast<const unsigned short*>(wr + (size_t)b * BB);
        rd[u] = __ldg(h);
        const unsigned short* q = h + (TYPE == LB_TYPE_Q8_0 ? 1 + 4 * part : 3 + ((8 * part) & 15) / 2);
        ra[u] = (uint32_t)__ldg(q) | ((uint32_t)__ldg(q + 1) << 16);
        rb2[u] = (uint32_t)__ldg(q + 2) | ((uint32_t)__ldg(q + 3) << 16);
        rh[u] = TYPE == LB_TYPE_Q5_0 ? ((uint32_t)__ldg(h + 1) | ((uint32_t)__ldg(h + 2) << 16)) : 0u;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int b = b0 + 8 * u + (lane >> 2);
        if (b >= nblk) continue;
        const float d = __half2float(__ushort_as_half((unsigned short)rd[u]));
        // each value byte becomes the float 2^23 + byte (one PRMT under the
        // exponent byte 0x4B); subtracting 2^23 + offset is exact
        uint32_t w[2];
        float off;
        if (TYPE == LB_TYPE_Q8_0) {  // signed bytes: xor 0x80 gives q + 128
          w[0] = ra[u] ^ 0x80808080u;
          w[1] = rb2[u] ^ 0x80808080u;
          off = 8388608.0f + 128.0f;
        } else {  // nibble | qh bit j << 4 gives q + 16
          const int sh = part >= 2 ? 4 : 0;
          const uint32_t hb = (rh[u] >> (8 * part)) & 0xFFu;  // qh bits 8 part .. 8 part + 7
          w[0] = ((ra[u] >> sh) & 0x0F0F0F0Fu) | ((((hb & 15u) * 0x00204081u) & 0x01010101u) << 4);
          w[1] = ((rb2[u] >> sh) & 0x0F0F0F0Fu) | ((((hb >> 4) * 0x00204081u) & 0x01010101u) << 4);
          off = 8388608.0f + 16.0f;
        }
        float q[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          q[i] = __uint_as_float(__byte_perm(w[0], 0x4B000000u, 0x7440u | i)) - off;
          q[4 + i] = __uint_as_float(__byte_perm(w[1], 0x4B000000u, 0x7440u | i)) - off;
        }
#pragma unroll
        for (int t = 0; t < kMaxTok; ++t) {
          if (t < tokens) {
            const float4* xb = reinterpret_cast<const float4*>(xs + t * K + b * 32 + 8 * part);
            const float4 xa = xb[0], xc = xb[1];
            float sum = q[0] * xa.x;
            sum = fmaf(q[1], xa.y, sum);
            sum = fmaf(q[2], xa.z, sum);
            sum = fmaf(q[3], xa.w, sum);
            sum = fmaf(q[4], xc.x, sum);
            sum = fmaf(q[5], xc.y, sum);
            sum = fmaf(q[6], xc.z, sum);
            sum = fmaf(q[7], xc.w, sum);
            acc[t] = fmaf(d, sum, acc[t]);
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < kMaxTok; ++t) {
      if (t < tokens) {
        const float v = warp_sum(acc[t]);
        if (lane == 0) y[(long)t * ldy + row] = v;
      }
    }
  }
}

// Q5_K rows (dot-product-with-q5-k-tensor-data, L4387-4441).  One warp per
// row, up to 8 tokens whose inputs sit in shared memory (zero past n_valid).
// Lane l takes values [8l, 8l + 8) of every block: sub-block s = l / 4
// (pair g = s / 2, high nibbles for odd s) at positions 8 (l % 4) .. + 7, so
// its 8 qs bytes and 8 qh bytes are two aligned 8-byte loads and the block
// header (d, dmin, packed scales) one 16-byte load shared by the warp.  Each
// value byte (nibble | qh bit s << 4, 0..31) becomes the float 2^23 + q by one
// byte permute under the exponent byte 0x4B; per sub-block the lane sums q*x
// and x in fp32 and applies the reference's delta = d*sc and offset =
// dmin*m once, (delta * sum(q x)) - (offset * sum(x)): the same products in
// another summation order.
__global__ void __launch_bounds__(256) gemv_q5k_kernel(const uint8_t* __restrict__ W, size_t rb,
                                                       int rows, int K,
                                                       const float* __restrict__ x, long ldx,
                                                       int n_valid, int tokens,
                                                       float* __restrict__ y, long ldy) {
  constexpr int kMaxTok = 8;
  extern __shared__ __align__(16) float xs[];  // [tokens][K]
  for (int i = threadIdx.x; i < tokens * K; i += blockDim.x) {
    const int t = i / K, c = i - t * K;
    xs[i] = c < n_valid ? x[(long)t * ldx + c] : 0.f;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nblk = K >> 8;
  const int sb = lane >> 2, pair = sb >> 1, pos = (lane & 3) * 8;
  const int nib_shift = (sb & 1) * 4;
  for (int row = blockIdx.x * 8 + warp; row < rows; row += gridDim.x * 8) {
    const uint8_t* wr = W + (size_t)row * rb;
    float acc[kMaxTok];
#pragma unroll
    for (int t = 0; t < kMaxTok; ++t) acc[t] = 0.f;
    constexpr int U = 4;  // blocks whose loads are issued before any is used
    for (int b0 = 0; b0 < nblk; b0 += U) {
      uint4 hdr[U];
      uint2 qh[U], qs[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint8_t* blk = wr + (size_t)min(b0 + u, nblk - 1) * LB_Q5K;  // clamped
        hdr[u] = __ldg(reinterpret_cast<const uint4*>(blk));
        qh[u] = __ldg(reinterpret_cast<const uint2*>(blk + 16 + pos));
        qs[u] = __ldg(reinterpret_cast<const uint2*>(blk + 48 + 32 * pair + pos));
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int b = b0 + u;
        if (b >= nblk) continue;
        const float d = __half2float(__ushort_as_half((unsigned short)(hdr[u].x & 0xFFFFu)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(hdr[u].x >> 16)));
        // get-scale-min-k4 (L4316-4336) of sub-block sb from scales[12] at
        // byte 4: scales[0..3] in hdr.y, [4..7] in hdr.z, [8..11] in hdr.w
        const int sh8 = 8 * (sb & 3);
        const uint32_t by = (hdr[u].y >> sh8) & 0xFFu, bz = (hdr[u].z >> sh8) & 0xFFu;
        uint32_t sc, mn;
        if (sb < 4) {
          sc = by & 63u;
          mn = bz & 63u;
        } else {
          const uint32_t bw = (hdr[u].w >> sh8) & 0xFFu;
          sc = (bw & 0x0Fu) | ((by >> 6) << 4);
          mn = (bw >> 4) | ((bz >> 6) << 4);
        }
        const float delta = d * (float)sc, offset = dmin * (float)mn;
        const uint32_t w0 = ((qs[u].x >> nib_shift) & 0x0F0F0F0Fu) |
                            (((qh[u].x >> sb) & 0x01010101u) << 4);
        const uint32_t w1 = ((qs[u].y >> nib_shift) & 0x0F0F0F0Fu) |
                            (((qh[u].y >> sb) & 0x01010101u) << 4);
        float q[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          q[i] = __uint_as_float(__byte_perm(w0, 0x4B000000u, 0x7440u | i)) - 8388608.0f;
          q[4 + i] = __uint_as_float(__byte_perm(w1, 0x4B000000u, 0x7440u | i)) - 8388608.0f;
        }
#pragma unroll
        for (int t = 0; t < kMaxTok; ++t) {
          if (t < tokens) {
            const float4* xb = reinterpret_cast<const float4*>(xs + t * K + b * 256 + 8 * lane);
            const float4 xa = xb[0], xc = xb[1];
            float qx = q[0] * xa.x;
            qx = fmaf(q[1], xa.y, qx);
            qx = fmaf(q[2], xa.z, qx);
            qx = fmaf(q[3], xa.w, qx);
            qx = fmaf(q[4], xc.x, qx);
            qx = fmaf(q[5], xc.y, qx);
            qx = fmaf(q[6], xc.z, qx);
            qx = fmaf(q[7], xc.w, qx);
            const float sx = ((xa.x + xa.y) + (xa.z + xa.w)) + ((xc.x + xc.y) + (xc.z + xc.w));
            acc[t] = fmaf(delta, qx, fmaf(-offset, sx, acc[t]));
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < kMaxTok; ++t) {
      if (t < tokens) {
        const float v = warp_sum(acc[t]);
        if (lane == 0) y[(long)t * ldy + row] = v;
      }
    }
  }
}

__global__ void check_scales_kernel(int type, const uint8_t* __restrict__ W, size_t blocks,
                                    unsigned* bad) {
  unsigned local = 0;
  for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < blocks;
       b += (size_t)gridDim.x * blockDim.x) {
    if (type == LB_TYPE_Q4_K || type == LB_TYPE_Q5_K) {  // d, dmin at bytes 0, 2
      const uint8_t* p = W + b * (type == LB_TYPE_Q4_K ? LB_Q4K : LB_Q5K);
      const uint32_t d = p[0] | (p[1] << 8), m = p[2] | (p[3] << 8);
      local += ((d & 0x7C00u) == 0x7C00u) || ((m & 0x7C00u) == 0x7C00u);
    } else if (type == LB_TYPE_Q5_0 || type == LB_TYPE_Q8_0) {
      const uint8_t* p = W + b * (type == LB_TYPE_Q5_0 ? LB_Q5_0 : LB_Q8_0);
      const uint32_t d = p[0] | (p[1] << 8);
      local += (d & 0x7C00u) == 0x7C00u;
    } else {
      const uint8_t* p = W + b * LB_Q6K + 208;
      const uint32_t d = p[0] | (p[1] << 8);
      local += (d & 0x7C00u) == 0x7C00u;
    }
  }
  local = __reduce_add_sync(0xffffffffu, local);
  if ((threadIdx.x & 31) == 0 && local) atomicAdd(bad, local);
}

__global__ void synth_q4k_kernel(uint64_t seed, uint64_t sid, uint64_t first, size_t n, float s,
                                 uint8_t* out) {
  for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < n;
       b += (size_t)gridDim.x * blockDim.x) {
    uint4 buf[9];
    lb_q4k_block(seed, sid, first + b, s, reinterpret_cast<uint8_t*>(buf));
    uint4* dst = reinterpret_cast<uint4*>(out + b * LB_Q4K);
#pragma unroll
    for (int i = 0; i < 9; ++i) dst[i] = buf[i];
  }
}

__global__ void synth_q6k_kernel(uint64_t seed, uint64_t sid, uint64_t first, size_t n, float s,
                                 uint8_t* out) {
  for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < n;
       b += (size_t)gridDim.x * blockDim.x) {
    unsigned short buf[105];
    lb_q6k_block(seed, sid, first + b, s, reinterpret_cast<uint8_t*>(buf));
    unsigned short* dst = reinterpret_cast<unsigned short*>(out + b * LB_Q6K);
#pragma unroll 5
    for (int i = 0; i < 105; ++i) dst[i] = buf[i];
  }
}

__global__ void synth_f32_kernel(uint64_t seed, uint64_t sid, uint64_t first, size_t n, float s,
                                 float* out) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    out[i] = lb_f32_value(seed, sid, first + i, s);
}

template <int TYPE, int LPR, int RL>
cudaError_t launch_dense(const UnitPlan& p, const void* W, size_t rb, int rows, int K,
                         const float* xp, int tokens, float* y, long ldy, int* status,
                         cudaStream_t stream) {
  auto kern = gemv_kernel<TYPE, LPR, RL>;
  const size_t smem = (size_t)p.warps * p.stages * (p.stage_bytes + 8);
  const int occ = prepared_occupancy(kern, p.warps * 32, smem);
  if (occ < 0) return cudaErrorUnknown;
  const int ru = RL * (32 / LPR);
  const long units = (rows + ru - 1) / ru;
  const long blocks = std::min<long>((units + p.warps - 1) / p.warps,
                                     (long)sm_count() * std::max(occ, 1));
  kern<<<(int)std::max<long>(blocks, 1), p.warps * 32, smem, stream>>>(
      static_cast<const uint8_t*>(W), rb, rows, K / 64, xp, tokens, y, ldy, p.stages,
      p.stage_bytes, status);
  return cudaGetLastError();
}

template <int NT, int NW>
cudaError_t launch_q4k_mma(const void* W, size_t rb, int rows, int K, const float* xp,
                           int tokens, float* y, long ldy, int* status, cudaStream_t stream) {
  auto kern = gemv_q4k_mma_kernel<NT, NW>;
  const size_t extra = 64 + (size_t)tile_red_floats<NT, 1, NW>() * 4;
  const TilePlan plan = tile_plan(rb, 1, kTileSmemBudget - extra);
  if (plan.stages < 2) return cudaErrorInvalidValue;
  const size_t smem = (size_t)plan.stages * plan.stage_bytes + extra;
  if (prepared_occupancy(kern, NW * 32, smem) < 1) return cudaErrorUnknown;
  const int tiles = (rows + kTileRows - 1) / kTileRows;
  const int grid = std::min(tiles, sm_count());
  kern<<<grid, NW * 32, smem, stream>>>(static_cast<const uint8_t*>(W), rb, rows, K / 256,
                                                reinterpret_cast<const uint8_t*>(xp), tokens, y,
                                                ldy, plan, status);
  return cudaGetLastError();
}

// CPS CTAs per SM, each with 1/CPS of the shared-memory budget: two smaller
// CTAs interleave their tiles' decode chains and barriers (config 1, one
// token: 11% faster than one CTA of 16 warps).  cudaErrorNotReady when the
// stages do not fit (the caller then takes another shape).
template <int NT, int NW, int CPS>
cudaError_t launch_q4k_fused(const void* W, size_t rb, int rows, int K, const float* x, long ldx,
                             int tokens, float* y, long ldy, int* status, cudaStream_t stream) {
  auto kern = gemv_q4k_fused_kernel<NT, NW>;
  const size_t extra =
      (size_t)NT * mx_bytes(K) + 32 + 64 + (size_t)tile_red_floats<NT, 1, NW>() * 4;
  if (kTileSmemBudget / CPS <= extra) return cudaErrorNotReady;
  const TilePlan plan = tile_plan(rb, 1, kTileSmemBudget / CPS - extra);
  if (plan.stages < 2) return CPS > 1 ? cudaErrorNotReady : cudaErrorInvalidValue;
  const size_t smem = (size_t)plan.stages * plan.stage_bytes + extra;
  const int occ = prepared_occupancy(kern, NW * 32, smem);
  if (occ < CPS) return CPS > 1 ? cudaErrorNotReady : cudaErrorUnknown;
  const int tiles = (rows + kTileRows - 1) / kTileRows;
  const int grid = std::min(tiles, CPS * sm_count());
  const cudaError_t e = launch_pdl(kern, dim3(grid), dim3(NW * 32), smem, stream,
                                   static_cast<const uint8_t*>(W), rb, rows, K / 256, x, ldx,
                                   tokens, y, ldy, plan, status);
  return e != cudaSuccess ? e : cudaGetLastError();
}

template <int NG, bool SLOT>
cudaError_t launch_q6k_slab(const void* W, size_t rb, int rows, int K, const uint8_t* m6,
                            int tokens, float* y, long ldy, int* status, cudaStream_t stream) {
  const int nsb = K / 256;
  const int stage_bytes = (int)((kTileRows * rb + 127) & ~size_t(127));
  const bool wide = nsb >= 16 && NG == 1;  // two groups need more than 96 registers
  const int cw = wide ? 16 : 8;
  const size_t per_stage = (size_t)stage_bytes + (size_t)cw * 32 * NG * sizeof(float2);
  const int stages = (int)std::min<size_t>(8, (kTileSmemBudget - sizeof(DenseSync)) / per_stage);
  if (stages < 2) return cudaErrorInvalidValue;
  const size_t smem = (size_t)stages * per_stage + sizeof(DenseSync);
  const int units = rows / kTileRows;
  const int grid = std::max(1, std::min(units, sm_count()));
  // programmatic launch: the weight copies start while the input's
  // preparation (the kernel before) still runs
  if constexpr (NG == 1) {  // only one group is instantiated wide
    if (wide) {
      auto kern = gemv_q6k_slab_kernel<NG, 16, SLOT>;
      if (prepared_occupancy(kern, 17 * 32, smem) < 1) return cudaErrorUnknown;
      const cudaError_t e =
          launch_pdl(kern, dim3(grid), dim3(17 * 32), smem, stream, static_cast<const uint8_t*>(W),
                     rb, rows, nsb, m6, tokens, y, ldy, stages, stage_bytes, status);
      return e != cudaSuccess ? e : cudaGetLastError();
    }
  }
  auto kern = gemv_q6k_slab_kernel<NG, 8, SLOT>;
  if (prepared_occupancy(kern, 9 * 32, smem) < 1) return cudaErrorUnknown;
  const cudaError_t e =
      launch_pdl(kern, dim3(grid), dim3(9 * 32), smem, stream, static_cast<const uint8_t*>(W), rb,
                 rows, nsb, m6, tokens, y, ldy, stages, stage_bytes, status);
  return e != cudaSuccess ? e : cudaGetLastError();
}

// The sliced kernel for 3..8 tokens when K is 8 or 16 super-blocks; false
// when it does not apply (the caller takes the streamed path).
template <int NG>
bool launch_q6k_slice(const void* W, size_t rb, int rows, int K, const uint8_t* m6, int tokens,
                      float* y, long ldy, int* status, cudaStream_t stream, cudaError_t* err) {
  const int nsb = K / 256, slices = nsb / kSliceSb;
  if (nsb % kSliceSb || slices < 1 || slices > 2 || tokens > 4 * NG) return false;
  const size_t per_stage = (size_t)kTileRows * kSliceSb * LB_Q6K +
                           (size_t)kSliceSb * 32 * NG * sizeof(float2);
  const size_t fixed = (size_t)4 * NG * (kSliceSb * 1152 + 16) + sizeof(SliceSync);
  if (fixed + 3 * per_stage > kTileSmemBudget) return false;
  const int stages = (int)std::min<size_t>(8, (kTileSmemBudget - fixed) / per_stage);
  const size_t smem = fixed + (size_t)stages * per_stage;
  auto kern = gemv_q6k_slice_kernel<NG>;
  if (prepared_occupancy(kern, (kSliceSb + 1) * 32, smem) < 1) return false;
  if (slices > 1) {
    *err = cudaMemset2DAsync(y, (size_t)ldy * sizeof(float), 0, (size_t)rows * sizeof(float),
                             tokens, stream);
    if (*err != cudaSuccess) return true;
  }
  const int grid = std::max(slices, sm_count() / slices * slices);
  kern<<<grid, (kSliceSb + 1) * 32, smem, stream>>>(static_cast<const uint8_t*>(W), rb, rows,
                                                     slices, m6, tokens, y, ldy, stages, status);
  *err = cudaGetLastError();
  return true;
}

}  // namespace

// ------------------------------------------------------------ host API

size_t xprep_floats(int K, int tokens) {
  return std::max({(size_t)xp_stride(K), mx_bytes(K) / 4, m6_bytes(K) / 4}) * tokens;
}

// Q6_K matrices of whole 16-row blocks run on the tensor cores, one or two
// tokens in the sub-block slot form.
static bool q6k_dense_mma(int rows) { return rows % kTileRows == 0; }
static bool q6k_dense_slots(int tokens) { return tokens <= 2; }

cudaError_t launch_prep(int type, int rows, const float* x, long ldx, int n_valid, int K,
                        int tokens, const int* gather, float* xp, cudaStream_t stream) {
  if (tokens <= 0) return cudaSuccess;
  if (K % 256) return cudaErrorInvalidValue;
  dim3 grid(K / 256, tokens);
  if (type == LB_TYPE_Q4_K)
    prep_kernel<LB_TYPE_Q4_K><<<grid, 64, 0, stream>>>(x, ldx, n_valid, K, gather, xp);
  else if (type == LB_TYPE_Q6_K && q6k_dense_mma(rows) && q6k_dense_slots(tokens))
    return launch_pdl(m6_prep_kernel<true>, grid, dim3(64), 0, stream, x, ldx, n_valid, K,
                      gather, reinterpret_cast<uint8_t*>(xp));
  else if (type == LB_TYPE_Q6_K && q6k_dense_mma(rows))
    return launch_pdl(m6_prep_kernel<false>, grid, dim3(64), 0, stream, x, ldx, n_valid, K,
                      gather, reinterpret_cast<uint8_t*>(xp));
  else if (type == LB_TYPE_Q6_K)
    prep_kernel<LB_TYPE_Q6_K><<<grid, 64, 0, stream>>>(x, ldx, n_valid, K, gather, xp);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t launch_gemv_prepped(int type, const void* W, size_t rb, int rows, int K,
                                const float* xp, int tokens, float* y, long ldy, int* status,
                                cudaStream_t stream) {
  if (rows <= 0 || tokens <= 0) return cudaSuccess;
  const UnitPlan p = plan_units(rb, K / 64, 1);
#define LB_DENSE(T, L, RR)                                                                   \
  if (type == T && p.lpr == L && p.rl == RR)                                                 \
    return launch_dense<T, L, RR>(p, W, rb, rows, K, xp, tokens, y, ldy, status, stream);
#define LB_DENSE_T(T)                                                                        \
  LB_DENSE(T, 8, 1) LB_DENSE(T, 8, 2) LB_DENSE(T, 8, 4) LB_DENSE(T, 16, 1) LB_DENSE(T, 16, 2)  \
  LB_DENSE(T, 16, 4) LB_DENSE(T, 32, 1) LB_DENSE(T, 32, 2) LB_DENSE(T, 32, 4)
  if (type == LB_TYPE_Q6_K && q6k_dense_mma(rows)) {
    const uint8_t* m6 = reinterpret_cast<const uint8_t*>(xp);
    if (q6k_dense_slots(tokens))
      return tokens == 1 ? launch_q6k_slab<1, true>(W, rb, rows, K, m6, 1, y, ldy, status, stream)
                         : launch_q6k_slab<2, true>(W, rb, rows, K, m6, 2, y, ldy, status, stream);
    for (int t0 = 0; t0 < tokens; t0 += 8) {  // 8 tokens per pass over the weights
      const int nt = std::min(8, tokens - t0);
      cudaError_t se = cudaSuccess;
      const uint8_t* m6t = m6 + (size_t)t0 * m6_bytes(K);
      float* yt = y + (long)t0 * ldy;
      if (nt <= 4 ? launch_q6k_slice<1>(W, rb, rows, K, m6t, nt, yt, ldy, status, stream, &se)
                  : launch_q6k_slice<2>(W, rb, rows, K, m6t, nt, yt, ldy, status, stream, &se)) {
        if (se != cudaSuccess) return se;
        continue;
      }
      const cudaError_t e =
          nt <= 4 ? launch_q6k_slab<1, false>(W, rb, rows, K, m6 + (size_t)t0 * m6_bytes(K), nt,
                                              y + (long)t0 * ldy, ldy, status, stream)
                  : launch_q6k_slab<2, false>(W, rb, rows, K, m6 + (size_t)t0 * m6_bytes(K), nt,
                                              y + (long)t0 * ldy, ldy, status, stream);
      if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
  }
  if (type == LB_TYPE_Q4_K) {
    if (tokens == 1) return launch_q4k_mma<1, 16>(W, rb, rows, K, xp, tokens, y, ldy, status, stream);
    if (tokens == 2) return launch_q4k_mma<2, 16>(W, rb, rows, K, xp, tokens, y, ldy, status, stream);
    return launch_q4k_mma<4, 8>(W, rb, rows, K, xp, tokens, y, ldy, status, stream);
  }
  LB_DENSE_T(LB_TYPE_Q6_K)
#undef LB_DENSE_T
#undef LB_DENSE
  return cudaErrorInvalidValue;
}

bool launch_gemv_fused(int type, const void* W, size_t rb, int rows, int K, const float* x,
                       long ldx, int tokens, float* y, long ldy, int* status, cudaStream_t stream,
                       cudaError_t* err) {
  if (type != LB_TYPE_Q4_K || tokens < 1 || tokens > 2 || K % 256 || (ldx & 3) ||
      (reinterpret_cast<uintptr_t>(x) & 15))
    return false;
  if (tokens == 1) {
    *err = launch_q4k_fused<1, 8, 2>(W, rb, rows, K, x, ldx, 1, y, ldy, status, stream);
    if (*err == cudaErrorNotReady)
      *err = launch_q4k_fused<1, 16, 1>(W, rb, rows, K, x, ldx, 1, y, ldy, status, stream);
  } else {
    *err = launch_q4k_fused<2, 16, 1>(W, rb, rows, K, x, ldx, 2, y, ldy, status, stream);
  }
  return true;
}

cudaError_t launch_gemv_f32(const void* W, int rows, int K, const float* x, long ldx, int tokens,
                            float* y, long ldy, cudaStream_t stream) {
  if (rows <= 0 || tokens <= 0) return cudaSuccess;
  const size_t smem = (size_t)(kF32Tok + 4 * kF32Rows) * K * sizeof(float);
  const bool vec = (K & 3) == 0 && (ldx & 3) == 0 && (reinterpret_cast<uintptr_t>(W) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  if (vec && smem <= 192 * 1024 && prepared_occupancy(gemv_f32_tile_kernel, 128, smem) >= 1) {
    dim3 grid((rows + kF32Rows * 4 - 1) / (kF32Rows * 4), (tokens + kF32Tok - 1) / kF32Tok);
    gemv_f32_tile_kernel<<<grid, 128, smem, stream>>>(static_cast<const float*>(W), rows, K, x,
                                                      ldx, tokens, y, ldy);
    return cudaGetLastError();
  }
  const long items = (long)rows * ((tokens + 7) / 8);
  const long blocks = std::min<long>((items + 3) / 4, (long)sm_count() * 16);
  gemv_f32_kernel<<<(int)std::max<long>(blocks, 1), 128, 0, stream>>>(
      static_cast<const float*>(W), rows, K, x, ldx, tokens, y, ldy);
  return cudaGetLastError();
}

namespace {

// Launches a shared-memory-input GEMV kernel (Q5_0 / Q8_0 / Q5_K) over the
// tokens in chunks of up to 8 whose inputs fit in 192 KB.
template <typename Kern>
cudaError_t launch_smem_gemv(Kern kern, const void* W, size_t rb, int rows, int K, const float* x,
                             long ldx, int n_valid, int tokens, float* y, long ldy,
                             cudaStream_t stream) {
  if ((size_t)K * 4 > 192 * 1024 || n_valid > K || n_valid < 0) return cudaErrorInvalidValue;
  const int per = std::max(1, std::min(8, (int)((192 * 1024) / ((size_t)K * 4))));
  const int grid = std::max(1, std::min((rows + 7) / 8, sm_count() * 8));
  for (int t0 = 0; t0 < tokens; t0 += per) {
    const int nt = std::min(per, tokens - t0);
    const size_t smem = (size_t)nt * K * 4;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)std::max<size_t>(smem, 1));
    if (e != cudaSuccess) return e;
    kern<<<grid, 256, smem, stream>>>(static_cast<const uint8_t*>(W), rb, rows, K,
                                      x + (long)t0 * ldx, ldx, n_valid, nt, y + (long)t0 * ldy,
                                      ldy);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace

cudaError_t launch_gemv_q32(int type, const void* W, size_t rb, int rows, int K, const float* x,
                            long ldx, int tokens, float* y, long ldy, cudaStream_t stream,
                            int n_valid) {
  if (rows <= 0 || tokens <= 0) return cudaSuccess;
  if ((type != LB_TYPE_Q5_0 && type != LB_TYPE_Q8_0) || K % 32) return cudaErrorInvalidValue;
  auto kern = type == LB_TYPE_Q5_0 ? gemv_q32_kernel<LB_TYPE_Q5_0> : gemv_q32_kernel<LB_TYPE_Q8_0>;
  return launch_smem_gemv(kern, W, rb, rows, K, x, ldx, n_valid < 0 ? K : n_valid, tokens, y,
                          ldy, stream);
}

cudaError_t launch_gemv_q5k(const void* W, size_t rb, int rows, int K, const float* x, long ldx,
                            int n_valid, int tokens, float* y, long ldy, cudaStream_t stream) {
  if (rows <= 0 || tokens <= 0) return cudaSuccess;
  if (K % 256 || rb != (size_t)K / 256 * LB_Q5K || (reinterpret_cast<uintptr_t>(W) & 15))
    return cudaErrorInvalidValue;
  return launch_smem_gemv(gemv_q5k_kernel, W, rb, rows, K, x, ldx, n_valid < 0 ? K : n_valid,
                          tokens, y, ldy, stream);
}

cudaError_t launch_projection(int type, const void* W, size_t rb, int rows, int K, const float* x,
                              long ldx, int n_valid, int tokens, float* y, long ldy, float* xp,
                              int* status, cudaStream_t stream) {
  if (rows <= 0 || tokens <= 0) return cudaSuccess;
  switch (type) {
    case LB_TYPE_F32:
      if (n_valid != K) return cudaErrorInvalidValue;
      return launch_gemv_f32(W, rows, K, x, ldx, tokens, y, ldy, stream);
    case LB_TYPE_Q5_0:
    case LB_TYPE_Q8_0:
      return launch_gemv_q32(type, W, rb, rows, K, x, ldx, tokens, y, ldy, stream, n_valid);
    case LB_TYPE_Q5_K:
      return launch_gemv_q5k(W, rb, rows, K, x, ldx, n_valid, tokens, y, ldy, stream);
    case LB_TYPE_Q4_K:
    case LB_TYPE_Q6_K: {
      cudaError_t e = cudaSuccess;
      if (n_valid == K && launch_gemv_fused(type, W, rb, rows, K, x, ldx, tokens, y, ldy, status,
                                            stream, &e))
        return e;
      e = launch_prep(type, rows, x, ldx, n_valid, K, tokens, nullptr, xp, stream);
      if (e != cudaSuccess) return e;
      return launch_gemv_prepped(type, W, rb, rows, K, xp, tokens, y, ldy, status, stream);
    }
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t check_fp16_scales(int type, const void* W, size_t blocks, unsigned* bad,
                              cudaStream_t stream) {
  if (type != LB_TYPE_Q4_K && type != LB_TYPE_Q6_K && type != LB_TYPE_Q5_0 &&
      type != LB_TYPE_Q8_0 && type != LB_TYPE_Q5_K)
    return cudaSuccess;
  const size_t grid = std::min<size_t>((blocks + 255) / 256, (size_t)sm_count() * 8);
  check_scales_kernel<<<(int)std::max<size_t>(grid, 1), 256, 0, stream>>>(
      type, static_cast<const uint8_t*>(W), blocks, bad);
  return cudaGetLastError();
}

cudaError_t synth_fill(int type, uint64_t seed, uint64_t sid, uint64_t first, size_t count,
                       float scale, void* out, cudaStream_t stream) {
  if (!count) return cudaSuccess;
  const float s = lb_sigma_scale(scale);
  const size_t grid = std::min<size_t>((count + 127) / 128, (size_t)sm_count() * 16);
  switch (type) {
    case LB_TYPE_Q4_K:
      synth_q4k_kernel<<<(int)grid, 128, 0, stream>>>(seed, sid, first, count, s,
                                                      static_cast<uint8_t*>(out));
      break;
    case LB_TYPE_Q6_K:
      synth_q6k_kernel<<<(int)grid, 128, 0, stream>>>(seed, sid, first, count, s,
                                                      static_cast<uint8_t*>(out));
      break;
    case LB_TYPE_F32:
      synth_f32_kernel<<<(int)grid, 128, 0, stream>>>(seed, sid, first, count, s,
                                                      static_cast<float*>(out));
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace lb
