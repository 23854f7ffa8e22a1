// Warp engine of the dequant-fused GEMV (v2): TMA-staged weight rows in
// shared memory, activations prepared once per call in global memory.
//
// Data flow per warp:
//   - a "unit" is R consecutive rows of one raw GGUF matrix (an expert's or
//     a dense tensor's); one lane issues a 1-D bulk TMA copy
//     (cp.async.bulk ... mbarrier::complete_tx) of the unit's 16-byte-aligned
//     byte range into one of the warp's S shared-memory stages, S-1 units
//     ahead of the unit being computed; the warp waits on the stage's
//     mbarrier with a bounded spin;
//   - lane L takes the 64-weight tasks L, L+32, ... of every row of the unit,
//     reads each activation float4 once from the prepared vector and applies
//     it to all R rows, so activation traffic is 4/R bytes per weight;
//   - a row of K columns has K/64 tasks of 64 weights:
//       Q4_K task t = (super-block t/4, sub-block pair p = t%4): qs bytes
//         [32p, 32p+32) hold sub-block 2p in their low nibbles and 2p+1 in
//         their high nibbles (dot-product-with-q4-k-m-tensor-data,
//         llambda.lisp L4338-4382; expand-q4-k-body, L4145-4201);
//       Q6_K task t = (super-block t/4, 128-chunk c = (t/2)%2, half h = t%2):
//         16 bytes of ql at 64c+16h and 64c+32+16h and 16 bytes of qh at
//         128+32c+16h give the 64 weights of sub-blocks 8c+h+2g, g = 0..3
//         (expand-q6-k-group, L4203-4310; q6-quant-1..4, L4115-4137);
//   - partial sums of the R rows meet in one warp shuffle reduction.
//
// Prepared activations ("xp"), per token, stride xp_stride(K) floats:
//   float4 xs[16][K/64]  task-minor (lane-consecutive 16-byte loads)
//   float  sx[K/32]      Q4_K only: sum of x over each 32-value sub-block
//
// Arithmetic per sub-block: weights stay exact integers; q becomes a float by
// one PRMT (2^23 + 2^16 q) and one packed f32x2 add removes the 2^23 bias (and
// Q6_K's -32 offset) exactly, leaving 2^16 q.  Q4_K then applies
// (d*sc)*sum(q*x) - (dmin*m)*sum(x) with the prepared sums of x, Q6_K
// (d*sc)*sum((q-32)*x).  Accumulation is fp32 (packed fma.rn.f32x2).
#pragma once

#include "common.cuh"

namespace lb {

// ------------------------------------------------------------ PTX helpers

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier generic-proxy accesses of shared memory before
// later async-proxy (TMA) accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void tma_load_1d(void* dst, const void* src, uint32_t bytes,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// 2-D tiled tensor copy global -> this CTA's shared memory (no multicast),
// completing on `bar`.  The innermost coordinate x times the element size
// must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], "
      "[%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// Prefetches [src, src + bytes) into L2 (src and bytes multiples of 16).
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  if (bytes)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// A try_wait suspends the thread until the phase completes or this many
// nanoseconds pass, so a waiting warp issues a handful of instructions
// instead of a spin loop.
constexpr uint32_t kSuspendNs = 200000;
// Every wait gives up after this long (a lost copy cannot hang the GPU).
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Programmatic dependent launch: a kernel launched with launch_pdl may start
// while the kernel before it in the stream is still running; it calls
// griddep_wait() before it reads anything that kernel wrote or writes
// anything it still reads (all of the earlier kernel's work is then done and
// visible), and griddep_launch() once its own CTAs are resident, so the next
// kernel can be scheduled early.  Both are no-ops without the attribute.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Barrier `id` (1-15; 0 is __syncthreads) over the first `threads` threads
// of the CTA (whole warps).
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n "
      "selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and sets bit 2 of *status) if the phase did
// not complete within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  do {
    if (mbar_try_wait(bar, parity)) return true;
  } while (global_ns() - t0 < kWaitLimitNs);
  if (status) atomicOr(status, 2);
  return false;
}

// Position in a ring of `stages` stages: the stage index and the parity of
// its current use, advanced without a division.
struct RingPos {
  int s = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next(int stages) {
    if (++s == stages) {
      s = 0;
      phase ^= 1u;
    }
  }
};

// Bounded wait that also gives up as soon as another warp of the CTA has
// raised *abort (after its own wait timed out).
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t* bar, uint32_t parity, int* status,
                                                   volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  do {
    if (*abort) return false;
    if (mbar_try_wait(bar, parity)) return true;
  } while (global_ns() - t0 < kWaitLimitNs);
  if (status) atomicOr(status, 2);
  *abort = 1;
  return false;
}

// Packed f32x2 FMA / add (sm_100): two lanes of fp32 work per instruction,
// each lane rounded exactly as a scalar fmaf / add.
__device__ __forceinline__ void ffma2(float2& acc, float a0, float a1, float b0, float b1) {
  acc = __ffma2_rn(make_float2(a0, a1), make_float2(b0, b1), acc);
}

// (a0 + b, a1 + b) with one packed add.
__device__ __forceinline__ void fadd2_const(float& a0, float& a1, float b) {
  const float2 r = __fadd2_rn(make_float2(a0, a1), make_float2(b, b));
  a0 = r.x;
  a1 = r.y;
}

// ------------------------------------------------------------ layouts

__host__ __device__ __forceinline__ int xp_stride(int K) { return K + K / 32; }

__device__ __forceinline__ uint32_t lds_u16(const uint8_t* p) {
  return (uint32_t)*reinterpret_cast<const unsigned short*>(p);
}

// Little-endian word at a 2-byte-aligned shared-memory address.
__device__ __forceinline__ uint32_t lds_w32_align2(const uint8_t* p) {
  return lds_u16(p) | (lds_u16(p + 2) << 16);
}

// Slot of element e of a K-vector in the prepared layout (float index).
template <int TYPE>
__device__ __forceinline__ int xp_index(int e, int tasks) {
  int task, i;
  if (TYPE == LB_TYPE_Q4_K) {
    task = e >> 6;
    i = (e & 63) >> 2;
  } else {
    const int sb = e >> 8, r = e & 255;
    const int c = r >> 7, r2 = r & 127;
    const int g = r2 >> 5, r3 = r2 & 31;
    const int h = r3 >> 4, m = (r3 & 15) >> 2;
    task = sb * 4 + c * 2 + h;
    i = g * 4 + m;
  }
  return (i * tasks + task) * 4 + (e & 3);
}

// ------------------------------------------------------------ row units
//
// One token per pass.  Lanes are split into groups of LPR lanes (LPR = 8, 16
// or 32, the smallest power of two covering the row's tasks, capped at 32);
// the 32/LPR groups take different rows of the unit and the LPR lanes of a
// group take the row's tasks.  A lane holds its task's 64 prepared
// activations in registers and applies them to every row it computes, and,
// when a row has no more tasks than a group has lanes, keeps them across
// units for as long as the activation vector does not change (XCache).
// Magic floats lose their 2^23 bias in a packed f32x2 add before they are
// accumulated, so the sums are plain fp32 sums of exact products.

constexpr float kMagic = 8388608.0f;  // 2^23

// The 64 activations of one task (and, for Q4_K, its two sub-block sums).
struct XCache {
  float4 v[16];
  float2 s;
  long key;  // identity of the cached vector and task; -1: empty
};

template <int TYPE>
__device__ __forceinline__ void load_task_x(XCache& xc, const float* xp, int tasks, int task) {
  const float4* x4 = reinterpret_cast<const float4*>(xp);
#pragma unroll
  for (int i = 0; i < 16; ++i) xc.v[i] = __ldg(x4 + i * tasks + task);
  if (TYPE == LB_TYPE_Q4_K) xc.s = __ldg(reinterpret_cast<const float2*>(xp + tasks * 64) + task);
}

// Dot of one Q4_K task (super-block sb, pair p) of the row whose super-block
// sb starts at `b` (shared memory, 16-byte aligned) with the cached x.
__device__ __forceinline__ float q4k_task_dot(const uint8_t* b, int p, const XCache& xc) {
  const uint4 hdr = *reinterpret_cast<const uint4*>(b);
  const uint4 qa = *reinterpret_cast<const uint4*>(b + 16 + 32 * p);
  const uint4 qb = *reinterpret_cast<const uint4*>(b + 32 + 32 * p);
  const float d = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
  int sc0, m0, sc1, m1;
  q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * p, sc0, m0);
  q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * p + 1, sc1, m1);
  // delta = d*sc, offset = dmin*m, each rounded once (L4363-4366)
  const float dsc0 = d * (float)sc0, dm0 = dmin * (float)m0;
  const float dsc1 = d * (float)sc1, dm1 = dmin * (float)m1;
  const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
  float2 al = make_float2(0.f, 0.f), ah = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t lo = w[j] & 0x0F0F0F0Fu, hi = (w[j] >> 4) & 0x0F0F0F0Fu;
    float l0 = magic_q<0>(lo), l1 = magic_q<1>(lo), l2 = magic_q<2>(lo), l3 = magic_q<3>(lo);
    float h0 = magic_q<0>(hi), h1 = magic_q<1>(hi), h2 = magic_q<2>(hi), h3 = magic_q<3>(hi);
    fadd2_const(l0, l1, -kMagic);  // exact: 2^16 * q
    fadd2_const(l2, l3, -kMagic);
    fadd2_const(h0, h1, -kMagic);
    fadd2_const(h2, h3, -kMagic);
    ffma2(al, l0, l1, xc.v[j].x, xc.v[j].y);
    ffma2(al, l2, l3, xc.v[j].z, xc.v[j].w);
    ffma2(ah, h0, h1, xc.v[8 + j].x, xc.v[8 + j].y);
    ffma2(ah, h2, h3, xc.v[8 + j].z, xc.v[8 + j].w);
  }
  float a = dsc0 * ((al.x + al.y) * kMagicUnscale);
  a = fmaf(-dm0, xc.s.x, a);
  a = fmaf(dsc1, (ah.x + ah.y) * kMagicUnscale, a);
  return fmaf(-dm1, xc.s.y, a);
}

// Dot of one Q6_K task (chunk c, half h) of the super-block at `blk` (shared
// memory, 2-byte aligned) with the cached x (xc.v[g*4 + j]: group g, float4 j).
__device__ __forceinline__ float q6k_task_dot(const uint8_t* blk, int c, int h, const XCache& xc) {
  // bias of a Q6_K magic float: 2^23 (magic) + 32 * 2^16 (the -32 offset)
  constexpr float kQ6Bias = -(8388608.0f + 32.0f * 65536.0f);
  const float d = half_bits_to_float(lds_u16(blk + 208));
  float2 acc[4];
#pragma unroll
  for (int g = 0; g < 4; ++g) acc[g] = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t A = lds_w32_align2(blk + 64 * c + 16 * h + 4 * j);
    const uint32_t B = lds_w32_align2(blk + 64 * c + 32 + 16 * h + 4 * j);
    const uint32_t H = lds_w32_align2(blk + 128 + 32 * c + 16 * h + 4 * j);
    uint32_t q[4];
    q[0] = (A & 0x0F0F0F0Fu) | ((H << 4) & 0x30303030u);
    q[1] = (B & 0x0F0F0F0Fu) | ((H << 2) & 0x30303030u);
    q[2] = ((A >> 4) & 0x0F0F0F0Fu) | (H & 0x30303030u);
    q[3] = ((B >> 4) & 0x0F0F0F0Fu) | ((H >> 2) & 0x30303030u);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      float f0 = magic_q<0>(q[g]), f1 = magic_q<1>(q[g]);
      float f2 = magic_q<2>(q[g]), f3 = magic_q<3>(q[g]);
      fadd2_const(f0, f1, kQ6Bias);  // exact: 2^16 * (q6 - 32)
      fadd2_const(f2, f3, kQ6Bias);
      ffma2(acc[g], f0, f1, xc.v[g * 4 + j].x, xc.v[g * 4 + j].y);
      ffma2(acc[g], f2, f3, xc.v[g * 4 + j].z, xc.v[g * 4 + j].w);
    }
  }
  float a = 0.f;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int sc = (int)(int8_t)(uint8_t)(lds_u16(blk + 192 + 8 * c + 2 * g) >> (8 * h));
    const float ds = d * (float)sc;  // delta = d*sc (L4470-4473)
    a = fmaf(ds, (acc[g].x + acc[g].y) * kMagicUnscale, a);
  }
  return a;
}

template <int TYPE>
__device__ __forceinline__ float task_dot(const uint8_t* row, int task, const XCache& xc) {
  if (TYPE == LB_TYPE_Q4_K)
    return q4k_task_dot(row + (task >> 2) * LB_Q4K, task & 3, xc);
  return q6k_task_dot(row + (task >> 2) * LB_Q6K, (task >> 1) & 1, task & 1, xc);
}

// Rows of one unit (RU = RL * 32/LPR rows per matrix; PAIR: a second matrix
// with the same activations).  Lane (grp, lt), grp = lane / LPR, computes
// rows grp + i * (32/LPR), i < RL, over tasks lt, lt + LPR, ...; y*[i] ends
// up with the full row sums on every lane of the group.  `key` names the
// activation vector xp so a cached one is reused.
template <int TYPE, int LPR, int RL, bool PAIR>
__device__ __forceinline__ void unit_rows(const uint8_t* rows0, int rb0, const uint8_t* rows1,
                                          int rb1, int nrows, int tasks, const float* xp, long key,
                                          XCache& xc, int lane, float (&y0)[RL], float (&y1)[RL]) {
  constexpr int RPP = 32 / LPR;
  const int grp = lane / LPR, lt = lane % LPR;
#pragma unroll
  for (int i = 0; i < RL; ++i) y0[i] = y1[i] = 0.f;
  for (int task = lt; task < tasks; task += LPR) {
    const long k = key * 64 + task;
    if (xc.key != k) {
      load_task_x<TYPE>(xc, xp, tasks, task);
      xc.key = k;
    }
#pragma unroll
    for (int i = 0; i < RL; ++i) {
      const int r = grp + i * RPP;
      if (r < nrows) {
        y0[i] += task_dot<TYPE>(rows0 + r * rb0, task, xc);
        if (PAIR) y1[i] += task_dot<TYPE>(rows1 + r * rb1, task, xc);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < RL; ++i) {
    y0[i] = warp_sum(y0[i], LPR);
    if (PAIR) y1[i] = warp_sum(y1[i], LPR);
  }
}

// Lanes per row group for a row of `tasks` tasks.
__host__ __device__ __forceinline__ int lanes_for(int tasks) {
  return tasks <= 8 ? 8 : tasks <= 16 ? 16 : 32;
}

// ------------------------------------------------------------ warp pipeline

// S-stage ring of one warp: stage s holds `stage_bytes` at smem + s*stage_bytes.
struct WarpRing {
  uint8_t* smem;
  uint64_t* bars;
  int stage_bytes;
  int stages;
};

__device__ __forceinline__ void ring_init(const WarpRing& ring, int lane) {
  if (lane == 0) {
    for (int s = 0; s < ring.stages; ++s) mbar_init(&ring.bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();
}

// Copies up to two contiguous byte ranges into stage s (lane 0 only).  Each
// range [src, src+bytes) is widened to 16-byte boundaries; the data of
// range k starts at stage + off_k + delta_k, where off_0 = 0 and off_1 =
// round_up(widened size of range 0).  Returns the deltas through d0/d1.
__device__ __forceinline__ void ring_issue(const WarpRing& ring, int s, const uint8_t* src0,
                                           size_t bytes0, const uint8_t* src1, size_t bytes1) {
  uint8_t* dst = ring.smem + (size_t)s * ring.stage_bytes;
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(src0) & ~uintptr_t(15);
  const uint32_t n0 =
      (uint32_t)(((reinterpret_cast<uintptr_t>(src0) + bytes0 + 15) & ~uintptr_t(15)) - a0);
  uint32_t n1 = 0;
  uintptr_t a1 = 0;
  if (src1) {
    a1 = reinterpret_cast<uintptr_t>(src1) & ~uintptr_t(15);
    n1 = (uint32_t)(((reinterpret_cast<uintptr_t>(src1) + bytes1 + 15) & ~uintptr_t(15)) - a1);
  }
  fence_proxy_async_smem();
  mbar_expect_tx(&ring.bars[s], n0 + n1);
  tma_load_1d(dst, reinterpret_cast<const void*>(a0), n0, &ring.bars[s]);
  if (src1) tma_load_1d(dst + n0, reinterpret_cast<const void*>(a1), n1, &ring.bars[s]);
}

// Dynamic shared-memory opt-in and occupancy of a kernel, computed once per
// (kernel address, shared-memory size).  Returns -1 on a CUDA error.
int kernel_occupancy(const void* kernel, int threads, size_t smem);

template <typename Kern>
inline int prepared_occupancy(Kern kern, int threads, size_t smem) {
  return kernel_occupancy(reinterpret_cast<const void*>(kern), threads, smem);
}

__device__ __forceinline__ uint32_t widened(const uint8_t* src, size_t bytes) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(src) & ~uintptr_t(15);
  return (uint32_t)(((reinterpret_cast<uintptr_t>(src) + bytes + 15) & ~uintptr_t(15)) - a);
}

}  // namespace lb
