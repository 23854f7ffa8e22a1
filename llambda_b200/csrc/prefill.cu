// Expert products of prefill-sized batches on the fifth-generation tensor
// cores (tcgen05, sm_100a).
//
// The decode kernels take an expert's tokens two to four at a time and decode
// its weights again for every pass.  A prefill batch routes tens of tokens to
// every expert, so this path decodes each 128-row block of an expert's
// weights ONCE per 64 tokens, into bf16 in shared memory, and multiplies it
// against all of those tokens with tcgen05.mma (accumulators in tensor
// memory):
//
//   gather   x (rms-normed when the layer has input_norm) -> bf16 rows grouped
//            by expert (xs: the routed entries in expert order, then the
//            shared expert's tokens), and the partial-output row of each
//   plan     tile lists: (expert, 64-token chunk, 128-row block) per pass
//   gate/up  D[128 rows x tokens] = W (decoded) . xs^T per tile; epilogue
//            silu(gate) * up (qwen3next-moe-into, llambda.lisp L5321-5426) or
//            relu(up)^2 (nemotron-h-moe-ffn-into, L5827-5949) -> bf16 rows hs
//   down     D = W_down (decoded) . hs^T -> fp32 partial outputs per (token,
//            rank), which the combine kernel weights and sums exactly as in
//            the decode path (L5380-5426, L5940-5949)
//
// Weight decode follows the reference's formulas: Q4_K w = (d*sc)*q - dmin*m
// (expand-q4-k-body, L4145-4201; get-scale-min-k4-at, L4316-4336), Q6_K
// w = d*sc*(q - 32) (q6-quant-1..4, L4115-4137; expand-q6-k-group,
// L4203-4310), each rounded once to bf16; tokens are rounded to bf16; all
// sums are fp32 in the tensor cores.
//
// One CTA per SM (persistent; tiles i, i + grid, ...), 22 warps:
//   warps 0-15 decode: thread (row r = tid % 128, part = tid / 128) turns
//              16 weights of its row into bf16 per 64-wide K chunk and stores
//              them (tcgen05.st) into its tensor-memory lane, where the MMA
//              reads its A operand (row = lane, two bf16 per column)
//   warps 18-21 epilogue: warp w reads tensor-memory lanes 32*(w%4)..+31
//              (weight rows) for all of the tile's tokens
//   warp 16    producer: per super-block, g tensor copies per weight matrix
//              (boxes of 128/g map rows of g weight rows each, from a 16-byte
//              boundary) and four of the tokens' bf16 rows (64 x 64,
//              128-byte swizzle)
//   warp 17    MMA: one thread issues tcgen05.mma (M=128, N = tokens rounded
//              up to 16, K=16, bf16 x bf16 -> fp32; A from tensor memory, B
//              from shared memory) and tcgen05.commit
// Tensor memory (512 columns): two accumulator buffers (64 fp32 columns per
// matrix), then a ring of 8 decoded 128 x 64 chunks (32 columns each).
// Pipelines (mbarriers, every wait bounded in time):
//   full/empty[3]     weight + token stages (producer -> decoders, MMA)
//   afull/aempty[8]   decoded chunks (decoders -> MMA)
//   tfull/tempty[2]   two accumulator buffers in tensor memory (MMA ->
//                     epilogue -> MMA), so the next tile's products start
//                     while the epilogue drains the last
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "engine.cuh"
#include "kernels.h"

namespace lb {

namespace {

constexpr int kPfM = 128;       // weight rows per tile (the MMA's M)
constexpr int kPfN = 64;        // tokens per tile
constexpr int kPfRing = 8;      // decoded chunks in flight (tensor memory)
constexpr int kPfStages = 3;    // weight + token stages (shared memory)
constexpr int kPfDecWarps = 16;
constexpr int kPfEpiWarps = 4;
constexpr int kPfThreads = (kPfDecWarps + 2 + kPfEpiWarps) * 32;
constexpr uint32_t kPfChunkCols = 32;            // 128 lanes x 64 bf16 (two per column)
constexpr uint32_t kPfTmemCols = 512;            // accumulators, then the decoded chunks
constexpr uint32_t kPfBoxBytes = kPfN * 128;     // 64 tokens x 64 bf16
constexpr uint32_t kPfBStage = 4 * kPfBoxBytes;  // one super-block of K
constexpr int kPfCarveMin = 64;                  // smallest max_tokens given prefill buffers
constexpr int kPfRouterSlices = 8;               // most K slices of the router GEMM

__host__ __device__ constexpr int pf_block_bytes(int wt) { return wt == LB_TYPE_Q4_K ? LB_Q4K : LB_Q6K; }
// Bytes of one staged row (the inner box of the weights' tensor map): a Q4_K
// super-block (144 bytes, always 16-byte aligned), or a Q6_K super-block with
// the 0-14 bytes before it down to a 16-byte boundary (210 + 14 = 224),
// rounded to 240: a 60-word row pitch puts a warp's rows on 8 distinct banks
// (a 56-word pitch on 4: 8-way conflicts on every decode load).
__host__ __device__ constexpr int pf_pitch(int wt) { return wt == LB_TYPE_Q4_K ? LB_Q4K : 240; }
__host__ __device__ constexpr uint32_t pf_wstage(int wt, int nmat) {
  return (uint32_t)(nmat * kPfM * pf_pitch(wt));
}

struct PfSync {
  uint64_t full[kPfStages], empty[kPfStages];
  uint64_t afull[kPfRing], aempty[kPfRing];
  uint64_t tfull[2], tempty[2], done;
  uint32_t tmem;
  int abort;
};

__host__ __device__ constexpr size_t pf_smem_bytes(int wt, int nmat) {
  return 1024 /* alignment slack */ + (size_t)kPfStages * kPfBStage +
         (size_t)kPfStages * pf_wstage(wt, nmat) + sizeof(PfSync);
}

// Tensor maps of one pass: the tokens' bf16 rows (64 x 64 boxes, 128-byte
// swizzle) and the weights (routed gate or up / down, routed up, the shared
// expert's), each viewed as a byte matrix whose rows are g weight rows, so
// the row pitch g * rb is a multiple of 16; a box is one super-block column
// (pf_pitch bytes from a 16-byte boundary) of 128 / g map rows.
struct PfMaps {
  CUtensorMap b, w0, w1, s0, s1;
};

// One pass (gate/up or down) of the prefill path.
struct PfPass {
  int g, g_sh;        // weight rows per tensor-map row
  long rb, rb_sh;     // row bytes
  int rows, rows_sh;  // rows of one expert matrix (valid rows of a tile)
  int nsb, nsb_sh;    // super-blocks per row
  const int4* tiles;  // {first grouped row, tokens, expert (-1 shared), row block}
  const int* ntiles;
  uint16_t* hs;       // gate/up output: bf16 [grouped row][ld_h]
  long ld_h;
  float* partial;     // down output: [T][k+1][H]
  const int* prow;    // partial row of each grouped row
  // Token dispatch across ranks (null otherwise): prow holds source rank << 24
  // | row, and the row lands in that rank's partial buffer over peer memory.
  float* const* partial_peers;
  int H;
  int* status;
};

// Bounded wait for the MMA thread: polls without suspending (one thread, so
// the polling costs one warp's issue slots), so a completed phase is seen at
// once; the clock is read every 64 polls.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n "
      "selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_spin_or_abort(uint64_t* bar, uint32_t parity, int* status,
                                                   volatile int* abort) {
  if (mbar_test(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    for (int i = 0; i < 64; ++i)
      if (mbar_test(bar, parity)) return true;
    if (*abort) return false;
    if (global_ns() - t0 >= kWaitLimitNs) break;
  }
  if (status) atomicOr(status, 2);
  *abort = 1;
  return false;
}

// ------------------------------------------------------------ tcgen05 PTX

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(dst)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
               : "memory");
}
// D[tmem] (+)= A[tmem] . B[smem]^T: A's rows in tensor-memory lanes 0-127,
// K along the columns (two bf16 per 32-bit column), K-major B.
__device__ __forceinline__ void tc_mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc,
                                          uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// 8 consecutive 32-bit columns of this thread's tensor-memory lane.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
      : "memory");
}
// Waits until this thread's tensor-memory stores are complete.
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// Arrives on bar once every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}
// 16 consecutive fp32 columns of this thread's tensor-memory lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];\n"
      "tcgen05.wait::ld.sync.aligned;"  // the registers are defined only after the wait
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor of a K-major operand in the 128-byte
// swizzled layout: rows of 128 bytes (64 bf16), groups of 8 rows 1024 bytes
// apart; p must be 1024-byte aligned (the swizzle phase is taken from the
// address).  Start address >> 4 in bits 0-13, stride-dimension offset
// (1024 >> 4) in bits 32-45, descriptor version 1 (bits 46-47), layout type
// 2 = 128-byte swizzle (bits 61-63).  Advancing K by 16 bf16 adds 32 bytes
// (2 in the start field).
__device__ __forceinline__ uint64_t sw128_desc(const void* p) {
  const uint32_t a = smem_addr(p);
  return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: fp32 accumulator (bits 4-5 = 1), A and
// B bf16 (bits 7-9 = 1, 10-12 = 1), both K-major, N >> 3 in bits 17-22,
// M >> 4 in bits 24-28.
__device__ __forceinline__ uint32_t mma_idesc(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(kPfM >> 4) << 24);
}

__device__ __forceinline__ uint32_t bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// N little-endian words from a 2-byte-aligned shared-memory address: N loads
// when it is word-aligned, else N + 1 aligned loads and a funnel shift each
// (the word after the run is read; the callers' runs end at least 4 bytes
// before the end of the staged row).
template <int N>
__device__ __forceinline__ void lds_run(const uint8_t* p, uint32_t* out) {
  const uint32_t a = smem_addr(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(p - (a & 3u));
  if ((a & 3u) == 0) {  // word-aligned run (warp-uniform for the prefill's staged rows)
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = w[i];
    return;
  }
  const uint32_t s = (a & 3u) * 8u;
  uint32_t v[N + 1];
#pragma unroll
  for (int i = 0; i <= N; ++i) v[i] = w[i];
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = __funnelshift_r(v[i], v[i + 1], s);
}

__device__ __forceinline__ __nv_bfloat162 as_bf2(uint32_t u) {
  __nv_bfloat162 r;
  memcpy(&r, &u, 4);
  return r;
}
__device__ __forceinline__ uint32_t as_u32(__nv_bfloat162 v) {
  uint32_t r;
  memcpy(&r, &v, 4);
  return r;
}

// Four 6- or 4-bit values q (bytes of v, each below 128) to two bf16 pairs
// (q0, q1), (q2, q3) minus `bias`, exactly: one PRMT puts a byte under the
// exponent byte 0x43, the bf16 number 128 + q, and a bf16 subtract of bias
// (128, or 160 = 128 + 32 for Q6_K's offset) leaves the small integer, which
// bf16 holds exactly.
__device__ __forceinline__ void q_pairs(uint32_t v, __nv_bfloat162 bias, __nv_bfloat162& a,
                                        __nv_bfloat162& b) {
  a = __hsub2(as_bf2(__byte_perm(v, 0x43434343u, 0x4140u)), bias);
  b = __hsub2(as_bf2(__byte_perm(v, 0x43434343u, 0x4342u)), bias);
}

// The scale factors of one thread's four chunks of a super-block (row part
// `part`: sub-blocks 2c + part/2 for Q4_K; scales 4c + part for Q6_K),
// computed once per super-block.  Q4_K: a = d*sc, b = -(dmin*m)
// (get-scale-min-k4-at, L4316-4336); Q6_K: a = d*sc.  Rounded to bf16.
struct SbScales {
  __nv_bfloat162 a[4], b[4];
};

// Small non-negative integer to float without a conversion instruction.
__device__ __forceinline__ float small_int_f(uint32_t v) {
  return __uint_as_float(0x4B000000u | v) - 8388608.0f;
}

// H = part / 2 (warp-uniform), a template argument so the sub-block indices
// and byte shifts are constants.
template <int WT, int H>
__device__ __forceinline__ void sb_scales(const uint8_t* blk, int part, SbScales& s) {
  constexpr int h = H;
  if (WT == LB_TYPE_Q4_K) {
    const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
    const float d = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      int sc, mn;
      q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * c + h, sc, mn);
      s.a[c] = __float2bfloat162_rn(d * small_int_f((uint32_t)sc));
      s.b[c] = __float2bfloat162_rn(-(dmin * small_int_f((uint32_t)mn)));
    }
  } else {
    const float d = half_bits_to_float(lds_u16(blk + 208));
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t w2 = lds_u16(blk + 192 + 4 * c + 2 * h);  // scales 4c + 2h, +1
      s.a[c] = __float2bfloat162_rn(d * (float)(int)(int8_t)((w2 >> (8 * (part & 1))) & 0xFFu));
      s.b[c] = s.a[c];
    }
  }
}

// 16 weights (K [64c + 16 part, +16) of the super-block at blk) as eight bf16
// pairs.  Q4_K: w = (d*sc)*q - dmin*m, one bf16 FMA per pair; Q6_K:
// w = (d*sc)*(q - 32), one bf16 multiply per pair.
template <int WT>
__device__ __forceinline__ void decode_chunk(const uint8_t* blk, int c, int part,
                                             const SbScales& s, uint32_t* o) {
  const int h = part >> 1, u = part & 1;
  if (WT == LB_TYPE_Q4_K) {
    // sub-block 2c + h: qs bytes [32c + 16u, +16), low nibbles (h = 0) or
    // high nibbles (h = 1)
    const __nv_bfloat162 k128 = as_bf2(0x43004300u);
    const uint4 q = *reinterpret_cast<const uint4*>(blk + 16 + 32 * c + 16 * u);
    const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
    const int sh = 4 * h;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 x0, x1;
      q_pairs((wd[i] >> sh) & 0x0F0F0F0Fu, k128, x0, x1);
      o[2 * i] = as_u32(__hfma2(x0, s.a[c], s.b[c]));
      o[2 * i + 1] = as_u32(__hfma2(x1, s.a[c], s.b[c]));
    }
  } else {
    // 128-half n = c / 2, quarter qd = 2 (c % 2) + h, l in [16u, 16u + 16):
    // ql bytes 64n + 32 (qd % 2) + l (low nibbles for qd < 2, high
    // otherwise), qh bytes 128 + 32n + l bits 2qd..2qd+1
    const int n = c >> 1, qd = (c & 1) * 2 + h;
    uint32_t ql[4], qh[4];
    lds_run<4>(blk + 64 * n + 32 * (qd & 1) + 16 * u, ql);
    lds_run<4>(blk + 128 + 32 * n + 16 * u, qh);
    const __nv_bfloat162 k160 = as_bf2(0x43204320u);
    const int shl = 4 * (qd >> 1), shh = 2 * qd;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      // q = ql nibble | qh 2 bits << 4 (below 64): no carry crosses a byte
      const uint32_t v = ((ql[i] >> shl) & 0x0F0F0F0Fu) + ((qh[i] >> shh) & 0x03030303u) * 16u;
      __nv_bfloat162 x0, x1;
      q_pairs(v, k160, x0, x1);
      o[2 * i] = as_u32(__hmul2(x0, s.a[c]));
      o[2 * i + 1] = as_u32(__hmul2(x1, s.a[c]));
    }
  }
}

// ------------------------------------------------------------ GEMM kernel
//
// PAIR: two weight matrices (gate, up) share the tokens; DOWN: the epilogue
// writes fp32 partial outputs instead of bf16 activations.
template <int WT, bool PAIR, bool DOWN>
__global__ void __launch_bounds__(kPfThreads, 1)
    pf_gemm_kernel(const __grid_constant__ PfMaps maps, const PfPass p) {
  constexpr int NMAT = PAIR ? 2 : 1;
  constexpr int BB = pf_block_bytes(WT), PITCH = pf_pitch(WT);
  constexpr uint32_t WSTAGE = pf_wstage(WT, NMAT);
  constexpr uint32_t ACC = NMAT * kPfN;  // columns of one accumulator buffer
  constexpr uint32_t ABASE = 2 * ACC;     // first column of the decoded-chunk ring
  constexpr int RING = kPfRing / NMAT;   // items (one K chunk of every matrix) in flight
  constexpr int RING_LOG = RING == 8 ? 3 : RING == 4 ? 2 : 1;
  static_assert((1 << RING_LOG) == RING, "ring of a power of two");
  static_assert(ABASE + kPfRing * kPfChunkCols <= kPfTmemCols, "tensor memory");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint8_t* b_st = smem;
  uint8_t* w_st = b_st + kPfStages * kPfBStage;
  PfSync* sy = reinterpret_cast<PfSync*>(w_st + kPfStages * WSTAGE);
  volatile int* abort = &sy->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(&sy->full[s], 1);
      mbar_init(&sy->empty[s], kPfDecWarps + 1);
    }
    for (int i = 0; i < kPfRing; ++i) {
      mbar_init(&sy->afull[i], kPfDecWarps);
      mbar_init(&sy->aempty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sy->tfull[b], 1);
      mbar_init(&sy->tempty[b], kPfEpiWarps);
    }
    mbar_init(&sy->done, 1);
    sy->abort = 0;
    fence_mbar_init();
  }
  if (warp == kPfDecWarps + 1) tmem_alloc(&sy->tmem, kPfTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sy->tmem;
  const int ntiles = *p.ntiles;

  if (warp == kPfDecWarps) {  // ------------------------------------ producer
    RingPos rp;
    int q = 0;
    uint32_t last_phase[kPfStages] = {};
    for (int tile = blockIdx.x; tile < ntiles && !*abort; tile += gridDim.x) {
      const int4 tl = p.tiles[tile];
      const bool sh = tl.z < 0;
      const int nsb = sh ? p.nsb_sh : p.nsb, rows = sh ? p.rows_sh : p.rows;
      const int g = sh ? p.g_sh : p.g, rows_g = kPfM / g;
      const long rb = sh ? p.rb_sh : p.rb;
      // this lane's box: matrix lane / g, weight rows j, j + g, ... (j = lane % g)
      const int mat = lane / g, j = lane - mat * g;
      const CUtensorMap* wm = mat == 0 ? (sh ? &maps.s0 : &maps.w0) : (sh ? &maps.s1 : &maps.w1);
      const int y = (int)(((sh ? 0L : (long)tl.z * rows) + (long)tl.w * kPfM) / g);
      for (int sb = 0; sb < nsb; ++sb) {
        if (q >= kPfStages &&
            !mbar_wait_or_abort(&sy->empty[rp.s], rp.phase ^ 1u, p.status, abort))
          break;
        uint8_t* wst = w_st + rp.s * WSTAGE;
        if (lane == 0) mbar_expect_tx(&sy->full[rp.s], WSTAGE + kPfBStage);
        __syncwarp();
        if (lane < NMAT * g) {
          const long x = (long)j * rb + (long)sb * BB;
          tma_load_2d(wst + (size_t)(mat * kPfM + j * rows_g) * PITCH, wm, (int)(x & ~15L), y,
                      &sy->full[rp.s]);
        }
        if (lane == 0)
#pragma unroll
          for (int c = 0; c < 4; ++c)
            tma_load_2d(b_st + rp.s * kPfBStage + c * kPfBoxBytes, &maps.b, sb * 256 + c * 64,
                        tl.x, &sy->full[rp.s]);
        last_phase[rp.s] = rp.phase;
        ++q;
        rp.next(kPfStages);
      }
    }
    // copies still in flight land before the CTA exits (bounded)
    for (int s = 0; s < kPfStages && s < q; ++s) mbar_wait(&sy->full[s], last_phase[s], nullptr);
  } else if (warp == kPfDecWarps + 1) {  // ---------------------------- MMA
    if (lane == 0) {
      RingPos rp;
      int auses = 0, it = 0;
      for (int tile = blockIdx.x; tile < ntiles && !*abort; tile += gridDim.x, ++it) {
        const int4 tl = p.tiles[tile];
        const int nsb = tl.z < 0 ? p.nsb_sh : p.nsb;
        const uint32_t idesc = mma_idesc((tl.y + 15) & ~15);
        const int buf = it & 1;
        const uint32_t dacc = tmem + buf * ACC;
        if (it >= 2 &&
            !mbar_spin_or_abort(&sy->tempty[buf], ((it >> 1) - 1) & 1, p.status, abort))
          break;
        tc_fence_after();
        bool ok = true;
        for (int sb = 0; sb < nsb && ok; ++sb) {
          if (!mbar_spin_or_abort(&sy->full[rp.s], rp.phase, p.status, abort)) {
            ok = false;
            break;
          }
          for (int c = 0; c < 4; ++c) {
            const int slot = auses & (RING - 1);
            if (!mbar_spin_or_abort(&sy->afull[slot], (auses >> RING_LOG) & 1, p.status, abort)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t bd = sw128_desc(b_st + rp.s * kPfBStage + c * kPfBoxBytes);
#pragma unroll
            for (int mat = 0; mat < NMAT; ++mat) {
              const uint32_t ad = tmem + ABASE + (slot * NMAT + mat) * kPfChunkCols;
#pragma unroll
              for (int j = 0; j < 4; ++j)  // K steps of 16: 8 columns of A, 32 bytes of B
                tc_mma_ts(dacc + mat * kPfN, ad + 8 * j, bd + 2 * j, idesc, (sb | c | j) != 0);
            }
            tc_commit(&sy->aempty[slot]);
            ++auses;
          }
          if (!ok) break;
          tc_commit(&sy->empty[rp.s]);
          rp.next(kPfStages);
        }
        if (!ok) break;
        tc_commit(&sy->tfull[buf]);
      }
      // every MMA issued has completed before the tensor memory is freed
      tc_commit(&sy->done);
      mbar_wait(&sy->done, 0, nullptr);
    }
    __syncwarp();
  } else if (warp < kPfDecWarps) {  // ------------------------------- decode
    const int tid = threadIdx.x, r = tid & (kPfM - 1), part = tid >> 7;
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;  // lanes r of this warp
    RingPos rp;
    int auses = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
      const int4 tl = p.tiles[tile];
      const bool sh = tl.z < 0;
      const int nsb = sh ? p.nsb_sh : p.nsb, rows = sh ? p.rows_sh : p.rows;
      const long rb = sh ? p.rb_sh : p.rb;
      const int r0 = tl.w * kPfM;
      const bool valid = r0 + r < rows;
      const int g = sh ? p.g_sh : p.g;
      const int jr = r % g;  // this row's box and its place in it
      const uint32_t srow = (uint32_t)(jr * (kPfM / g) + r / g) * PITCH;
      for (int sb = 0; sb < nsb && ok; ++sb) {
        if (!mbar_wait_or_abort(&sy->full[rp.s], rp.phase, p.status, abort)) {
          ok = false;
          break;
        }
        const uint8_t* wst = w_st + rp.s * WSTAGE;
        // the super-block's offset in its box row (the box starts 16-byte aligned)
        const uint32_t mis = (uint32_t)(((long)jr * rb + (long)sb * BB) & 15L);
        SbScales scl[NMAT];
        if (valid)
#pragma unroll
          for (int mat = 0; mat < NMAT; ++mat) {
            const uint8_t* blk = wst + (size_t)mat * kPfM * PITCH + srow + mis;
            if (part >> 1)  // warp-uniform
              sb_scales<WT, 1>(blk, part, scl[mat]);
            else
              sb_scales<WT, 0>(blk, part, scl[mat]);
          }
        for (int c = 0; c < 4; c += 2) {  // two items per wait for the stores
          const int slot = auses & (RING - 1);  // items auses, auses + 1: slots slot, slot + 1
          // the later slot's last use ends after the earlier one's (commits complete in order)
          if (auses + 1 >= RING &&
              !mbar_wait_or_abort(&sy->aempty[slot + 1], (((auses + 1) >> RING_LOG) - 1) & 1,
                                  p.status, abort)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int mat = 0; mat < NMAT; ++mat) {
              uint32_t o[8] = {0, 0, 0, 0, 0, 0, 0, 0};
              if (valid)
                decode_chunk<WT>(wst + (size_t)mat * kPfM * PITCH + srow + mis, c + i, part,
                                 scl[mat], o);
              tmem_st8(tmem + lane_base + ABASE + ((slot + i) * NMAT + mat) * kPfChunkCols +
                           8 * part,
                       o);
            }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&sy->afull[slot]);
            mbar_arrive(&sy->afull[slot + 1]);
          }
          auses += 2;
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&sy->empty[rp.s]);
        rp.next(kPfStages);
      }
      if (!ok) break;
    }
  } else {  // ------------------------------------------------------ epilogue
    const int q = warp & 3, r = 32 * q + lane;  // tensor-memory lanes of this warp
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    int it = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
      const int4 tl = p.tiles[tile];
      const int buf = it & 1;
      if (!mbar_wait_or_abort(&sy->tfull[buf], (it >> 1) & 1, p.status, abort)) break;
      tc_fence_after();
      const int ntok = tl.y;
      const int rows = tl.z < 0 ? p.rows_sh : p.rows;
      const int row = tl.w * kPfM + r;
      const uint32_t acc = tmem + lane_base + buf * ACC;
#pragma unroll 1
      for (int n0 = 0; n0 < ntok; n0 += 16) {  // warp-uniform
        float y0[16], y1[16];
        tmem_ld16(acc + n0, y0);
        if (PAIR) tmem_ld16(acc + kPfN + n0, y1);
        if (DOWN) {
          if (row < p.H) {
            if (p.partial_peers) {  // the source rank's partial row, over NVLink
#pragma unroll
              for (int j = 0; j < 16; ++j)
                if (n0 + j < ntok) {
                  const int pr = __ldg(p.prow + tl.x + n0 + j);
                  p.partial_peers[pr >> 24][(long)(pr & 0xFFFFFF) * p.H + row] = y0[j];
                }
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j)
                if (n0 + j < ntok)
                  p.partial[(long)__ldg(p.prow + tl.x + n0 + j) * p.H + row] = y0[j];
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (n0 + j < ntok) {
              float hv = 0.f;
              if (row < rows) {
                if (PAIR) {
                  hv = __fmul_rn(__fdividef(y0[j], 1.0f + __expf(-y0[j])), y1[j]);
                } else {
                  const float u = y0[j] > 0.f ? y0[j] : 0.f;
                  hv = __fmul_rn(u, u);
                }
              }
              const __nv_bfloat16 hb = __float2bfloat16_rn(hv);
              p.hs[(long)(tl.x + n0 + j) * p.ld_h + row] = *reinterpret_cast<const uint16_t*>(&hb);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sy->tempty[buf]);
    }
    // dispatch: this thread's stores to other ranks are performed before it
    // exits, so the flag raised after this launch orders behind them
    if (DOWN && p.partial_peers) __threadfence_system();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kPfDecWarps + 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kPfTmemCols);
  }
}

// ------------------------------------------------------------ gather + plan

// One CTA per token: the token's bf16 row (the rms-normed row when the layer
// has input_norm) copied to each grouped row it is routed to on this device,
// zero-padded from H to k_in.
__global__ void __launch_bounds__(256) pf_gather_kernel(MoeDevice m, MoeWork w,
                                                        const float* __restrict__ x, int T) {
  __shared__ int s_dst[33], s_prow[33], s_n;
  const int t = blockIdx.x, H = m.hidden, K = m.k_in, k = m.top_k;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* xt = (m.input_norm ? w.xn : x) + (long)t * H;  // rms-normed by pf_norm_kernel
  if (warp == 0) {
    int dst = -1;
    if (lane < k) {
      const int id = t * k + lane;
      const int e = w.sel[id];
      if (e >= m.expert_begin && e < m.expert_end) dst = w.offsets[e] + w.entries[id];
    }
    const unsigned own = __ballot_sync(0xffffffffu, dst >= 0);
    const int slot = __popc(own & ((1u << lane) - 1u));
    if (dst >= 0) {
      s_dst[slot] = dst;
      s_prow[slot] = t * (k + 1) + lane;
    }
    if (lane == 0) {
      int n = __popc(own);
      int t0, t1;
      shared_tokens(m, T, t0, t1);
      if (m.shared_here && m.inter_sh && t >= t0 && t < t1) {
        s_dst[n] = T * k + t;
        s_prow[n] = t * (k + 1) + k;
        ++n;
      }
      s_n = n;
    }
  }
  __syncthreads();
  const int nd = s_n;
  uint16_t* xs = w.pf_xs;
  for (int c0 = threadIdx.x * 8; c0 < K; c0 += blockDim.x * 8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = c0 + j;
      v[j] = i < H ? xt[i] : 0.f;
    }
    const uint4 pk = make_uint4(bf16x2(v[0], v[1]), bf16x2(v[2], v[3]), bf16x2(v[4], v[5]),
                                bf16x2(v[6], v[7]));
    for (int d = 0; d < nd; ++d)
      *reinterpret_cast<uint4*>(xs + (long)s_dst[d] * K + c0) = pk;
  }
  if (threadIdx.x < nd) w.pf_prow[s_dst[threadIdx.x]] = s_prow[threadIdx.x];
}

// Tile lists of both passes, in expert order (then the shared expert): for
// each active expert, its row blocks, each with its 64-token chunks in a row,
// so CTAs running side by side read the same weight rows.
// shared_base: the grouped row of the shared expert's first token (T*k when
// this device routed its own T tokens; the dispatch path's fixed base).
__global__ void __launch_bounds__(1024) pf_plan_kernel(MoeDevice m, MoeWork w, int T,
                                                       int shared_base) {
  __shared__ int s_warp[32];
  const int E = m.experts, na = w.active[E];
  const int a = threadIdx.x, warp = a >> 5, lane = a & 31;
  int e = -1, cnt = 0, nch = 0;
  if (a < na) {
    e = w.active[a];
    cnt = w.counts[e];
    nch = (cnt + kPfN - 1) / kPfN;
  }
  int incl = nch;  // inclusive scan over the block
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int v = s_warp[lane], iv = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, iv, o);
      if (lane >= o) iv += u;
    }
    s_warp[lane] = iv - v;  // exclusive
  }
  __syncthreads();
  const int base = s_warp[warp] + incl - nch;  // chunks of the active experts before a
  __shared__ int s_total;
  if (a == blockDim.x - 1) s_total = base + nch;
  __syncthreads();
  const int routed = s_total;
  const int mbu = m.k_down / kPfM, mbd = (m.hidden + kPfM - 1) / kPfM;
  int4* up = w.pf_tiles;
  int4* dn = w.pf_tiles + w.pf_max_up;
  if (a < na) {
    const int off = w.offsets[e];
    for (int mb = 0; mb < mbu; ++mb)
      for (int ch = 0; ch < nch; ++ch)
        up[(long)base * mbu + mb * nch + ch] =
            make_int4(off + ch * kPfN, min(kPfN, cnt - ch * kPfN), e, mb);
    for (int mb = 0; mb < mbd; ++mb)
      for (int ch = 0; ch < nch; ++ch)
        dn[(long)base * mbd + mb * nch + ch] =
            make_int4(off + ch * kPfN, min(kPfN, cnt - ch * kPfN), e, mb);
  }
  int nsh = 0, mbu_sh = 0, t0 = 0, t1 = 0;
  if (m.shared_here && m.inter_sh) {
    shared_tokens(m, T, t0, t1);
    nsh = (t1 - t0 + kPfN - 1) / kPfN;
    mbu_sh = m.k_down_sh / kPfM;
  }
  for (int i = a; i < nsh * mbu_sh; i += blockDim.x) {
    const int mb = i / nsh, ch = i - mb * nsh;
    up[(long)routed * mbu + i] =
        make_int4(shared_base + t0 + ch * kPfN, min(kPfN, t1 - t0 - ch * kPfN), -1, mb);
  }
  for (int i = a; i < nsh * mbd; i += blockDim.x) {
    const int mb = i / nsh, ch = i - mb * nsh;
    dn[(long)routed * mbd + i] =
        make_int4(shared_base + t0 + ch * kPfN, min(kPfN, t1 - t0 - ch * kPfN), -1, mb);
  }
  if (a == 0) {
    w.pf_count[0] = routed * mbu + nsh * mbu_sh;
    w.pf_count[1] = (routed + nsh) * mbd;
  }
}

// ------------------------------------------------------------ router

// rms-norm-into (llambda.lisp L859-879) of every token into w.xn: scale =
// 1/sqrt(mean(x^2) + eps), xn = (x * weight) * scale.  One CTA per token,
// the row held in registers between the sum and the scaling.
__global__ void __launch_bounds__(256) pf_norm_kernel(MoeDevice m, MoeWork w,
                                                      const float* __restrict__ x, int T) {
  constexpr int kPer = 16;  // values per thread held in registers (H <= 4096)
  __shared__ float s_red[8];
  const int t = blockIdx.x, H = m.hidden, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* xt = x + (long)t * H;
  float v[kPer];
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int i = threadIdx.x + j * 256;
    v[j] = i < H ? xt[i] : 0.f;
    acc = fmaf(v[j], v[j], acc);
  }
  for (int i = threadIdx.x + kPer * 256; i < H; i += 256) acc = fmaf(xt[i], xt[i], acc);
  acc = warp_sum(acc);
  if (lane == 0) s_red[warp] = acc;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) tot += s_red[q];
  const float scale =
      __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)H), m.norm_epsilon)));
  float* o = w.xn + (long)t * H;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int i = threadIdx.x + j * 256;
    if (i < H) o[i] = __fmul_rn(__fmul_rn(v[j], m.input_norm[i]), scale);
  }
  for (int i = threadIdx.x + kPer * 256; i < H; i += 256)
    o[i] = __fmul_rn(__fmul_rn(xt[i], m.input_norm[i]), scale);
}

constexpr int kRtTok = 128, kRtRows = 64, kRtK = 32;

// tf32 value of an fp32 (its top 10 mantissa bits) and the rest
__device__ __forceinline__ uint32_t tf32_hi(float v) { return __float_as_uint(v) & 0xFFFFE000u; }
__device__ __forceinline__ uint32_t tf32_lo(float v) {
  return __float_as_uint(v - __uint_as_float(tf32_hi(v))) & 0xFFFFE000u;
}

__device__ __forceinline__ void mma_tf32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Router logits of a prefill batch (dot-product-with-f32-tensor-data,
// L4096-4107, for every router row; row E of the logits is the qwen3next
// shared-expert gate, L3491-3500) on the tensor cores in three-pass tf32:
// every fp32 operand is split into a tf32 high part and a tf32 part of the
// rest, and each product is accumulated as lo*hi + hi*lo + hi*hi (the
// dropped lo*lo and the truncations leave about 2^-21 of each product), fp32
// accumulation.  A CTA takes 128 tokens x 64 rows over one K slice, K in
// chunks of 32 staged through shared memory (the next chunk's float4 loads
// in flight during the current one's mma); warp (wm, wn) of 4 x 2 takes 32
// tokens x 32 rows, mma.m16n8k8: A = the tokens (rows of xs), B = the router
// rows (rows of ws), rows 36 floats apart so the fragment loads of a warp
// hit 32 distinct banks.  (The fp32 FMA form of the same tiling ran at 32
// TFLOP/s: 134 us at batch 2048.)
__global__ void __launch_bounds__(256) pf_router_kernel(MoeDevice m, MoeWork w,
                                                        const float* __restrict__ xr, int T,
                                                        int all_rows, int kc) {
  constexpr int P = kRtK + 4;  // row pitch (floats)
  __shared__ __align__(16) float xs[kRtTok][P];
  __shared__ __align__(16) float ws[kRtRows][P];
  const int t0 = blockIdx.y * kRtTok, r0 = blockIdx.x * kRtRows;
  // K slice blockIdx.z of kc values (gridDim.z slices; one: the whole row)
  const int kb = blockIdx.z * kc, K = min(m.hidden - kb, kc);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3, wm = warp & 3, wn = warp >> 2;
  // staging: token row tid/2 (16 values from (tid&1)*16), router row tid/4 (8 from (tid&3)*8)
  const int xr_row = tid >> 1, xk = (tid & 1) * 16, wr_row = tid >> 2, wk = (tid & 3) * 8;
  const float* xrow = xr + (long)min(t0 + xr_row, T - 1) * m.hidden + kb;
  const int rr = min(r0 + wr_row, all_rows - 1);
  const float* wrow =
      (rr < m.router_rows ? m.router + (long)rr * m.hidden : m.router_extra_row) + kb;
  const bool vec = ((m.hidden | kb) & 3) == 0 &&
                   ((reinterpret_cast<uintptr_t>(xr) | reinterpret_cast<uintptr_t>(m.router) |
                     reinterpret_cast<uintptr_t>(m.router_extra_row)) & 15) == 0;
  float acc[2][4][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[i][j][c] = 0.f;
  float xv[16], wv[8];
  auto fetch = [&](int k0) {
    if (vec && k0 + kRtK <= K) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(xrow + k0 + xk) + j);
        xv[4 * j] = v.x, xv[4 * j + 1] = v.y, xv[4 * j + 2] = v.z, xv[4 * j + 3] = v.w;
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(wrow + k0 + wk) + j);
        wv[4 * j] = v.x, wv[4 * j + 1] = v.y, wv[4 * j + 2] = v.z, wv[4 * j + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) xv[j] = k0 + xk + j < K ? __ldg(xrow + k0 + xk + j) : 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) wv[j] = k0 + wk + j < K ? __ldg(wrow + k0 + wk + j) : 0.f;
    }
  };
  fetch(0);
  for (int k0 = 0; k0 < K; k0 += kRtK) {
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<float4*>(&xs[xr_row][xk + 4 * j]) =
          make_float4(xv[4 * j], xv[4 * j + 1], xv[4 * j + 2], xv[4 * j + 3]);
#pragma unroll
    for (int j = 0; j < 2; ++j)
      *reinterpret_cast<float4*>(&ws[wr_row][wk + 4 * j]) =
          make_float4(wv[4 * j], wv[4 * j + 1], wv[4 * j + 2], wv[4 * j + 3]);
    __syncthreads();
    if (k0 + kRtK < K) fetch(k0 + kRtK);
#pragma unroll
    for (int ks = 0; ks < kRtK; ks += 8) {
      uint32_t ah[2][4], al[2][4], bh[4][2], bl[4][2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int mr = wm * 32 + i * 16 + g;
        const float a[4] = {xs[mr][ks + t], xs[mr + 8][ks + t], xs[mr][ks + t + 4],
                            xs[mr + 8][ks + t + 4]};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          ah[i][c] = tf32_hi(a[c]);
          al[i][c] = tf32_lo(a[c]);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int nr = wn * 32 + j * 8 + g;
        const float b[2] = {ws[nr][ks + t], ws[nr][ks + t + 4]};
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          bh[j][c] = tf32_hi(b[c]);
          bl[j][c] = tf32_lo(b[c]);
        }
      }
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          mma_tf32(acc[i][j], al[i][0], al[i][1], al[i][2], al[i][3], bh[j][0], bh[j][1]);
          mma_tf32(acc[i][j], ah[i][0], ah[i][1], ah[i][2], ah[i][3], bl[j][0], bl[j][1]);
          mma_tf32(acc[i][j], ah[i][0], ah[i][1], ah[i][2], ah[i][3], bh[j][0], bh[j][1]);
        }
    }
  }
  const int E1 = m.experts + 1;
  float* dst = gridDim.z == 1 ? w.logits : w.pf_rlog + (long)blockIdx.z * T * E1;
  // D of tile (i, j): [0] token g, row 2t; [1] token g, row 2t+1; [2], [3] token g+8
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int tok = t0 + wm * 32 + i * 16 + g + 8 * h;
      if (tok >= T) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int r = r0 + wn * 32 + j * 8 + 2 * t + c;
          if (r < all_rows) dst[(long)tok * E1 + r] = acc[i][j][2 * h + c];
        }
    }
}

// logits = the K slices' partial logits summed in slice order.
__global__ void __launch_bounds__(256) pf_router_sum_kernel(MoeDevice m, MoeWork w, int T,
                                                            int all_rows, int slices) {
  const int E1 = m.experts + 1;
  const long n = (long)T * E1;
  for (long i = blockIdx.x * 256L + threadIdx.x; i < n; i += (long)gridDim.x * 256) {
    if ((int)(i % E1) >= all_rows) continue;
    float v = w.pf_rlog[i];
    for (int z = 1; z < slices; ++z) v = __fadd_rn(v, w.pf_rlog[(long)z * n + i]);
    w.logits[i] = v;
  }
}

// ------------------------------------------------------------ host side

std::atomic<int> g_prefill_min{128};

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return encode;
}

// bf16 rows [rows][cols] (row pitch cols * 2 bytes), 64 x 64 boxes with the
// 128-byte swizzle; rows past the end read as zeros.
bool bf16_rows_map(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows) {
  const auto encode = tensor_map_encoder();
  if (!encode || rows == 0 || (cols * 2) % 16) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)kPfN};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int pf_down_ld(const MoeDevice& m) {
  return std::max(m.k_down, m.shared_here && m.inter_sh ? m.k_down_sh : 0);
}

void pf_tile_bounds(const MoeDevice& m, int T, long* max_up, long* max_dn) {
  const long entries = (long)T * m.top_k;
  const long owned = std::max(1, m.expert_end - m.expert_begin);
  const long chunks_r = entries / kPfN + std::min(owned, entries) + 1;
  const long chunks_sh = m.shared_here && m.inter_sh ? (T + kPfN - 1) / kPfN : 0;
  const long mbu = m.k_down / kPfM, mbd = (m.hidden + kPfM - 1) / kPfM;
  const long mbu_sh = m.shared_here && m.inter_sh ? m.k_down_sh / kPfM : 0;
  *max_up = chunks_r * mbu + chunks_sh * mbu_sh;
  *max_dn = (chunks_r + chunks_sh) * mbd;
}

bool q_type(int t) { return t == LB_TYPE_Q4_K || t == LB_TYPE_Q6_K; }

// Weight rows per tensor-map row: the smallest g in 1, 2, 4, 8 with g * rb a
// multiple of 16 bytes that divides the tensor's rows and one expert's rows
// (a Q6_K row of n super-blocks is 2n mod 16 bytes); 0 if none.
int pf_group(long rb, long rows_total, long rows_e) {
  for (int g = 1; g <= 8; g *= 2)
    if ((g * rb) % 16 == 0 && rows_total % g == 0 && rows_e % g == 0) return g;
  return 0;
}

bool pf_weight_map(CUtensorMap* map, const uint8_t* base, long rb, long rows_total, int g,
                   int pitch) {
  const auto encode = tensor_map_encoder();
  if (!encode || !base || !g || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)(g * rb), (cuuint64_t)(rows_total / g)};
  const cuuint64_t strides[1] = {(cuuint64_t)(g * rb)};
  const cuuint32_t box[2] = {(cuuint32_t)pitch, (cuuint32_t)(kPfM / g)};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(base), dims, strides,
                box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool weights_ok(const uint8_t* base, long rb, long rows_total, long rows_e) {
  return base && (reinterpret_cast<uintptr_t>(base) & 15) == 0 &&
         pf_group(rb, rows_total, rows_e) != 0;
}

template <int WT, bool PAIR, bool DOWN>
cudaError_t launch_pf_gemm(const PfMaps& maps, const PfPass& p, cudaStream_t s) {
  auto kern = pf_gemm_kernel<WT, PAIR, DOWN>;
  const size_t smem = pf_smem_bytes(WT, PAIR ? 2 : 1);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<sm_count(), kPfThreads, smem, s>>>(maps, p);
  return cudaGetLastError();
}

template <bool DOWN>
cudaError_t launch_pf_pass(int wt, bool pair, const PfMaps& maps, const PfPass& p,
                           cudaStream_t s) {
  if (wt == LB_TYPE_Q4_K)
    return pair ? launch_pf_gemm<LB_TYPE_Q4_K, true, DOWN>(maps, p, s)
                : launch_pf_gemm<LB_TYPE_Q4_K, false, DOWN>(maps, p, s);
  return pair ? launch_pf_gemm<LB_TYPE_Q6_K, true, DOWN>(maps, p, s)
              : launch_pf_gemm<LB_TYPE_Q6_K, false, DOWN>(maps, p, s);
}

}  // namespace

void set_prefill_min_tokens(int n) { g_prefill_min.store(std::max(kPfCarveMin, n)); }
int prefill_min_tokens() { return g_prefill_min.load(); }

size_t prefill_work_bytes(const MoeDevice& m, int T, size_t* parts) {
  if (T < kPfCarveMin) {
    for (int i = 0; i < 6; ++i) parts[i] = 0;
    return 0;
  }
  const long rows = (long)T * m.top_k + T;
  long max_up, max_dn;
  pf_tile_bounds(m, T, &max_up, &max_dn);
  parts[0] = (size_t)rows * m.k_in * 2;          // xs
  parts[1] = (size_t)rows * pf_down_ld(m) * 2;   // hs
  parts[2] = (size_t)rows * 4;                   // prow
  parts[3] = (size_t)(max_up + max_dn) * 16;     // tiles
  parts[4] = 16;                                 // counts
  parts[5] = (size_t)kPfRouterSlices * T * (m.experts + 1) * 4;  // router K-slice logits
  size_t total = 0;
  for (int i = 0; i < 6; ++i) total += (parts[i] + 255) & ~size_t(255);
  return total;
}

long prefill_max_up_tiles(const MoeDevice& m, int T) {
  long max_up, max_dn;
  pf_tile_bounds(m, T, &max_up, &max_dn);
  return max_up;
}

cudaError_t launch_prefill_router(const MoeDevice& m, const MoeWork& w, const float* x, int T,
                                  cudaStream_t s) {
  cudaError_t e;
  if (m.input_norm) {
    pf_norm_kernel<<<T, 256, 0, s>>>(m, w, x, T);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  const int all_rows = m.router_rows + (m.router_extra_row ? 1 : 0);
  const int tiles = ((all_rows + kRtRows - 1) / kRtRows) * ((T + kRtTok - 1) / kRtTok);
  // K slices so that about four CTAs run per SM, each slice a multiple of 32
  int slices = std::min(kPfRouterSlices, std::max(1, (4 * sm_count() + tiles - 1) / tiles));
  int kc = (m.hidden + slices - 1) / slices;
  kc = (kc + kRtK - 1) / kRtK * kRtK;
  slices = (m.hidden + kc - 1) / kc;
  dim3 grid((all_rows + kRtRows - 1) / kRtRows, (T + kRtTok - 1) / kRtTok, slices);
  pf_router_kernel<<<grid, 256, 0, s>>>(m, w, m.input_norm ? w.xn : x, T, all_rows, kc);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if (slices > 1) {
    const long n = (long)T * (m.experts + 1);
    pf_router_sum_kernel<<<(int)std::min<long>((n + 255) / 256, 4L * sm_count()), 256, 0, s>>>(
        m, w, T, all_rows, slices);
  }
  return cudaGetLastError();
}

bool prefill_applies(const MoeDevice& m, const MoeWork& w, int T) {
  if (T < g_prefill_min.load() || !w.pf_xs || T > w.max_tokens) return false;
  if (m.ep_world > 1) return false;
  if (!q_type(m.up_type) || !q_type(m.down_type)) return false;
  const bool pair = m.arch == 0;
  if (pair && m.gate_type != m.up_type) return false;
  const long E = m.experts;
  if (!weights_ok(m.up_exps, (long)m.up_rb, E * m.inter, m.inter)) return false;
  if (pair && !weights_ok(m.gate_exps, (long)m.gate_rb, E * m.inter, m.inter)) return false;
  if (!weights_ok(m.down_exps, (long)m.down_rb, E * m.hidden, m.hidden)) return false;
  if (m.shared_here && m.inter_sh) {
    if (m.up_sh_type != m.up_type || m.down_sh_type != m.down_type) return false;
    if (pair && m.gate_sh_type != m.gate_type) return false;
    if (m.k_in_sh != m.k_in) return false;
    if (!weights_ok(m.up_sh, (long)m.up_sh_rb, m.inter_sh, m.inter_sh)) return false;
    if (pair && !weights_ok(m.gate_sh, (long)m.gate_sh_rb, m.inter_sh, m.inter_sh)) return false;
    if (!weights_ok(m.down_sh, (long)m.down_sh_rb, m.hidden, m.hidden)) return false;
  }
  constexpr size_t kSmemMax = 227 * 1024;
  if (pf_smem_bytes(m.up_type, pair ? 2 : 1) > kSmemMax || pf_smem_bytes(m.down_type, 1) > kSmemMax)
    return false;
  return (m.k_in % 256) == 0 && (m.k_down % 256) == 0;
}

namespace {

// Plan, gate/up and down passes over the grouped rows already in w.pf_xs
// (the routed entries, then T shared-expert rows from shared_base on).
// partial_peers: the token dispatch's partial regions of every rank (the
// down pass stores each row into its source rank's), or null.
cudaError_t pf_gemm_passes(const MoeDevice& m, const MoeWork& w, int T, int shared_base,
                           float* const* partial_peers, cudaStream_t s,
                           const cudaEvent_t* marks) {
  cudaError_t e;
  auto mark = [&](int i) { return marks ? cudaEventRecord(marks[i], s) : cudaSuccess; };
  pf_plan_kernel<<<1, 1024, 0, s>>>(m, w, T, shared_base);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  const long rows = (long)shared_base + T;
  const int ld_h = pf_down_ld(m);
  const bool pair = m.arch == 0;
  const bool shared = m.shared_here && m.inter_sh;
  const long E = m.experts;
  const int pq_up = pf_pitch(m.up_type), pq_dn = pf_pitch(m.down_type);
  PfMaps um, dm;
  PfPass up{}, dn{};
  up.g = pf_group((long)m.up_rb, E * m.inter, m.inter);
  dn.g = pf_group((long)m.down_rb, E * m.hidden, m.hidden);
  if (!bf16_rows_map(&um.b, w.pf_xs, m.k_in, rows) || !bf16_rows_map(&dm.b, w.pf_hs, ld_h, rows) ||
      !pf_weight_map(&um.w0, pair ? m.gate_exps : m.up_exps, (long)m.up_rb, E * m.inter, up.g,
                     pq_up) ||
      !pf_weight_map(&um.w1, m.up_exps, (long)m.up_rb, E * m.inter, up.g, pq_up) ||
      !pf_weight_map(&dm.w0, m.down_exps, (long)m.down_rb, E * m.hidden, dn.g, pq_dn))
    return cudaErrorInvalidValue;
  dm.w1 = dm.w0;
  if (shared) {
    up.g_sh = pf_group((long)m.up_sh_rb, m.inter_sh, m.inter_sh);
    dn.g_sh = pf_group((long)m.down_sh_rb, m.hidden, m.hidden);
    if (!pf_weight_map(&um.s0, pair ? m.gate_sh : m.up_sh, (long)m.up_sh_rb, m.inter_sh, up.g_sh,
                       pq_up) ||
        !pf_weight_map(&um.s1, m.up_sh, (long)m.up_sh_rb, m.inter_sh, up.g_sh, pq_up) ||
        !pf_weight_map(&dm.s0, m.down_sh, (long)m.down_sh_rb, m.hidden, dn.g_sh, pq_dn))
      return cudaErrorInvalidValue;
    dm.s1 = dm.s0;
  } else {  // no shared tiles: the maps are never read
    up.g_sh = up.g;
    dn.g_sh = dn.g;
    um.s0 = um.w0;
    um.s1 = um.w1;
    dm.s0 = dm.s1 = dm.w0;
  }
  if ((e = mark(0)) != cudaSuccess) return e;
  up.rb = (long)m.up_rb;
  up.rb_sh = shared ? (long)m.up_sh_rb : 0;
  up.rows = m.inter;
  up.rows_sh = shared ? m.inter_sh : 0;
  up.nsb = m.k_in / 256;
  up.nsb_sh = m.k_in / 256;
  up.tiles = w.pf_tiles;
  up.ntiles = w.pf_count;
  up.hs = w.pf_hs;
  up.ld_h = ld_h;
  up.H = m.hidden;
  up.status = w.status;
  if ((e = launch_pf_pass<false>(m.up_type, pair, um, up, s)) != cudaSuccess) return e;
  if ((e = mark(1)) != cudaSuccess) return e;
  dn.rb = (long)m.down_rb;
  dn.rb_sh = shared ? (long)m.down_sh_rb : 0;
  dn.rows = m.hidden;
  dn.rows_sh = m.hidden;
  dn.nsb = m.k_down / 256;
  dn.nsb_sh = shared ? m.k_down_sh / 256 : 0;
  dn.tiles = w.pf_tiles + w.pf_max_up;
  dn.ntiles = w.pf_count + 1;
  dn.partial = w.partial;
  dn.prow = w.pf_prow;
  dn.partial_peers = partial_peers;
  dn.H = m.hidden;
  dn.status = w.status;
  if ((e = launch_pf_pass<true>(m.down_type, false, dm, dn, s)) != cudaSuccess) return e;
  return mark(2);
}

}  // namespace

cudaError_t launch_prefill_passes(const MoeDevice& m, const MoeWork& w, const float* x, int T,
                                  cudaStream_t s, const cudaEvent_t* marks) {
  cudaError_t e;
  if (m.experts > 1024) return cudaErrorInvalidValue;
  pf_gather_kernel<<<T, 256, 0, s>>>(m, w, x, T);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  return pf_gemm_passes(m, w, T, T * m.top_k, nullptr, s, marks);
}

// ------------------------------------------------------------ token dispatch
//
// Expert-parallel prefill: every rank holds a share of the tokens and a share
// of the experts.  Per layer call, each rank normalises and routes its own
// tokens, then (one CTA per token) stores the token's bf16 row into the
// landing zone of each rank that owns one of its experts, over NVLink peer
// memory, with the expert and the token's partial row beside it; the last CTA
// raises one epoch-tagged flag per destination carrying the entry count,
// after a single system-scope fence.  Each rank waits (bounded) for every
// source's flag, groups what it received by expert, copies the rows into the
// grouped layout the tcgen05 GEMMs read, and runs the gate/up and down passes;
// the down pass's epilogue stores every output row straight into its source
// rank's partial buffer.  A done flag per rank then lets each source combine
// its own tokens (weights, shared expert, residual) exactly as on one device.
// A rank sends rows of call n + 1 only after its combine of call n, which
// waited for every rank's done flag of call n, so no landing zone or partial
// buffer is overwritten while it is read.

__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_sys_acq_rel() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Waits (bounded) until flag >> 32 == epoch; returns the low 32 bits, or -1
// after the time limit (status bit 2, value 4).
__device__ int dx_wait_flag(const uint64_t* flag, uint32_t epoch, int* status) {
  const uint64_t t0 = global_ns();
  for (;;) {
    const uint64_t v = ld_relaxed_sys_u64(flag);
    if ((uint32_t)(v >> 32) == epoch) {
      fence_sys_acq_rel();
      return (int)(v & 0xFFFFFFFFu);
    }
    if (global_ns() - t0 > kWaitLimitNs) {
      atomicOr(status, 4);
      return -1;
    }
    __nanosleep(32);
  }
}

// The rank owning expert e: rank q holds [q*E/world, (q+1)*E/world).
__device__ __forceinline__ int dx_owner(const MoeDevice& m, int e) {
  int q = m.dx_world - 1;
  while (q > 0 && (long)q * m.experts / m.dx_world > e) --q;
  return q;
}

__global__ void __launch_bounds__(256) dx_send_kernel(MoeDevice m, MoeWork w,
                                                      const float* __restrict__ x, int T) {
  __shared__ int s_q[32], s_pos[32];
  __shared__ uint32_t s_epoch;
  __shared__ int s_last;
  const int t = blockIdx.x, k = m.top_k, H = m.hidden, K = m.k_in, me = m.dx_rank;
  uint32_t* hdr = static_cast<uint32_t*>(m.dx_peers[me]);
  const DxLayout L = dx_layout(m.dx_world, m.dx_cap, k, K, H);
  const size_t src_base = (size_t)me * m.dx_cap * k;  // this rank's slots at a destination
  if (threadIdx.x == 0) s_epoch = hdr[0] + 1u;  // the last CTA advances hdr[0]
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int q = -1, pos = 0;
    if (lane < k) {
      const int id = t * k + lane;
      const int e = w.sel[id];
      if (e >= 0 && e < m.experts) {  // an unselectable rank (status bit 0) sends nothing
        q = dx_owner(m, e);
        pos = (int)atomicAdd(&hdr[2 + q], 1u);
        int2* meta = reinterpret_cast<int2*>(static_cast<uint8_t*>(m.dx_peers[q]) + L.meta);
        meta[src_base + pos] = make_int2(e, t * (k + 1) + lane);
      }
    }
    s_q[lane] = q;
    s_pos[lane] = pos;
  }
  __syncthreads();
  const float* xt = (m.input_norm ? w.xn : x) + (long)t * H;
  for (int c0 = threadIdx.x * 8; c0 < K; c0 += blockDim.x * 8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = c0 + j < H ? xt[c0 + j] : 0.f;
    const uint4 pk = make_uint4(bf16x2(v[0], v[1]), bf16x2(v[2], v[3]), bf16x2(v[4], v[5]),
                                bf16x2(v[6], v[7]));
    for (int j = 0; j < k; ++j) {
      const int q = s_q[j];
      if (q < 0) continue;
      uint16_t* rows = reinterpret_cast<uint16_t*>(static_cast<uint8_t*>(m.dx_peers[q]) + L.rows);
      *reinterpret_cast<uint4*>(rows + (src_base + s_pos[j]) * K + c0) = pk;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // this CTA's rows and entries before its arrival
    s_last = atomicAdd(&hdr[1], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last || threadIdx.x != 0) return;
  __threadfence();
  const uint32_t epoch = s_epoch;
  for (int q = 0; q < m.dx_world; ++q) {
    const uint32_t cnt = atomicExch(&hdr[2 + q], 0u);
    uint64_t* dflag = reinterpret_cast<uint64_t*>(static_cast<uint8_t*>(m.dx_peers[q]) + 64) + me;
    st_relaxed_sys_u64(dflag, ((uint64_t)epoch << 32) | cnt);
  }
  hdr[1] = 0;
  hdr[0] = epoch;
}

// One CTA: waits for every source's rows, groups the received entries by
// owned expert (counts, offsets, active list as the routing writes them for
// the tile plan), and maps each grouped row to its landing slot (second half
// of w.entries) and to its source's partial row (pf_prow: source << 24 | row).
// The order of entries inside an expert's group does not matter: each row's
// products depend on that row alone.
__global__ void __launch_bounds__(1024) dx_group_kernel(MoeDevice m, MoeWork w, int T,
                                                        int shared_base) {
  __shared__ int s_cnt[kEpMaxWorld + 1], s_base[kEpMaxWorld + 1];
  __shared__ int s_count[1024], s_warp[32], s_wact[32];
  const int E = m.experts, k = m.top_k, W = m.dx_world, me = m.dx_rank;
  const int eb = m.expert_begin, ne = m.expert_end - m.expert_begin;
  const uint8_t* self = static_cast<const uint8_t*>(m.dx_peers[me]);
  const uint32_t epoch = reinterpret_cast<const uint32_t*>(self)[0];
  const DxLayout L = dx_layout(W, m.dx_cap, k, m.k_in, m.hidden);
  const int2* meta = reinterpret_cast<const int2*>(self + L.meta);
  const long nk = (long)w.max_tokens * k;
  if (threadIdx.x < W) {
    const int c = dx_wait_flag(reinterpret_cast<const uint64_t*>(self + 64) + threadIdx.x, epoch,
                               w.status);
    s_cnt[threadIdx.x] = c < 0 ? 0 : min(c, m.dx_cap * k);
  }
  for (int e = threadIdx.x; e < ne; e += blockDim.x) s_count[e] = 0;
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int q = 0; q < W; ++q) {
      s_base[q] = run;
      run += s_cnt[q];
    }
    s_base[W] = run;
  }
  __syncthreads();
  const int M = s_base[W];
  for (int i = threadIdx.x; i < M; i += blockDim.x) {  // slot of each entry in its expert
    int q = 0;
    while (i >= s_base[q + 1]) ++q;
    const int e = meta[(size_t)q * m.dx_cap * k + (i - s_base[q])].x - eb;
    w.entries[i] = (e >= 0 && e < ne) ? atomicAdd(&s_count[e], 1) : -1;
  }
  __syncthreads();
  // exclusive scans over the owned experts: entry offsets and the active list
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = threadIdx.x;
  const int cnt = e < ne ? s_count[e] : 0;
  int incl = cnt, act = cnt > 0 ? 1 : 0;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    const int a = __shfl_up_sync(0xffffffffu, act, o);
    if (lane >= o) {
      incl += v;
      act += a;
    }
  }
  if (lane == 31) {
    s_warp[warp] = incl;
    s_wact[warp] = act;
  }
  __syncthreads();
  int wbase = 0, abase = 0;
  for (int q = 0; q < warp; ++q) {
    wbase += s_warp[q];
    abase += s_wact[q];
  }
  const int off = wbase + incl - cnt;
  __syncthreads();
  if (e < ne) {
    w.counts[eb + e] = cnt;
    w.offsets[eb + e] = off;
    if (cnt > 0) w.active[abase + act - 1] = eb + e;
    s_count[e] = off;  // from here: the expert's first grouped row
  }
  if (threadIdx.x == blockDim.x - 1) {
    w.active[E] = abase + act;
    w.offsets[E] = M;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < M; i += blockDim.x) {
    int q = 0;
    while (i >= s_base[q + 1]) ++q;
    const int slot = i - s_base[q];
    const int2 mt = meta[(size_t)q * m.dx_cap * k + slot];
    const int pos = w.entries[i];
    // a source's partial row lies inside its [cap][k+1] region
    if (pos < 0 || mt.y < 0 || mt.y >= m.dx_cap * (k + 1)) continue;
    const int g = s_count[mt.x - eb] + pos;
    w.entries[nk + g] = (q << 24) | slot;
    w.pf_prow[g] = (q << 24) | mt.y;
  }
  if (m.shared_here && m.inter_sh)
    for (int t = threadIdx.x; t < T; t += blockDim.x)
      w.pf_prow[shared_base + t] = (me << 24) | (t * (k + 1) + k);
}

// One warp per grouped row: the received bf16 rows into their grouped slots,
// then this rank's tokens (rms-normed when the layer has input_norm) as the
// shared expert's rows, zero-padded from H to k_in.
__global__ void __launch_bounds__(256) dx_copy_kernel(MoeDevice m, MoeWork w,
                                                      const float* __restrict__ x, int T,
                                                      int shared_base) {
  const int k = m.top_k, K = m.k_in, H = m.hidden;
  const uint8_t* self = static_cast<const uint8_t*>(m.dx_peers[m.dx_rank]);
  const DxLayout L = dx_layout(m.dx_world, m.dx_cap, k, K, H);
  const uint16_t* rows = reinterpret_cast<const uint16_t*>(self + L.rows);
  const long nk = (long)w.max_tokens * k;
  const int M = w.offsets[m.experts];
  const int nsh = (m.shared_here && m.inter_sh) ? T : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = blockIdx.x * 8 + warp; r < M + nsh; r += gridDim.x * 8) {
    if (r < M) {
      const int map = w.entries[nk + r];
      const size_t slot = (size_t)(map >> 24) * m.dx_cap * k + (map & 0xFFFFFF);
      const uint4* src = reinterpret_cast<const uint4*>(rows + slot * K);
      uint4* dst = reinterpret_cast<uint4*>(w.pf_xs + (long)r * K);
      for (int c = lane; c < K / 8; c += 32) dst[c] = src[c];
    } else {
      const int t = r - M;
      const float* xt = (m.input_norm ? w.xn : x) + (long)t * H;
      uint4* dst = reinterpret_cast<uint4*>(w.pf_xs + (long)(shared_base + t) * K);
      for (int c = lane; c < K / 8; c += 32) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = 8 * c + j < H ? xt[8 * c + j] : 0.f;
        dst[c] = make_uint4(bf16x2(v[0], v[1]), bf16x2(v[2], v[3]), bf16x2(v[4], v[5]),
                            bf16x2(v[6], v[7]));
      }
    }
  }
}

// After the down pass: every rank learns that this rank's rows for it landed.
__global__ void dx_done_kernel(MoeDevice m) {
  if (threadIdx.x != 0) return;
  const uint32_t epoch = static_cast<const uint32_t*>(m.dx_peers[m.dx_rank])[0];
  __threadfence_system();
  for (int q = 0; q < m.dx_world; ++q)
    st_relaxed_sys_u64(reinterpret_cast<uint64_t*>(static_cast<uint8_t*>(m.dx_peers[q]) + 128) +
                           m.dx_rank,
                       (uint64_t)epoch << 32);
}

// Before the combine: every rank's rows for this rank's tokens have landed.
__global__ void dx_wait_kernel(MoeDevice m, MoeWork w) {
  const uint8_t* self = static_cast<const uint8_t*>(m.dx_peers[m.dx_rank]);
  const uint32_t epoch = reinterpret_cast<const uint32_t*>(self)[0];
  if ((int)threadIdx.x < m.dx_world)
    dx_wait_flag(reinterpret_cast<const uint64_t*>(self + 128) + threadIdx.x, epoch, w.status);
}

cudaError_t launch_moe_dispatch(const MoeDevice& m_in, const MoeWork& w, const float* x, int T,
                                float* out, cudaStream_t s, const cudaEvent_t* marks) {
  cudaError_t e;
  auto mark = [&](int i) { return marks ? cudaEventRecord(marks[i], s) : cudaSuccess; };
  MoeDevice m = m_in;  // the decode reduction plays no part; the shared expert
  m.ep_world = 0;      // runs on all of this rank's own tokens
  m.ep_peers = nullptr;
  m.sh_parts = 0;
  if (T > m.dx_cap || T > w.max_tokens || !w.pf_xs || m.experts > 1024 ||
      m.expert_end - m.expert_begin > 1024 || (long)m.dx_world * m.dx_cap > w.max_tokens ||
      m.top_k > 32 || (m.k_in % 256) != 0)
    return cudaErrorInvalidValue;
  const int shared_base = w.max_tokens * m.top_k;
  if ((e = mark(3)) != cudaSuccess) return e;
  if ((e = launch_prefill_router(m, w, x, T, s)) != cudaSuccess) return e;
  if ((e = mark(6)) != cudaSuccess) return e;
  if ((e = launch_topk(m, w, T, -1, s)) != cudaSuccess) return e;
  dx_send_kernel<<<T, 256, 0, s>>>(m, w, x, T);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  dx_group_kernel<<<1, 1024, 0, s>>>(m, w, T, shared_base);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  dx_copy_kernel<<<4 * sm_count(), 256, 0, s>>>(m, w, x, T, shared_base);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if ((e = pf_gemm_passes(m, w, T, shared_base, m.dx_partials, s, marks)) != cudaSuccess) return e;
  dx_done_kernel<<<1, 32, 0, s>>>(m);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if ((e = mark(4)) != cudaSuccess) return e;
  dx_wait_kernel<<<1, 32, 0, s>>>(m, w);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  // every expert's row of this rank's tokens is in the local partial region
  MoeDevice mc = m;
  mc.expert_begin = 0;
  mc.expert_end = m.experts;
  MoeWork wc = w;
  wc.partial = m.dx_partial_local;
  if ((e = launch_combine(mc, wc, T, x, out, s)) != cudaSuccess) return e;
  return mark(5);
}

}  // namespace lb
