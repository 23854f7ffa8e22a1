// Tensor-core dequant-GEMV for Q4_K rows (the gate/up projections of the MoE
// experts and dense Q4_K matrices).
//
// Exactness.  A 4-bit quant q becomes the f16 subnormal q * 2^-24 (low
// nibble) or 16q * 2^-24 (high nibble) by one AND of the packed qs word, so
// the tensor core multiplies exact integers.  The activations of each
// 32-value sub-block are scaled by a power of two so that the largest lies in
// [1024, 2048) and split into an f16 high part and an f16 low part (x' = hi +
// lo to 2^-23 of the sub-block's largest value).  Both parts are columns of
// the same mma, so every product is exact and the sums are fp32 sums.  The
// K-quant arithmetic around them is the reference's: per sub-block
// (d*sc) * sum(q*x) - (dmin*m) * sum(x) (dot-product-with-q4-k-m-tensor-data,
// llambda.lisp L4338-4382).
//
// Fragment mapping ("slots").  mma.sync.m16n8k16 (A 16x16 f16 row-major, B
// 16x8 f16 column-major, D fp32) is used with thread (g, t) of each quad
// (g = lane/4, t = lane%4) holding A at k in {2t, 2t+1, 2t+8, 2t+9}; all four
// positions belong to sub-block slot t.  Output column n = 2*slot + part
// (part 0: high, 1: low), and B[k][n] is zero unless k's slot is n's slot.
// After a k-step thread (g, t) therefore holds, for rows g and g+8, the sums
// over its own sub-block in both parts (its D columns 2t, 2t+1), and applies
// that sub-block's scale and min itself: each scale is decoded once per row.
//
// A Q4_K super-block is 16 k-steps: for j = 0..7, word j of the 32 qs bytes
// of pair t (bytes 32t + 4j .. 32t + 4j + 3, values 4j..4j+3 of sub-blocks 2t
// in the low nibbles and 2t+1 in the high nibbles) gives the low-set step
// (AND 0x000F000F: values 4j, 4j+2 at k = 2t, 2t+1; the same of the word
// shifted right by 8: values 4j+1, 4j+3 at k = 2t+8, 2t+9) and the high-set
// step (AND 0x00F000F0).
//
// Pipeline.  A CTA of W warps owns a contiguous run of 16-row tiles.  Each
// tile's rows (of one or two matrices: gate and up) are copied by per-row 1-D
// bulk copies, one lane per row, into a stage whose row pitch is 16 bytes
// past a multiple of 128 (so the 8 row groups of a fragment load fall in
// different shared-memory banks); stages complete on an mbarrier and are
// waited on with a bounded spin.  The warps split the tile's (matrix,
// super-block) items, partial sums meet in shared memory, and one CTA barrier
// per token group also tells the producer that the stage may be refilled.
#pragma once

#include "engine.cuh"

namespace lb {

constexpr int kTileRows = 16;
// Dynamic shared memory of a tile kernel (stages, barriers, partial sums);
// kernel_occupancy() opts every kernel in to 200 KiB.
constexpr size_t kTileSmemBudget = 200 * 1024;

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ------------------------------------------------------------ activations
//
// Prepared activations of one token for the Q4_K mma path ("mx"),
// mx_bytes(K) bytes (16-byte aligned):
//   frag[sb][set][col][j] : uint2 (b0, b1), the B fragment of k-step j of
//       super-block sb's set (0: even sub-blocks, low nibbles; 1: odd, high
//       nibbles) for the thread of column col = 2*slot + part: halves
//       (x[4j], x[4j+2]) and (x[4j+1], x[4j+3]) of sub-block 2*slot + set,
//       scaled, part 0 = high, part 1 = low;
//   meta[sb][slot] : float4 (back_even, sum_even, back_odd, sum_odd): back
//       turns a D sum of the set back into sum(q*x) (the inverse power of two
//       times 2^24 for the low nibbles, 2^20 for the high nibbles), sum is
//       the plain fp32 sum of the sub-block's x.
__host__ __device__ __forceinline__ size_t mx_bytes(int K) { return (size_t)(K / 256) * 1088; }

__device__ __forceinline__ float pow2f(int e) {  // 2^e, e in [-126, 127]
  return __uint_as_float((uint32_t)(127 + e) << 23);
}

__device__ __forceinline__ uint32_t pack_half2(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// Stores the four values e..e+3 (e % 4 == 0) of one token into its mx
// buffer.  The 8 consecutive lanes (lane % 8 == 0 first) that hold one
// 32-value sub-block must call this together.
__device__ __forceinline__ void mx_store4(uint8_t* mx, int K, int e, float4 v) {
  float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
  float sum = (v.x + v.y) + (v.z + v.w);
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) {
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
  }
  // amax = m * 2^ex with m in [0.5, 1); ex is clamped so every scale is a
  // normal binary32 number (sub-blocks whose largest |x| lies outside
  // [2^-101, 2^100) lose precision gradually instead).
  int ex = (int)((__float_as_uint(amax) >> 23) & 0xFF) - 126;
  ex = min(max(ex, -100), 100);
  const float f = pow2f(11 - ex);
  const float xs[4] = {v.x * f, v.y * f, v.z * f, v.w * f};
  __half hi[4], lo[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    hi[q] = __float2half_rn(xs[q]);
    lo[q] = __float2half_rn(xs[q] - __half2float(hi[q]));
  }
  const int sb = e >> 8, s = (e >> 5) & 7, j = (e & 31) >> 2;
  const int set = s & 1, slot = s >> 1;
  uint2* frag = reinterpret_cast<uint2*>(mx);
  const long u = (((long)sb * 2 + set) * 8 + 2 * slot) * 8 + j;
  frag[u] = make_uint2(pack_half2(hi[0], hi[2]), pack_half2(hi[1], hi[3]));
  frag[u + 8] = make_uint2(pack_half2(lo[0], lo[2]), pack_half2(lo[1], lo[3]));
  if ((e & 31) == 0) {
    float* meta = reinterpret_cast<float*>(mx + (size_t)(K / 256) * 1024) + (sb * 4 + slot) * 4;
    meta[set * 2 + 0] = pow2f(ex + (set ? 9 : 13));  // 2^(ex-11) * 2^24 or 2^20
    meta[set * 2 + 1] = sum;
  }
}

// ------------------------------------------------------------ tile math

// d*sc and dmin*m of sub-blocks 2t and 2t+1 of the Q4_K super-block whose
// first 16 bytes are hh (get-scale-min-k4-at, llambda.lisp L4316-4336, for
// both sub-blocks at once and without branches: bytes 2t, 2t+1 of the scale
// words are one 16-bit field).  delta = d*sc, offset = dmin*m, each rounded
// once (L4363-4366).
__device__ __forceinline__ void q4k_pair_scales(const uint4& hh, int t, float2& dsc,
                                                float2& dmn) {
  const float d = half_bits_to_float(hh.x), dmin = half_bits_to_float(hh.x >> 16);
  const int sh = (t & 1) * 16;
  const uint32_t h0 = hh.y >> sh, h1 = hh.z >> sh, h2 = hh.w >> sh;
  const uint32_t sc_a = h0 & 0x3F3Fu, mn_a = h1 & 0x3F3Fu;  // sub-blocks 0..3
  const uint32_t sc_b = (h2 & 0x0F0Fu) | ((h0 >> 2) & 0x3030u);  // sub-blocks 4..7
  const uint32_t mn_b = ((h2 >> 4) & 0x0F0Fu) | ((h1 >> 2) & 0x3030u);
  const uint32_t sc = t < 2 ? sc_a : sc_b, mn = t < 2 ? mn_a : mn_b;
  // 6-bit integers to float exactly: 2^23 + v, minus 2^23
  const float2 bias = make_float2(-8388608.0f, -8388608.0f);
  const float2 scf = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(sc, 0x4B000000u, 0x7440u)),
                                            __uint_as_float(__byte_perm(sc, 0x4B000000u, 0x7441u))),
                                bias);
  const float2 mnf = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(mn, 0x4B000000u, 0x7440u)),
                                            __uint_as_float(__byte_perm(mn, 0x4B000000u, 0x7441u))),
                                bias);
  dsc = __fmul2_rn(make_float2(d, d), scf);
  dmn = __fmul2_rn(make_float2(dmin, dmin), mnf);
}

// One token's activations for one Q4_K super-block: its 1024 fragment bytes
// (frag[set][col][j]) and its 64 meta bytes (meta[slot]), in global memory or
// staged in shared memory.
struct BSlice {
  const uint8_t* frag;
  const uint8_t* meta;
};

__device__ __forceinline__ BSlice mx_slice(const uint8_t* mx, int sb, int nsb) {
  return BSlice{mx + (size_t)sb * 1024, mx + (size_t)nsb * 1024 + (size_t)sb * 64};
}

template <bool SMEM>
__device__ __forceinline__ uint4 ld_b16(const void* p) {
  if (SMEM) return *reinterpret_cast<const uint4*>(p);
  return __ldg(reinterpret_cast<const uint4*>(p));
}
template <bool SMEM>
__device__ __forceinline__ uint2 ld_b8(const void* p) {
  if (SMEM) return *reinterpret_cast<const uint2*>(p);
  return __ldg(reinterpret_cast<const uint2*>(p));
}

// 32 zero bytes in global memory (the B source of the threads without a
// column of their own when the inputs are read through L1).
static __device__ __align__(16) const uint8_t kZero32[32] = {};


// Adds to y[n][r] (r = 0: row g, r = 1: row g + 8 of a 16-row block; .x the
// even sub-block of the lane's slot, .y the odd one) this lane's share of the
// dot products of one super-block of the block's rows with the NT tokens of
// bs (SMEM: the slices are in shared memory).  rg / rg8: the super-block of
// rows g and g+8 in shared memory (16-byte aligned; the 8 row groups must
// fall in different bank groups, e.g. rows 144 bytes apart or a pitch of 16
// mod 128).  bz: 32 zero bytes in the slices' memory, the B source of the
// threads whose column cannot be non-zero.
template <int NT, bool SMEM>
__device__ __forceinline__ void q4k_sb_mma(const uint8_t* rg, const uint8_t* rg8,
                                           const BSlice (&bs)[NT], const uint8_t* bz, int lane,
                                           float2 (&y)[NT][2]) {
  const int g = lane >> 2, t = lane & 3;
  const bool bthread = t == (g >> 1);  // the lane whose B column g can be non-zero
  {
    const uint4 wg0 = *reinterpret_cast<const uint4*>(rg + 16 + 32 * t);
    const uint4 w80 = *reinterpret_cast<const uint4*>(rg8 + 16 + 32 * t);
    const uint4 wg1 = *reinterpret_cast<const uint4*>(rg + 32 + 32 * t);
    const uint4 w81 = *reinterpret_cast<const uint4*>(rg8 + 32 + 32 * t);
    const uint32_t Wg[8] = {wg0.x, wg0.y, wg0.z, wg0.w, wg1.x, wg1.y, wg1.z, wg1.w};
    const uint32_t W8[8] = {w80.x, w80.y, w80.z, w80.w, w81.x, w81.y, w81.z, w81.w};
    float de[NT][4], dodd[NT][4];  // D of the even and odd set
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int q = 0; q < 4; ++q) de[n][q] = dodd[n][q] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      uint4 be[NT], bo[NT];  // B of k-steps j, j+1 (even set, odd set)
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const uint4* fr = reinterpret_cast<const uint4*>(bs[n].frag) + g * 4;
        be[n] = ld_b16<SMEM>(bthread ? reinterpret_cast<const uint8_t*>(fr + j / 2) : bz);
        bo[n] = ld_b16<SMEM>(bthread ? reinterpret_cast<const uint8_t*>(fr + 32 + j / 2) : bz);
      }
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const uint32_t wg = Wg[j + jj], w8 = W8[j + jj];
        const uint32_t gs = wg >> 8, g8s = w8 >> 8;
        const uint32_t al0 = wg & 0x000F000Fu, al1 = w8 & 0x000F000Fu;
        const uint32_t al2 = gs & 0x000F000Fu, al3 = g8s & 0x000F000Fu;
        const uint32_t ah0 = wg & 0x00F000F0u, ah1 = w8 & 0x00F000F0u;
        const uint32_t ah2 = gs & 0x00F000F0u, ah3 = g8s & 0x00F000F0u;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          const uint32_t e0 = jj ? be[n].z : be[n].x, e1 = jj ? be[n].w : be[n].y;
          const uint32_t o0 = jj ? bo[n].z : bo[n].x, o1 = jj ? bo[n].w : bo[n].y;
          mma_f16(de[n], al0, al1, al2, al3, e0, e1);
          mma_f16(dodd[n], ah0, ah1, ah2, ah3, o0, o1);
        }
      }
    }
    float2 dsc[2], dmn[2];
    q4k_pair_scales(*reinterpret_cast<const uint4*>(rg), t, dsc[0], dmn[0]);
    q4k_pair_scales(*reinterpret_cast<const uint4*>(rg8), t, dsc[1], dmn[1]);
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const uint4 mw = ld_b16<SMEM>(bs[n].meta + 16 * t);
      const float4 mt = make_float4(__uint_as_float(mw.x), __uint_as_float(mw.y),
                                    __uint_as_float(mw.z), __uint_as_float(mw.w));
      const float2 back = make_float2(mt.x, mt.z), sums = make_float2(-mt.y, -mt.w);
      // D: [0] row g high, [1] row g low, [2] row g+8 high, [3] row g+8 low
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float2 s = __fadd2_rn(make_float2(de[n][2 * r], dodd[n][2 * r]),
                              make_float2(de[n][2 * r + 1], dodd[n][2 * r + 1]));
        s = __fmul2_rn(s, back);  // sum(q*x) of the even and odd sub-block
        float2 a = __ffma2_rn(dsc[r], s, y[n][r]);
        y[n][r] = __ffma2_rn(dmn[r], sums, a);
      }
    }
  }
}

// q4k_sb_mma for nt (1..NT) tokens: the first nt entries of bs and y.
template <int NT, bool SMEM>
__device__ __forceinline__ void q4k_sb_mma_n(int nt, const uint8_t* rg, const uint8_t* rg8,
                                             const BSlice (&bs)[NT], const uint8_t* bz,
                                             int lane, float2 (&y)[NT][2]) {
  if constexpr (NT == 1) {
    q4k_sb_mma<1, SMEM>(rg, rg8, bs, bz, lane, y);
  } else {
    if (nt >= NT)
      q4k_sb_mma<NT, SMEM>(rg, rg8, bs, bz, lane, y);
    else
      q4k_sb_mma_n<NT - 1, SMEM>(nt, rg, rg8, reinterpret_cast<const BSlice(&)[NT - 1]>(bs), bz,
                                 lane, reinterpret_cast<float2(&)[NT - 1][2]>(y));
  }
}

// q4k_sb_mma over super-blocks [sb0, sb1) of a 16-row tile whose row 0 is
// `tile`, rows `pitch` bytes apart (pitch % 128 == 16), with nt tokens whose
// prepared activations start at mx[n] (SMEM: in shared memory, with the
// 32 zero bytes bz there too; else global memory).
template <int NT, bool SMEM = false>
__device__ __forceinline__ void q4k_tile_mma(const uint8_t* tile, int pitch, int sb0, int sb1,
                                             const uint8_t* const (&mx)[NT], int nt, int nsb,
                                             int lane, float2 (&y)[NT][2],
                                             const uint8_t* bz = kZero32) {
  const int g = lane >> 2;
  for (int sb = sb0; sb < sb1; ++sb) {
    const uint8_t* rg = tile + g * pitch + sb * LB_Q4K;
    BSlice bs[NT];
#pragma unroll
    for (int n = 0; n < NT; ++n) bs[n] = mx_slice(mx[n], sb, nsb);
    q4k_sb_mma_n<NT, SMEM>(nt, rg, rg + 8 * pitch, bs, bz, lane, y);
  }
}

// This warp's share of a staged tile: the (matrix, super-block) items
// [warp*I/W, (warp+1)*I/W) of I = MATS * nsb.
template <int NT, int MATS, int W, bool SMEM = false>
__device__ __forceinline__ void tile_items(const uint8_t* stage, int pitch, int nsb, int warp,
                                           int lane, const uint8_t* const (&mx)[NT], int nt,
                                           float2 (&y)[MATS][NT][2],
                                           const uint8_t* bz = kZero32) {
  const int items = MATS * nsb;
  const int i0 = warp * items / W, i1 = (warp + 1) * items / W;
#pragma unroll
  for (int mat = 0; mat < MATS; ++mat) {
    const int sb0 = max(i0 - mat * nsb, 0), sb1 = min(i1 - mat * nsb, nsb);
    if (sb0 < sb1)
      q4k_tile_mma<NT, SMEM>(stage + (size_t)mat * kTileRows * pitch, pitch, sb0, sb1, mx, nt,
                             nsb, lane, y[mat], bz);
  }
}

// Sums y over each quad and stores the row sums into red[warp][mat][row][n].
template <int NT, int MATS>
__device__ __forceinline__ void tile_partials_store(float* red, int warp, int lane,
                                                    const float2 (&y)[MATS][NT][2]) {
  float v[MATS][2][NT];
#pragma unroll
  for (int mat = 0; mat < MATS; ++mat)
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        float s = y[mat][n][r].x + y[mat][n][r].y;
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        v[mat][r][n] = s;
      }
  if ((lane & 3) == 0) {
    const int g = lane >> 2;
#pragma unroll
    for (int mat = 0; mat < MATS; ++mat)
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int n = 0; n < NT; ++n)
          red[((warp * MATS + mat) * kTileRows + g + 8 * r) * NT + n] = v[mat][r][n];
  }
}

// Row sum (row r, token n, matrix mat) of a tile from the warps' partials.
template <int NT, int MATS, int W>
__device__ __forceinline__ float tile_row_sum(const float* red, int mat, int r, int n) {
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < W; ++w) s += red[((w * MATS + mat) * kTileRows + r) * NT + n];
  return s;
}

template <int NT, int MATS, int W>
__host__ __device__ __forceinline__ int tile_red_floats() {
  return 2 * W * MATS * kTileRows * NT;  // double-buffered
}

// ------------------------------------------------------------ Q6_K rows
//
// A Q6_K sub-block is 16 values, so one m16n8k16 k-step is one sub-block of
// all 16 rows of a block, and no slot mapping is needed: the B columns are
// 4 tokens x (high, low) parts (column n = 2*token + part), and lane (g, t)
// ends the k-step holding the whole sub-block's sums of token t for rows g
// and g+8 (D columns 2t, 2t+1).  The quant q (0..63) enters as the exact f16
// subnormal q * 2^-24; the reference's -32 offset is applied with the
// sub-block sum of x: sum((q-32)*x) = sum(q*x) - 32*sum(x), scaled by
// delta = d*sc (dot-product-with-q6-k-tensor-data, llambda.lisp L4458-4506).
//
// Lane t supplies k = 2t, 2t+1, 2t+8, 2t+9 = values 4t, 4t+2, 4t+1, 4t+3 of
// the sub-block, i.e. bytes 0, 2, 1, 3 of word t of its 16-byte runs.  The 16
// k-steps of a super-block run in the order q = (2c + h) * 4 + gg over chunk
// c, half h and group gg, sub-block s = 8c + 2gg + h (expand-q6-k-group,
// L4203-4310): value i of sub-block s has its low 4 bits in ql byte
// 64c + 32(gg%2) + 16h + i (low nibble for gg < 2, high nibble otherwise)
// and its high 2 bits in qh byte 128 + 32c + 16h + i, bits 2gg and 2gg+1.

// Prepared input of one token for Q6_K rows ("m6"), m6_bytes(K) bytes
// (16-byte aligned), per super-block (1152 bytes):
//   frag[q / 2][part][t][q % 2] : uint2, halves (x[4t], x[4t+2]) and
//       (x[4t+1], x[4t+3]) of k-step q's sub-block, scaled, part 0 = high,
//       1 = low (1024 bytes): the eight threads that load one k-step pair
//       of a token read 128 consecutive bytes (no bank conflicts);
//   meta[q] : float2 (back, -32 * sum(x)) of k-step q's sub-block (128 bytes).
__host__ __device__ __forceinline__ size_t m6_bytes(int K) { return (size_t)(K / 256) * 1152; }

__host__ __device__ __forceinline__ int q6_step_of(int s) {
  return ((s >> 3) * 2 + (s & 1)) * 4 + ((s & 7) >> 1);
}

// Stores sub-block s_glob of one entry into its m6 buffer: lane (g, 0) holds
// value g in va and value g + 8 in vb; the other lanes pass zeros.  Whole
// warp.
__device__ __forceinline__ void m6_store_subblock(uint8_t* m6, int s_glob, float va, float vb,
                                                  int lane) {
  float amax = fmaxf(fabsf(va), fabsf(vb)), sum = va + vb;
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
  }
  int ex = (int)((__float_as_uint(amax) >> 23) & 0xFF) - 126;  // as in mx_store4
  ex = min(max(ex, -100), 100);
  const float f = pow2f(11 - ex);
  uint8_t* base = m6 + (size_t)(s_glob >> 4) * 1152;
  const int q = q6_step_of(s_glob & 15);
  if ((lane & 3) == 0) {
    const int g = lane >> 2;
    __half* h = reinterpret_cast<__half*>(base);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int i = g + 8 * r;
      const float xs = (r ? vb : va) * f;
      const __half hi = __float2half_rn(xs);
      const __half lo = __float2half_rn(xs - __half2float(hi));
      const int t4 = i >> 2, pos = i & 3, hp = (pos & 1) * 2 + (pos >> 1);
      h[((((q >> 1) * 2 + 0) * 4 + t4) * 2 + (q & 1)) * 4 + hp] = hi;
      h[((((q >> 1) * 2 + 1) * 4 + t4) * 2 + (q & 1)) * 4 + hp] = lo;
    }
    if (g == 0)
      reinterpret_cast<float2*>(base + 1024)[q] = make_float2(pow2f(ex + 13), -32.0f * sum);
  }
}

// Zeroes sub-block s_glob of an m6 buffer (padding past the matrix's rows).
// 16 lanes; lane l < 8 writes the 8 bytes of (part l / 4, t l % 4), lane 0
// the meta.
__device__ __forceinline__ void m6_zero_subblock(uint8_t* m6, int s_glob, int l) {
  uint8_t* base = m6 + (size_t)(s_glob >> 4) * 1152;
  const int q = q6_step_of(s_glob & 15);
  if (l < 8)
    reinterpret_cast<uint2*>(base)[(((q >> 1) * 2 + (l >> 2)) * 4 + (l & 3)) * 2 + (q & 1)] =
        make_uint2(0, 0);
  if (l == 0) reinterpret_cast<float2*>(base + 1024)[q] = make_float2(0.f, 0.f);
}

// int8 byte b of w as a float, exactly (2^23 + 128 + v, minus 2^23 + 128).
__device__ __forceinline__ float s8_to_float(uint32_t w_xor80, int b) {
  return __uint_as_float(__byte_perm(w_xor80, 0x4B000000u, 0x7440u | b)) - 8388736.0f;
}

// Adds token t's (this lane's) dot products over super-block sb of a 16-row
// Q6_K block to y[grp] (.x row g, .y row g+8) for NG groups of 4 tokens: token
// 4*grp + t, if below nt.  rg / rg8: the super-block of rows g and g+8 in
// shared memory (2-byte aligned); m6[n]: the m6 buffers of the tokens (n < nt
// valid; SMEM: staged in shared memory).  The A fragments are decoded once
// per k-step and serve every group.
template <bool SMEM, int NG>
__device__ __forceinline__ void q6k_sb_mma(const uint8_t* rg, const uint8_t* rg8, int sb,
                                           const uint8_t* const (&m6)[4 * NG], int nt, int lane,
                                           float2 (&y)[NG]) {
  const int g = lane >> 2, t = lane & 3;
  const int bn = g >> 1, part = g & 1;
  const uint4* bsrc[NG];
  const float4* msrc[NG];
  bool bval[NG], mval[NG];
#pragma unroll
  for (int grp = 0; grp < NG; ++grp) {
    bval[grp] = 4 * grp + bn < nt;
    mval[grp] = 4 * grp + t < nt;
    const uint8_t* pb = m6[4 * grp];  // m6[4 grp + bn], m6[4 grp + t] without indexing
    const uint8_t* pm = m6[4 * grp];  // the pointer array by a register (local memory)
#pragma unroll
    for (int i = 1; i < 4; ++i) {
      if (bn == i) pb = m6[4 * grp + i];
      if (t == i) pm = m6[4 * grp + i];
    }
    bsrc[grp] = reinterpret_cast<const uint4*>(pb + (size_t)sb * 1152) + part * 4 + t;
    msrc[grp] = reinterpret_cast<const float4*>(pm + (size_t)sb * 1152 + 1024);
  }
  const float d = half_bits_to_float(lds_u16(rg + 208));
  const float d8 = half_bits_to_float(lds_u16(rg8 + 208));
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    // 8 scale bytes of chunk c (sub-blocks 8c..8c+7), sign bit flipped
    const uint32_t sg0 = lds_w32_align2(rg + 192 + 8 * c) ^ 0x80808080u;
    const uint32_t sg1 = lds_w32_align2(rg + 196 + 8 * c) ^ 0x80808080u;
    const uint32_t s80 = lds_w32_align2(rg8 + 192 + 8 * c) ^ 0x80808080u;
    const uint32_t s81 = lds_w32_align2(rg8 + 196 + 8 * c) ^ 0x80808080u;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int o = 64 * c + 16 * h + 4 * t;
      uint32_t qg[4], q8[4];
      {
        const uint32_t A = lds_w32_align2(rg + o), B = lds_w32_align2(rg + o + 32);
        const uint32_t H = lds_w32_align2(rg + 128 + 32 * c + 16 * h + 4 * t);
        qg[0] = (A & 0x0F0F0F0Fu) | ((H << 4) & 0x30303030u);
        qg[1] = (B & 0x0F0F0F0Fu) | ((H << 2) & 0x30303030u);
        qg[2] = ((A >> 4) & 0x0F0F0F0Fu) | (H & 0x30303030u);
        qg[3] = ((B >> 4) & 0x0F0F0F0Fu) | ((H >> 2) & 0x30303030u);
      }
      {
        const uint32_t A = lds_w32_align2(rg8 + o), B = lds_w32_align2(rg8 + o + 32);
        const uint32_t H = lds_w32_align2(rg8 + 128 + 32 * c + 16 * h + 4 * t);
        q8[0] = (A & 0x0F0F0F0Fu) | ((H << 4) & 0x30303030u);
        q8[1] = (B & 0x0F0F0F0Fu) | ((H << 2) & 0x30303030u);
        q8[2] = ((A >> 4) & 0x0F0F0F0Fu) | (H & 0x30303030u);
        q8[3] = ((B >> 4) & 0x0F0F0F0Fu) | ((H >> 2) & 0x30303030u);
      }
      const int q0 = (2 * c + h) * 4;  // first k-step of this (c, h)
      uint4 b01[NG], b23[NG];
      float4 m01[NG], m23[NG];
#pragma unroll
      for (int grp = 0; grp < NG; ++grp) {
        b01[grp] = b23[grp] = make_uint4(0, 0, 0, 0);
        if (bval[grp]) {
          b01[grp] = ld_b16<SMEM>(bsrc[grp] + (q0 / 2) * 8);
          b23[grp] = ld_b16<SMEM>(bsrc[grp] + (q0 / 2 + 1) * 8);
        }
        m01[grp] = m23[grp] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (mval[grp]) {
          const uint4 u01 = ld_b16<SMEM>(msrc[grp] + q0 / 2);
          const uint4 u23 = ld_b16<SMEM>(msrc[grp] + q0 / 2 + 1);
          m01[grp] = make_float4(__uint_as_float(u01.x), __uint_as_float(u01.y),
                                 __uint_as_float(u01.z), __uint_as_float(u01.w));
          m23[grp] = make_float4(__uint_as_float(u23.x), __uint_as_float(u23.y),
                                 __uint_as_float(u23.z), __uint_as_float(u23.w));
        }
      }
#pragma unroll
      for (int gg = 0; gg < 4; ++gg) {
        const uint32_t a0 = __byte_perm(qg[gg], 0, 0x4240), a1 = __byte_perm(q8[gg], 0, 0x4240);
        const uint32_t a2 = __byte_perm(qg[gg], 0, 0x4341), a3 = __byte_perm(q8[gg], 0, 0x4341);
        // sub-block s = 8c + 2gg + h: scale byte 2gg + h of the chunk's 8
        const int sbyte = 2 * gg + h;
        const uint32_t wg = sbyte < 4 ? sg0 : sg1, w8 = sbyte < 4 ? s80 : s81;
        const float2 dsc = __fmul2_rn(make_float2(d, d8),
                                      make_float2(s8_to_float(wg, sbyte & 3),
                                                  s8_to_float(w8, sbyte & 3)));
#pragma unroll
        for (int grp = 0; grp < NG; ++grp) {
          float dv[4] = {0.f, 0.f, 0.f, 0.f};
          const uint4& bl = gg < 2 ? b01[grp] : b23[grp];
          const uint32_t b0 = (gg & 1) ? bl.z : bl.x, b1 = (gg & 1) ? bl.w : bl.y;
          mma_f16(dv, a0, a1, a2, a3, b0, b1);
          const float4& ml = gg < 2 ? m01[grp] : m23[grp];
          const float back = (gg & 1) ? ml.z : ml.x, off = (gg & 1) ? ml.w : ml.y;
          float2 s2 = __fadd2_rn(make_float2(dv[0], dv[2]), make_float2(dv[1], dv[3]));
          s2 = __ffma2_rn(s2, make_float2(back, back), make_float2(off, off));
          y[grp] = __ffma2_rn(dsc, s2, y[grp]);
        }
      }
    }
  }
}

// ----------------------------------------------- Q6_K rows, sub-block slots
//
// With one or two tokens most of the eight B columns of the form above are
// empty while every k-step still pays for a scale and three fp32 updates per
// thread.  This form gives the four threads of a quad four different
// sub-blocks instead (the Q4_K slot mapping): in k-step j of a group of four,
// thread t supplies values 4j..4j+3 of its own sub-block at k = 2t, 2t+1,
// 2t+8, 2t+9, and B column 2u + part carries slot u's activations at thread
// u's positions and zeros elsewhere, so after four k-steps D columns 2t, 2t+1
// hold thread t's whole sub-block sums (high and low part) for rows g and
// g+8, and the scale work falls to once per sub-block.  One mma per token and
// k-step; the decoded A serves every token.
//
// Thread t owns sub-blocks 4i + t of each super-block: in 64-byte chunk c it
// reads ql run t (bytes 64c + 16t.., low nibbles: sub-block 8c + t, high
// nibbles: 8c + 4 + t) and qh run t & 1 (bytes 128 + 32c + 16(t & 1).., bits
// 2(t >> 1) and 4 + 2(t >> 1)), with the chunk's scale bytes 8c + t and
// 8c + 4 + t.  The quad's four partial sums are added once per row block.
//
// Prepared input of one entry ("i6", i6_bytes(K), 1152 bytes per 256 values):
//   frag[s][part][j] : uint2, halves (x[4j], x[4j+2]) and (x[4j+1], x[4j+3])
//       of sub-block s, scaled, part 0 = high, 1 = low (1024 bytes);
//   meta[s] : float2 (back, -32 * sum(x)) of sub-block s (128 bytes).
__host__ __device__ __forceinline__ size_t i6_bytes(int K) { return (size_t)(K / 256) * 1152; }

// Stores sub-block s_glob of one entry: lane (g, 0) holds value g in va and
// value g + 8 in vb; the other lanes pass zeros.  Whole warp.
__device__ __forceinline__ void i6_store_subblock(uint8_t* xi, int s_glob, float va, float vb,
                                                  int lane) {
  float amax = fmaxf(fabsf(va), fabsf(vb)), sum = va + vb;
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
  }
  int ex = (int)((__float_as_uint(amax) >> 23) & 0xFF) - 126;  // as in mx_store4
  ex = min(max(ex, -100), 100);
  const float f = pow2f(11 - ex);
  uint8_t* base = xi + (size_t)(s_glob >> 4) * 1152;
  const int sl = s_glob & 15;
  if ((lane & 3) == 0) {
    const int g = lane >> 2;
    __half* h = reinterpret_cast<__half*>(base);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int i = g + 8 * r;
      const float xs = (r ? vb : va) * f;
      const __half hi = __float2half_rn(xs);
      const __half lo = __float2half_rn(xs - __half2float(hi));
      const int j = i >> 2, pos = i & 3, hp = (pos & 1) * 2 + (pos >> 1);
      h[(sl * 2 + 0) * 16 + j * 4 + hp] = hi;
      h[(sl * 2 + 1) * 16 + j * 4 + hp] = lo;
    }
    if (g == 0)
      reinterpret_cast<float2*>(base + 1024)[sl] = make_float2(pow2f(ex + 13), -32.0f * sum);
  }
}

// Zeroes sub-block s_glob of an i6 buffer (padding past the matrix's rows).
// 16 lanes; lane l < 8 writes 8 bytes of the fragments, lane 0 the meta.
__device__ __forceinline__ void i6_zero_subblock(uint8_t* xi, int s_glob, int l) {
  uint8_t* base = xi + (size_t)(s_glob >> 4) * 1152;
  const int sl = s_glob & 15;
  if (l < 8) reinterpret_cast<uint2*>(base)[sl * 8 + l] = make_uint2(0, 0);  // (part, j) = l
  if (l == 0) reinterpret_cast<float2*>(base + 1024)[sl] = make_float2(0.f, 0.f);
}

// N little-endian words from a shared-memory address p that is 4-byte
// aligned (MIS = 0), 2 past a multiple of 4 (MIS = 1: N + 1 aligned loads and
// one byte permute per word) or either (MIS = 2: decided per thread).
template <int MIS, int N>
__device__ __forceinline__ void lds_words(const uint8_t* p, uint32_t (&w)[N]) {
  if (MIS == 0) {
#pragma unroll
    for (int i = 0; i < N; ++i) w[i] = reinterpret_cast<const uint32_t*>(p)[i];
  } else {
    const int mis = MIS == 1 ? 2 : (int)(reinterpret_cast<uintptr_t>(p) & 2);
    const uint32_t* a = reinterpret_cast<const uint32_t*>(p - mis);  // keeps the address space
    const uint32_t sel = mis ? 0x5432u : 0x3210u;
    uint32_t v[N + 1];
#pragma unroll
    for (int i = 0; i <= N; ++i) v[i] = a[i];  // within the super-block: runs end by byte 208
#pragma unroll
    for (int i = 0; i < N; ++i) w[i] = __byte_perm(v[i], v[i + 1], sel);
  }
}

// Adds this thread's share of the dot products of super-block sb of a 16-row
// Q6_K block with NTOK tokens to y[n] (.x row g, .y row g+8): only sub-blocks
// 4i + t enter, the caller adds the quad.  rg / rg8: the super-block of rows
// g and g+8 in shared memory (alignment as MIS of lds_words); xi[n]: token
// n's i6 buffer (SMEM: in shared memory); bz: 32 zero bytes in the same
// memory, the B source of the threads that carry no column of theirs.
template <bool SMEM, int NTOK, int MIS>
__device__ __forceinline__ void q6i_sb_mma(const uint8_t* rg, const uint8_t* rg8, int sb,
                                           const uint8_t* const (&xi)[NTOK], const uint8_t* bz,
                                           int lane, float2 (&y)[NTOK]) {
  const int g = lane >> 2, t = lane & 3;
  const bool bcol = (g >> 1) == t;  // this thread carries B column g (slot t, part g & 1)
  const uint32_t ssel = 0x7440u | (uint32_t)t;
  const int hsh = 2 * (t >> 1);
  const float d = half_bits_to_float(lds_u16(rg + 208));
  const float d8 = half_bits_to_float(lds_u16(rg8 + 208));
  const size_t sbo = (size_t)sb * 1152;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint32_t lg[4], l8[4], hg[4], h8[4], sw[2], s8w[2];
    lds_words<MIS>(rg + 64 * c + 16 * t, lg);
    lds_words<MIS>(rg8 + 64 * c + 16 * t, l8);
    lds_words<MIS>(rg + 128 + 32 * c + 16 * (t & 1), hg);
    lds_words<MIS>(rg8 + 128 + 32 * c + 16 * (t & 1), h8);
    lds_words<MIS>(rg + 192 + 8 * c, sw);
    lds_words<MIS>(rg8 + 192 + 8 * c, s8w);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      hg[j] >>= hsh;
      h8[j] >>= hsh;
    }
#pragma unroll
    for (int n = 0; n < 2; ++n) {  // n = 0: low nibbles, sub-block 8c + t; 1: high, 8c + 4 + t
      // scale byte 8c + 4n + t of rows g and g+8 (int8, exactly)
      const float2 dsc = __fmul2_rn(
          make_float2(d, d8),
          __fadd2_rn(
              make_float2(__uint_as_float(__byte_perm(sw[n] ^ 0x80808080u, 0x4B000000u, ssel)),
                          __uint_as_float(__byte_perm(s8w[n] ^ 0x80808080u, 0x4B000000u, ssel))),
              make_float2(-8388736.0f, -8388736.0f)));
      const int so = (8 * c + 4 * n) * 64;  // first fragment byte of the four sub-blocks
      uint4 b01[NTOK], b23[NTOK];
      float2 mt[NTOK];
#pragma unroll
      for (int k = 0; k < NTOK; ++k) {
        const uint8_t* pb = bcol ? xi[k] + sbo + so + g * 32 : bz;
        b01[k] = ld_b16<SMEM>(pb);
        b23[k] = ld_b16<SMEM>(pb + 16);
        const uint2 mu = ld_b8<SMEM>(xi[k] + sbo + 1024 + (8 * c + 4 * n + t) * 8);
        mt[k] = make_float2(__uint_as_float(mu.x), __uint_as_float(mu.y));
      }
      float acc[NTOK][4];
#pragma unroll
      for (int k = 0; k < NTOK; ++k) acc[k][0] = acc[k][1] = acc[k][2] = acc[k][3] = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t qg, q8;
        if (n == 0) {
          qg = (lg[j] & 0x0F0F0F0Fu) | ((hg[j] << 4) & 0x30303030u);
          q8 = (l8[j] & 0x0F0F0F0Fu) | ((h8[j] << 4) & 0x30303030u);
        } else {
          qg = ((lg[j] >> 4) & 0x0F0F0F0Fu) | (hg[j] & 0x30303030u);
          q8 = ((l8[j] >> 4) & 0x0F0F0F0Fu) | (h8[j] & 0x30303030u);
        }
        const uint32_t a0 = __byte_perm(qg, 0, 0x4240), a1 = __byte_perm(q8, 0, 0x4240);
        const uint32_t a2 = __byte_perm(qg, 0, 0x4341), a3 = __byte_perm(q8, 0, 0x4341);
#pragma unroll
        for (int k = 0; k < NTOK; ++k) {
          const uint4& bl = j < 2 ? b01[k] : b23[k];
          mma_f16(acc[k], a0, a1, a2, a3, (j & 1) ? bl.z : bl.x, (j & 1) ? bl.w : bl.y);
        }
      }
#pragma unroll
      for (int k = 0; k < NTOK; ++k) {
        float2 s2 = __fadd2_rn(make_float2(acc[k][0], acc[k][2]), make_float2(acc[k][1], acc[k][3]));
        s2 = __ffma2_rn(s2, make_float2(mt[k].x, mt[k].x), make_float2(mt[k].y, mt[k].y));
        y[k] = __ffma2_rn(dsc, s2, y[k]);
      }
    }
  }
}

// One 16-row Q6_K block (rows of rb bytes from blk, 16-byte aligned in shared
// memory) times NTOK tokens xin[0..NTOK) over super-blocks [sb0, sb1):
// returns, in thread t of quad g, rows g and g+8 for token t - tok0 (the
// quad's threads summed), r unchanged where that is not one of the NTOK.
template <bool SMEM, int NTOK>
__device__ __forceinline__ void q6i_block(const uint8_t* blk, size_t rb, int sb0, int sb1,
                                          const uint8_t* const* xin, const uint8_t* bz, int lane,
                                          int tok0, float2& r) {
  const uint8_t* xi[NTOK];
#pragma unroll
  for (int n = 0; n < NTOK; ++n) xi[n] = xin[n];
  float2 y[NTOK];
#pragma unroll
  for (int n = 0; n < NTOK; ++n) y[n] = make_float2(0.f, 0.f);
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* rg = blk + g * rb;
  const uint8_t* rg8 = blk + (g + 8) * rb;
  if ((rb & 3) == 0) {  // rows 4-byte aligned: super-blocks at 0 and 2 mod 4 in turn
    for (int sb = sb0; sb < sb1; ++sb) {
      if (sb & 1)
        q6i_sb_mma<SMEM, NTOK, 1>(rg + sb * LB_Q6K, rg8 + sb * LB_Q6K, sb, xi, bz, lane, y);
      else
        q6i_sb_mma<SMEM, NTOK, 0>(rg + sb * LB_Q6K, rg8 + sb * LB_Q6K, sb, xi, bz, lane, y);
    }
  } else {
    for (int sb = sb0; sb < sb1; ++sb)
      q6i_sb_mma<SMEM, NTOK, 2>(rg + sb * LB_Q6K, rg8 + sb * LB_Q6K, sb, xi, bz, lane, y);
  }
#pragma unroll
  for (int n = 0; n < NTOK; ++n)
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
      y[n].x += __shfl_xor_sync(0xffffffffu, y[n].x, o);
      y[n].y += __shfl_xor_sync(0xffffffffu, y[n].y, o);
    }
#pragma unroll
  for (int n = 0; n < NTOK; ++n)
    if (t == tok0 + n) r = y[n];
}

// ------------------------------------------------------------ tile staging

// Shared-memory plan of a tile pipeline.
struct TilePlan {
  int pitch;        // padded row pitch in shared memory
  int stage_bytes;  // MATS * 16 * pitch, rounded to 128
  int stages;
};

__host__ __device__ __forceinline__ TilePlan tile_plan(size_t row_bytes, int mats, size_t budget) {
  TilePlan p;
  p.pitch = (int)(((row_bytes + 127) & ~size_t(127)) + 16);  // pitch % 128 == 16
  p.stage_bytes = (int)(((size_t)mats * kTileRows * p.pitch + 127) & ~size_t(127));
  p.stages = (int)(budget / p.stage_bytes);
  if (p.stages > 5) p.stages = 5;
  return p;
}

// Issues the copies of one tile into stage `st` (all lanes of one warp):
// rows [0, nr) of matrix 0 from src0 and, when src1 is set, of matrix 1 from
// src1, each row `rb` bytes (rb % 16 == 0, sources 16-byte aligned).
__device__ __forceinline__ void tile_issue(uint8_t* st, uint64_t* bar, int pitch, int nr,
                                           size_t rb, const uint8_t* src0, const uint8_t* src1,
                                           int lane) {
  const int mats = src1 ? 2 : 1;
  if (lane == 0) mbar_expect_tx(bar, (uint32_t)(mats * nr * rb));
  __syncwarp();
  const int mat = lane >> 4, r = lane & 15;
  if (mat < mats && r < nr)
    tma_load_1d(st + (size_t)(mat * kTileRows + r) * pitch, (mat ? src1 : src0) + (size_t)r * rb,
                (uint32_t)rb, bar);
}

}  // namespace lb
