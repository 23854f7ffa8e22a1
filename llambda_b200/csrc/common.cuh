// Shared device helpers for the llambda B200 quantized-FFN kernels.
//
// GGUF super-block layouts (256 values each), as read by llambda
// (llambda.lisp L2142-2144, L4338-4506):
//   Q4_K (144 B): d:f16 @0, dmin:f16 @2, scales[12] @4, qs[128] @16
//   Q6_K (210 B): ql[128] @0, qh[64] @128, scales:int8[16] @192, d:f16 @208
//   Q5_K (176 B): d:f16 @0, dmin:f16 @2, scales[12] @4, qh[32] @16, qs[128] @48
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define LB_QK 256
#define LB_Q4K 144
#define LB_Q6K 210
#define LB_Q5K 176

// GGML type tags (llambda.lisp L24-31).
#define LB_TYPE_F32 0
#define LB_TYPE_Q5_0 6
#define LB_TYPE_Q8_0 8
#define LB_TYPE_Q4_K 12
#define LB_TYPE_Q5_K 13
#define LB_TYPE_Q6_K 14

// 32-value block formats (llambda.lisp L2139-2140):
//   Q5_0 (22 B): d:f16 @0, qh:u32 @2, qs[16] @6
//   Q8_0 (34 B): d:f16 @0, qs:int8[32] @2
#define LB_Q5_0 22
#define LB_Q8_0 34

namespace lb {

constexpr int kWarp = 32;

__device__ __forceinline__ float warp_sum(float v, int width = 32) {
#pragma unroll
  for (int o = width >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Byte i (0..3) of w, whose bytes hold unsigned values below 128, becomes the
// binary32 number 2^23 + 2^16 * q: the byte is placed in bits 16..23 under the
// exponent byte 0x4B.  One PRMT per weight instead of an integer-to-float
// conversion; the 2^23 bias is removed per sub-block with the sum of x.
template <int I>
__device__ __forceinline__ float magic_q(uint32_t w) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7044u | (I << 8)));
}
constexpr float kMagicUnscale = 1.0f / 65536.0f;  // 2^-16
constexpr float kMagicBias = 128.0f;              // 2^23 * 2^-16

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
  return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFFu)));
}

// get-scale-min-k4-at (llambda.lisp L4316-4336) for sub-block j of a Q4_K
// block whose 12 scale bytes are in words s0 (bytes 0-3), s1 (4-7), s2 (8-11).
__device__ __forceinline__ void q4k_scale_min(uint32_t s0, uint32_t s1, uint32_t s2, int j,
                                              int& sc, int& m) {
  const int jj = j & 3;
  const int b0 = (s0 >> (8 * jj)) & 0xFF;  // byte j (j<4) or j-4 (j>=4)
  const int b1 = (s1 >> (8 * jj)) & 0xFF;  // byte j+4 (j<4) or j (j>=4)
  const int b2 = (s2 >> (8 * jj)) & 0xFF;  // byte j+4 (j>=4)
  if (j < 4) {
    sc = b0 & 63;
    m = b1 & 63;
  } else {
    sc = (b2 & 15) | ((b0 >> 6) << 4);
    m = (b2 >> 4) | ((b1 >> 6) << 4);
  }
}

// 16 bytes from a 2-byte-aligned global address, as four little-endian words.
__device__ __forceinline__ uint4 ldg16_align2(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t s = (uint32_t)(a & 3u) * 8u;  // 0 or 16
  // The fifth word is read even when p is 4-aligned: every chunk this is used
  // for ends at least 4 bytes before the end of its 210-byte block.
  const uint32_t w0 = __ldg(w), w1 = __ldg(w + 1), w2 = __ldg(w + 2), w3 = __ldg(w + 3);
  const uint32_t w4 = __ldg(w + 4);
  uint4 r;
  r.x = __funnelshift_r(w0, w1, s);
  r.y = __funnelshift_r(w1, w2, s);
  r.z = __funnelshift_r(w2, w3, s);
  r.w = __funnelshift_r(w3, w4, s);
  return r;
}

__device__ __forceinline__ uint32_t ldg_u16(const uint8_t* p) {
  return (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(p));
}

}  // namespace lb
