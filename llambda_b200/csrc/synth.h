/*
 * Seeded synthetic GGUF workload generator, shared bit-for-bit by host (gcc/g++)
 * and device (nvcc) code.
 *
 * Every value is derived from a counter-based hash (the SplitMix64 finaliser of
 * Steele, Lea and Flood, "Fast splittable pseudorandom number generators",
 * OOPSLA 2014) of (seed, stream, counter), using integer arithmetic only.  The
 * single floating-point step per value is one IEEE-754 binary32 multiply by a
 * constant, which is correctly rounded on both the CPU and the GPU, and the
 * fp16 encoding is an integer round-to-nearest-even.  So a block generated on
 * the device is byte-identical to the same block generated on the host, and
 * parity tests can fill hundreds of megabytes on the GPU while the CPU oracle
 * regenerates exactly the rows it checks.
 *
 * Distributions follow the benchmark configurations:
 *   Q4_K: scales/mins uniform 0..63, nibbles uniform 0..15,
 *         d and dmin = fp16(|N(0,1)| * dscale)
 *   Q6_K: 6-bit quants uniform 0..63, int8 sub-scales uniform -128..127,
 *         d = fp16(|N(0,1)| * dscale)  (dscale 0.001 produces fp16 subnormals)
 *   F32:  N(0, sigma)
 * N(0,1) is approximated by a standardised Irwin-Hall sum of four uniform
 * 16-bit integers (mean 131070, standard deviation 65536/sqrt(3)); the
 * approximation keeps the generator integer-exact on both sides.
 *
 * Block layouts are those of GGUF (ggml) super-blocks of 256 values:
 *   Q4_K: d:f16, dmin:f16, scales[12], qs[128]            = 144 bytes
 *   Q6_K: ql[128], qh[64], scales:int8[16], d:f16          = 210 bytes
 */
#ifndef LLAMBDA_B200_SYNTH_H
#define LLAMBDA_B200_SYNTH_H

#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define LB_HD __host__ __device__ __forceinline__
#else
#define LB_HD static inline
#endif

#define LB_QK_K 256
#define LB_Q4K_BYTES 144
#define LB_Q6K_BYTES 210

/* Irwin-Hall(4) of 16-bit uniforms: mean and 1/sigma. */
#define LB_IH_MEAN 131070
/* 1 / 37837.227 rounded to binary32, written exactly so every compiler agrees */
#define LB_IH_INV_SIGMA 0x1.bb67b0p-16f

LB_HD uint64_t lb_mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

LB_HD uint64_t lb_hash(uint64_t seed, uint64_t stream, uint64_t counter) {
  uint64_t key = lb_mix64(seed ^ lb_mix64(stream * 0xD1342543DE82EF95ull + 1ull));
  return lb_mix64(key ^ (counter * 0x9E3779B97F4A7C15ull));
}

/* Signed Irwin-Hall deviate in [-131070, 131070] from one 64-bit word. */
LB_HD int32_t lb_ih_deviate(uint64_t w) {
  int32_t s = (int32_t)(w & 0xFFFF) + (int32_t)((w >> 16) & 0xFFFF) +
              (int32_t)((w >> 32) & 0xFFFF) + (int32_t)((w >> 48) & 0xFFFF);
  return s - LB_IH_MEAN;
}

/* Scale factor turning an Irwin-Hall deviate into N(0, sigma): one correctly
 * rounded binary32 multiply, so host and device agree. */
LB_HD float lb_sigma_scale(float sigma) { return sigma * LB_IH_INV_SIGMA; }

/* N(0, sigma) sample: exact int->float, then one correctly rounded multiply
 * (no add, so no FMA contraction can change it). */
LB_HD float lb_normal(uint64_t w, float sigma_over_ih) {
  return (float)lb_ih_deviate(w) * sigma_over_ih;
}

LB_HD uint32_t lb_f32_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof(u));
  return u;
}

/* IEEE binary32 -> binary16 bits, round to nearest even, integer-only. */
LB_HD uint16_t lb_f32_to_f16_rne(float f) {
  uint32_t x = lb_f32_bits(f);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) { /* inf or nan */
    return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x0200u : 0u));
  }
  if (ax >= 0x477FF000u) { /* >= 65520 rounds to inf */
    return (uint16_t)(sign | 0x7C00u);
  }
  if (ax >= 0x38800000u) { /* normal half: |f| >= 2^-14 */
    uint32_t r = ax - 0x38000000u; /* rebias exponent 127 -> 15 */
    uint32_t lsb = (r >> 13) & 1u;
    r = (r + 0x0FFFu + lsb) >> 13;
    return (uint16_t)(sign | r);
  }
  if (ax < 0x33000000u) { /* < 2^-25: rounds to zero (2^-25 ties to even 0) */
    return (uint16_t)sign;
  }
  /* subnormal half: value / 2^-24 rounded to nearest even integer */
  {
    uint32_t e = ax >> 23;                      /* 102 .. 112 */
    uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;  /* 24-bit significand */
    uint32_t shift = 126u - e;                  /* 14 .. 24 */
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (q & 1u))) q += 1u;
    return (uint16_t)(sign | q);
  }
}

/* Stream ids keep tensors of one layer independent. */
enum {
  LB_STREAM_ACTIVATION = 1,
  LB_STREAM_ROUTER = 2,
  LB_STREAM_ROUTER_BIAS = 3,
  LB_STREAM_SHARED_GATE_INP = 4,
  LB_STREAM_GATE_EXPS = 5,
  LB_STREAM_UP_EXPS = 6,
  LB_STREAM_DOWN_EXPS = 7,
  LB_STREAM_GATE_SHEXP = 8,
  LB_STREAM_UP_SHEXP = 9,
  LB_STREAM_DOWN_SHEXP = 10,
  LB_STREAM_DENSE = 11
};

/* Counters per block: 32 hash words per block index leave room for both types. */
#define LB_WORDS_PER_BLOCK 32ull

/* Writes the 144-byte Q4_K super-block number `block`. */
LB_HD void lb_q4k_block(uint64_t seed, uint64_t stream, uint64_t block,
                        float dscale_over_ih, uint8_t *out) {
  uint64_t base = block * LB_WORDS_PER_BLOCK;
  for (int j = 0; j < 18; ++j) {
    uint64_t w = lb_hash(seed, stream, base + (uint64_t)j);
    for (int b = 0; b < 8; ++b) out[j * 8 + b] = (uint8_t)(w >> (8 * b));
  }
  {
    int32_t nd = lb_ih_deviate(lb_hash(seed, stream, base + 18u));
    int32_t nm = lb_ih_deviate(lb_hash(seed, stream, base + 19u));
    float d = (float)(nd < 0 ? -nd : nd) * dscale_over_ih;
    float dmin = (float)(nm < 0 ? -nm : nm) * dscale_over_ih;
    uint16_t hd = lb_f32_to_f16_rne(d), hm = lb_f32_to_f16_rne(dmin);
    out[0] = (uint8_t)hd;
    out[1] = (uint8_t)(hd >> 8);
    out[2] = (uint8_t)hm;
    out[3] = (uint8_t)(hm >> 8);
  }
}

/* Writes the 210-byte Q6_K super-block number `block`. */
LB_HD void lb_q6k_block(uint64_t seed, uint64_t stream, uint64_t block,
                        float dscale_over_ih, uint8_t *out) {
  uint64_t base = block * LB_WORDS_PER_BLOCK;
  for (int j = 0; j < 27; ++j) {
    uint64_t w = lb_hash(seed, stream, base + (uint64_t)j);
    for (int b = 0; b < 8; ++b) {
      int k = j * 8 + b;
      if (k < 208) out[k] = (uint8_t)(w >> (8 * b));
    }
  }
  {
    int32_t nd = lb_ih_deviate(lb_hash(seed, stream, base + 27u));
    float d = (float)(nd < 0 ? -nd : nd) * dscale_over_ih;
    uint16_t hd = lb_f32_to_f16_rne(d);
    out[208] = (uint8_t)hd;
    out[209] = (uint8_t)(hd >> 8);
  }
}

/* Element `index` of an F32 tensor drawn from N(0, sigma). */
LB_HD float lb_f32_value(uint64_t seed, uint64_t stream, uint64_t index,
                         float sigma_over_ih) {
  return lb_normal(lb_hash(seed, stream, index), sigma_over_ih);
}

#endif /* LLAMBDA_B200_SYNTH_H */
