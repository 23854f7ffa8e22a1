// Dequant-fused row dots for Q4_K and Q6_K on CUDA cores.
//
// A row of K columns is split into K/64 "tasks" of 64 weights:
//   Q4_K task t = (super-block t/4, sub-block pair p = t%4): qs bytes
//     [32p, 32p+32) hold sub-block 2p in their low nibbles and 2p+1 in their
//     high nibbles (dot-product-with-q4-k-m-tensor-data, llambda.lisp
//     L4338-4382, expand-q4-k-body L4145-4201).
//   Q6_K task t = (super-block t/4, 128-chunk c = (t/2)%2, half h = t%2): 16 bytes
//     of ql at 64c+16h and 64c+32+16h and 16 bytes of qh at 128+32c+16h give
//     the 64 weights of sub-blocks 8c+h+2g, g = 0..3 (expand-q6-k-group,
//     L4203-4310, q6-quant-1..4, L4115-4137).
// Lanes of a warp take tasks of one row in stride, so a warp's loads cover
// whole super-blocks, and partial sums meet in a shuffle reduction.
//
// Arithmetic: sum(d*sc*q - dmin*m) * x over a sub-block is evaluated as
// (d*sc) * sum(q*x) - (dmin*m) * sum(x).  q becomes a float with one PRMT
// (magic_q: 2^23 + 2^16 q), so sum(q*x) = acc * 2^-16 - 128 * sum(x); the
// per-sub-block sums of x are staged once per token with the activations.
// Weights stay exact small integers, every product and sum is fp32.
#pragma once

#include "common.cuh"

namespace lb {

// Activation staging in shared memory, per token:
//   xs[tok][i][task] : float4 i (0..15) of the task's 64 activations,
//                      task-minor so that lanes reading consecutive tasks
//                      hit consecutive 16-byte bank groups;
//   sx[tok][grp]     : sum of x over each sub-block (32 values for Q4_K,
//                      16 values for Q6_K).
struct XView {
  const float4* xs;
  const float* sx;
  int tasks;   // K / 64
  int groups;  // K / 32 (Q4_K) or K / 16 (Q6_K)
};

// Element e (0..K-1) of the activation vector -> (task, float4 slot) in xs.
template <int TYPE>
__device__ __forceinline__ void stage_slot(int e, int& task, int& i) {
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
}

template <int TYPE>
__host__ __device__ constexpr int group_size() { return TYPE == LB_TYPE_Q4_K ? 32 : 16; }

// Stage `ntok` activation vectors (token t at src[t * ld], n_valid values,
// zero-padded to K) into xs/sx.  Called by all threads of the block; the
// caller synchronises before use.  `gather` (optional) maps the staged token
// index to the source row.
template <int TYPE>
__device__ void stage_x(float4* xs, float* sx, const float* src, long ld, const int* gather,
                        int ntok, int K, int n_valid) {
  const int tasks = K >> 6;
  const int nf4 = K >> 2;
  for (int idx = threadIdx.x; idx < ntok * nf4; idx += blockDim.x) {
    const int tok = idx / nf4, f = idx - tok * nf4;
    const long row = gather ? gather[tok] : tok;
    const float* s = src + row * ld;
    const int e = f * 4;
    float4 v;
    if (e + 3 < n_valid && (reinterpret_cast<uintptr_t>(s + e) & 15u) == 0) {
      v = *reinterpret_cast<const float4*>(s + e);
    } else {
      v.x = e < n_valid ? s[e] : 0.f;
      v.y = e + 1 < n_valid ? s[e + 1] : 0.f;
      v.z = e + 2 < n_valid ? s[e + 2] : 0.f;
      v.w = e + 3 < n_valid ? s[e + 3] : 0.f;
    }
    int task, i;
    stage_slot<TYPE>(e, task, i);
    xs[(tok * 16 + i) * tasks + task] = v;
  }
  constexpr int G = group_size<TYPE>();
  const int groups = K / G;
  for (int idx = threadIdx.x; idx < ntok * groups; idx += blockDim.x) {
    const int tok = idx / groups, g = idx - tok * groups;
    const long row = gather ? gather[tok] : tok;
    const float* s = src + row * ld + g * G;
    float acc = 0.f;
#pragma unroll 4
    for (int j = 0; j < G; ++j) acc += (g * G + j < n_valid) ? s[j] : 0.f;
    sx[tok * groups + g] = acc;
  }
}

// One Q4_K task of one row against NTOK staged tokens; adds into y[].
template <int NTOK>
__device__ __forceinline__ void q4k_task(const uint8_t* row, int task, const XView& xv, int ntok,
                                         float (&y)[NTOK]) {
  const int sb = task >> 2, p = task & 3;
  const uint8_t* blk = row + (size_t)sb * LB_Q4K;
  const uint4 hdr = __ldg(reinterpret_cast<const uint4*>(blk));
  const uint4 qa = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 32 * p));
  const uint4 qb = __ldg(reinterpret_cast<const uint4*>(blk + 32 + 32 * p));
  const float d = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
  int sc0, m0, sc1, m1;
  q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * p, sc0, m0);
  q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * p + 1, sc1, m1);
  // delta = d * sc and offset = dmin * m, single-rounded as in L4363-4366.
  const float dsc0 = d * (float)sc0, dm0 = dmin * (float)m0;
  const float dsc1 = d * (float)sc1, dm1 = dmin * (float)m1;
  const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
  float al[NTOK], ah[NTOK];
#pragma unroll
  for (int t = 0; t < NTOK; ++t) al[t] = ah[t] = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t lo = w[j] & 0x0F0F0F0Fu, hi = (w[j] >> 4) & 0x0F0F0F0Fu;
    const float l0 = magic_q<0>(lo), l1 = magic_q<1>(lo), l2 = magic_q<2>(lo), l3 = magic_q<3>(lo);
    const float h0 = magic_q<0>(hi), h1 = magic_q<1>(hi), h2 = magic_q<2>(hi), h3 = magic_q<3>(hi);
#pragma unroll
    for (int t = 0; t < NTOK; ++t) {
      if (t < ntok) {
        const float4 xl = xv.xs[(t * 16 + j) * xv.tasks + task];
        const float4 xh = xv.xs[(t * 16 + 8 + j) * xv.tasks + task];
        al[t] = fmaf(l0, xl.x, al[t]); al[t] = fmaf(l1, xl.y, al[t]);
        al[t] = fmaf(l2, xl.z, al[t]); al[t] = fmaf(l3, xl.w, al[t]);
        ah[t] = fmaf(h0, xh.x, ah[t]); ah[t] = fmaf(h1, xh.y, ah[t]);
        ah[t] = fmaf(h2, xh.z, ah[t]); ah[t] = fmaf(h3, xh.w, ah[t]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < NTOK; ++t) {
    if (t < ntok) {
      const float sxl = xv.sx[t * xv.groups + 2 * task];
      const float sxh = xv.sx[t * xv.groups + 2 * task + 1];
      const float ql = fmaf(al[t], kMagicUnscale, -kMagicBias * sxl);  // sum(q*x), low
      const float qh = fmaf(ah[t], kMagicUnscale, -kMagicBias * sxh);  // sum(q*x), high
      float acc = y[t];
      acc = fmaf(dsc0, ql, acc);
      acc = fmaf(-dm0, sxl, acc);
      acc = fmaf(dsc1, qh, acc);
      acc = fmaf(-dm1, sxh, acc);
      y[t] = acc;
    }
  }
}

// One Q6_K task of one row against NTOK staged tokens; adds into y[].
template <int NTOK>
__device__ __forceinline__ void q6k_task(const uint8_t* row, int task, const XView& xv, int ntok,
                                         float (&y)[NTOK]) {
  const int sb = task >> 2, c = (task >> 1) & 1, h = task & 1;
  const uint8_t* blk = row + (size_t)sb * LB_Q6K;
  const uint4 qa = ldg16_align2(blk + 64 * c + 16 * h);
  const uint4 qb = ldg16_align2(blk + 64 * c + 32 + 16 * h);
  const uint4 qhv = ldg16_align2(blk + 128 + 32 * c + 16 * h);
  const float d = half_bits_to_float(ldg_u16(blk + 208));
  float ds[4];
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int s = (int)(int8_t)(uint8_t)(ldg_u16(blk + 192 + 8 * c + 2 * g) >> (8 * h));
    ds[g] = d * (float)s;  // delta = d * sc, L4470-4473
  }
  const uint32_t A[4] = {qa.x, qa.y, qa.z, qa.w};
  const uint32_t B[4] = {qb.x, qb.y, qb.z, qb.w};
  const uint32_t H[4] = {qhv.x, qhv.y, qhv.z, qhv.w};
  float acc[4][NTOK];
#pragma unroll
  for (int g = 0; g < 4; ++g)
#pragma unroll
    for (int t = 0; t < NTOK; ++t) acc[g][t] = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    // 6-bit values 0..63 (the -32 is applied per sub-block below).
    uint32_t q[4];
    q[0] = (A[j] & 0x0F0F0F0Fu) | ((H[j] << 4) & 0x30303030u);
    q[1] = (B[j] & 0x0F0F0F0Fu) | ((H[j] << 2) & 0x30303030u);
    q[2] = ((A[j] >> 4) & 0x0F0F0F0Fu) | (H[j] & 0x30303030u);
    q[3] = ((B[j] >> 4) & 0x0F0F0F0Fu) | ((H[j] >> 2) & 0x30303030u);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const float f0 = magic_q<0>(q[g]), f1 = magic_q<1>(q[g]);
      const float f2 = magic_q<2>(q[g]), f3 = magic_q<3>(q[g]);
#pragma unroll
      for (int t = 0; t < NTOK; ++t) {
        if (t < ntok) {
          const float4 xq = xv.xs[(t * 16 + g * 4 + j) * xv.tasks + task];
          float a = acc[g][t];
          a = fmaf(f0, xq.x, a); a = fmaf(f1, xq.y, a);
          a = fmaf(f2, xq.z, a); a = fmaf(f3, xq.w, a);
          acc[g][t] = a;
        }
      }
    }
  }
  const int gbase = sb * 16 + c * 8 + h;  // global 16-value sub-block of g = 0
#pragma unroll
  for (int t = 0; t < NTOK; ++t) {
    if (t < ntok) {
      float out = y[t];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const float s = xv.sx[t * xv.groups + gbase + 2 * g];
        // sum((q6 - 32) * x) = acc * 2^-16 - (128 + 32) * sum(x)
        const float qs = fmaf(acc[g][t], kMagicUnscale, -(kMagicBias + 32.0f) * s);
        out = fmaf(ds[g], qs, out);
      }
      y[t] = out;
    }
  }
}

// Lanes per row: the row's tasks are spread over a power-of-two lane group.
__host__ __device__ __forceinline__ int lanes_per_row(int tasks) {
  int l = 1;
  while (l < tasks && l < 32) l <<= 1;
  return l;
}

// Dot products of one row (given by its byte pointer) with the staged tokens,
// computed by the lane group `lt` (0..lpr-1) and reduced within the group.
template <int TYPE, int NTOK>
__device__ __forceinline__ void row_dot(const uint8_t* row, bool valid, const XView& xv, int ntok,
                                        int lt, int lpr, float (&y)[NTOK]) {
#pragma unroll
  for (int t = 0; t < NTOK; ++t) y[t] = 0.f;
  if (valid) {
    for (int task = lt; task < xv.tasks; task += lpr) {
      if (TYPE == LB_TYPE_Q4_K)
        q4k_task<NTOK>(row, task, xv, ntok, y);
      else
        q6k_task<NTOK>(row, task, xv, ntok, y);
    }
  }
#pragma unroll
  for (int t = 0; t < NTOK; ++t) y[t] = warp_sum(y[t], lpr);
}

template <int TYPE>
__host__ __device__ __forceinline__ size_t stage_bytes(int ntok, int K) {
  return (size_t)ntok * ((size_t)K * 4 + (size_t)(K / group_size<TYPE>()) * 4);
}

}  // namespace lb
