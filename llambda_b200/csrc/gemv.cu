// Dense dequant-fused GEMV for raw GGUF Q4_K / Q6_K / F32 tensors, the fp16
// scale validator and the synthetic-data fill kernels.
//
// Replaces %gguf-model-matrix-vector-multiply-into (llambda.lisp L4542-4658),
// which splits rows over lparallel workers and runs an 8-lane AVX2 loop per
// row.  Here every warp owns rows and its lanes own 64-weight tasks of a row;
// weights stream once from HBM in 16-byte loads and never touch shared memory,
// activations are staged once per CTA in a bank-conflict-free task-minor
// layout and reused by every row the CTA computes.
#include <algorithm>

#include "kernels.h"
#include "rowdot.cuh"
#include "synth.h"

namespace lb {

namespace {

constexpr int kThreads = 256;

template <int TYPE, int NT>
__global__ void __launch_bounds__(kThreads) gemv_quant_kernel(const uint8_t* __restrict__ W,
                                                               size_t rb, int rows, int K,
                                                               const float* __restrict__ x,
                                                               long ldx, int n_valid, int tokens,
                                                               float* __restrict__ y, long ldy) {
  extern __shared__ float4 smem4[];
  const int tasks = K >> 6;
  constexpr int G = group_size<TYPE>();
  float4* xs = smem4;
  float* sx = reinterpret_cast<float*>(smem4 + NT * 16 * tasks);
  const XView xv{xs, sx, tasks, K / G};
  const int lpr = lanes_per_row(tasks);
  const int rpw = 32 / lpr;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int lt = lane % lpr;
  for (int t0 = 0; t0 < tokens; t0 += NT) {
    const int nt = min(NT, tokens - t0);
    if (t0) __syncthreads();
    stage_x<TYPE>(xs, sx, x + (long)t0 * ldx, ldx, nullptr, nt, K, n_valid);
    __syncthreads();
    for (int r0 = (blockIdx.x * nwarps + warp) * rpw; r0 < rows; r0 += gridDim.x * nwarps * rpw) {
      const int row = r0 + lane / lpr;
      const bool ok = row < rows;
      float acc[NT];
      row_dot<TYPE, NT>(W + (size_t)(ok ? row : 0) * rb, ok, xv, nt, lt, lpr, acc);
      if (lt == 0 && ok) {
#pragma unroll
        for (int t = 0; t < NT; ++t)
          if (t < nt) y[(long)(t0 + t) * ldy + row] = acc[t];
      }
    }
  }
}

// F32 rows (the MoE router, ffn_gate_inp): one warp per row, float4 loads.
template <int NT>
__global__ void __launch_bounds__(kThreads) gemv_f32_kernel(const float* __restrict__ W, int rows,
                                                             int K, const float* __restrict__ x,
                                                             long ldx, int tokens,
                                                             float* __restrict__ y, long ldy) {
  extern __shared__ float4 smem4[];
  float* xs = reinterpret_cast<float*>(smem4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int K4 = K >> 2;
  for (int t0 = 0; t0 < tokens; t0 += NT) {
    const int nt = min(NT, tokens - t0);
    if (t0) __syncthreads();
    for (int i = threadIdx.x; i < nt * K; i += blockDim.x) {
      const int t = i / K, k = i - t * K;
      xs[t * K + k] = x[(long)(t0 + t) * ldx + k];
    }
    __syncthreads();
    for (int row = blockIdx.x * nwarps + warp; row < rows; row += gridDim.x * nwarps) {
      const float* wr = W + (size_t)row * K;
      float acc[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t] = 0.f;
      if ((reinterpret_cast<uintptr_t>(wr) & 15) == 0) {
        const float4* w4 = reinterpret_cast<const float4*>(wr);
        for (int k4 = lane; k4 < K4; k4 += 32) {
          const float4 w = __ldg(w4 + k4);
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            if (t < nt) {
              const float4 v = reinterpret_cast<const float4*>(xs + t * K)[k4];
              acc[t] = fmaf(w.x, v.x, acc[t]);
              acc[t] = fmaf(w.y, v.y, acc[t]);
              acc[t] = fmaf(w.z, v.z, acc[t]);
              acc[t] = fmaf(w.w, v.w, acc[t]);
            }
          }
        }
        for (int k = K4 * 4 + lane; k < K; k += 32) {
          const float w = __ldg(wr + k);
#pragma unroll
          for (int t = 0; t < NT; ++t)
            if (t < nt) acc[t] = fmaf(w, xs[t * K + k], acc[t]);
        }
      } else {
        for (int k = lane; k < K; k += 32) {
          const float w = __ldg(wr + k);
#pragma unroll
          for (int t = 0; t < NT; ++t)
            if (t < nt) acc[t] = fmaf(w, xs[t * K + k], acc[t]);
        }
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t] = warp_sum(acc[t]);
      if (lane == 0) {
#pragma unroll
        for (int t = 0; t < NT; ++t)
          if (t < nt) y[(long)(t0 + t) * ldy + row] = acc[t];
      }
    }
  }
}

__global__ void check_scales_kernel(int type, const uint8_t* __restrict__ W, size_t blocks,
                                    unsigned* bad) {
  unsigned local = 0;
  for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < blocks;
       b += (size_t)gridDim.x * blockDim.x) {
    if (type == LB_TYPE_Q4_K) {
      const uint8_t* p = W + b * LB_Q4K;
      const uint32_t d = p[0] | (p[1] << 8), m = p[2] | (p[3] << 8);
      local += ((d & 0x7C00u) == 0x7C00u) || ((m & 0x7C00u) == 0x7C00u);
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

template <int TYPE, int NT>
cudaError_t launch_quant(const void* W, size_t rb, int rows, int K, const float* x, long ldx,
                         int n_valid, int tokens, float* y, long ldy, cudaStream_t stream) {
  const size_t smem = stage_bytes<TYPE>(NT, K);
  auto kern = gemv_quant_kernel<TYPE, NT>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
  }
  const int tasks = K / 64;
  const int rpw = 32 / lanes_per_row(tasks);
  const long warps_needed = (rows + rpw - 1) / rpw;
  const int per_sm = std::max(1, (int)std::min<size_t>(8, (200 * 1024) / std::max<size_t>(smem, 1)));
  const long blocks = std::min<long>((warps_needed + 7) / 8, (long)sm_count() * per_sm);
  kern<<<(int)std::max<long>(blocks, 1), kThreads, smem, stream>>>(
      static_cast<const uint8_t*>(W), rb, rows, K, x, ldx, n_valid, tokens, y, ldy);
  return cudaGetLastError();
}

template <int NT>
cudaError_t launch_f32(const void* W, int rows, int K, const float* x, long ldx, int tokens,
                       float* y, long ldy, cudaStream_t stream) {
  const size_t smem = (size_t)NT * K * 4;
  auto kern = gemv_f32_kernel<NT>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
  }
  const long blocks = std::min<long>((rows + 7) / 8, (long)sm_count() * 8);
  kern<<<(int)std::max<long>(blocks, 1), kThreads, smem, stream>>>(
      static_cast<const float*>(W), rows, K, x, ldx, tokens, y, ldy);
  return cudaGetLastError();
}

// Largest token tile (1, 2, 4 or 8) whose staging fits comfortably in shared memory.
int token_tile(int tokens, size_t bytes_per_token) {
  int nt = 1;
  while (nt < 8 && nt < tokens && (size_t)(nt * 2) * bytes_per_token <= 160 * 1024) nt *= 2;
  return nt;
}

}  // namespace

cudaError_t launch_gemv(int type, const void* W, size_t rb, int rows, int K, const float* x,
                        long ldx, int n_valid, int tokens, float* y, long ldy,
                        cudaStream_t stream) {
  if (rows <= 0 || tokens <= 0) return cudaSuccess;
  if (type == LB_TYPE_F32) {
    const int nt = token_tile(tokens, (size_t)K * 4);
    switch (nt) {
      case 1: return launch_f32<1>(W, rows, K, x, ldx, tokens, y, ldy, stream);
      case 2: return launch_f32<2>(W, rows, K, x, ldx, tokens, y, ldy, stream);
      case 4: return launch_f32<4>(W, rows, K, x, ldx, tokens, y, ldy, stream);
      default: return launch_f32<8>(W, rows, K, x, ldx, tokens, y, ldy, stream);
    }
  }
  if (type == LB_TYPE_Q4_K) {
    const int nt = token_tile(tokens, stage_bytes<LB_TYPE_Q4_K>(1, K));
    switch (nt) {
      case 1: return launch_quant<LB_TYPE_Q4_K, 1>(W, rb, rows, K, x, ldx, n_valid, tokens, y, ldy, stream);
      case 2: return launch_quant<LB_TYPE_Q4_K, 2>(W, rb, rows, K, x, ldx, n_valid, tokens, y, ldy, stream);
      case 4: return launch_quant<LB_TYPE_Q4_K, 4>(W, rb, rows, K, x, ldx, n_valid, tokens, y, ldy, stream);
      default: return launch_quant<LB_TYPE_Q4_K, 8>(W, rb, rows, K, x, ldx, n_valid, tokens, y, ldy, stream);
    }
  }
  if (type == LB_TYPE_Q6_K) {
    const int nt = token_tile(tokens, stage_bytes<LB_TYPE_Q6_K>(1, K));
    switch (nt) {
      case 1: return launch_quant<LB_TYPE_Q6_K, 1>(W, rb, rows, K, x, ldx, n_valid, tokens, y, ldy, stream);
      case 2: return launch_quant<LB_TYPE_Q6_K, 2>(W, rb, rows, K, x, ldx, n_valid, tokens, y, ldy, stream);
      case 4: return launch_quant<LB_TYPE_Q6_K, 4>(W, rb, rows, K, x, ldx, n_valid, tokens, y, ldy, stream);
      default: return launch_quant<LB_TYPE_Q6_K, 8>(W, rb, rows, K, x, ldx, n_valid, tokens, y, ldy, stream);
    }
  }
  return cudaErrorInvalidValue;
}

cudaError_t check_fp16_scales(int type, const void* W, size_t blocks, unsigned* bad,
                              cudaStream_t stream) {
  if (type != LB_TYPE_Q4_K && type != LB_TYPE_Q6_K) return cudaSuccess;
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
