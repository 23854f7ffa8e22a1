// Routed-MoE feed-forward layer (qwen3next and nemotron_h_moe) for a batch of
// tokens on device-resident raw GGUF expert tensors.
//
// Reference: qwen3next-moe-into (llambda.lisp L5321-5426) and
// nemotron-h-moe-ffn-into (L5827-5949).  The reference runs one token at a
// time and, per selected expert, three (or two) separate row-parallel GEMVs.
// Here one layer call is four launches over the whole batch:
//   1. router GEMV (F32) for every token, plus the qwen3next shared-gate row;
//   2. route: top-k per token (select-top-k-logits-into, L5265-5292),
//      sigmoid weights with the reference's normalisation rules, and a stable
//      grouping of (token, rank) entries by expert;
//   3. up: for every active expert and row chunk, gate/up rows for all of its
//      tokens with SwiGLU (silu(gate) * up) or ReLU^2 applied in registers;
//   4. down: the expert's down rows for the same tokens, then a combine that
//      adds weight * down in rank order (vector-add-scaled-in-place, L3465)
//      and the shared expert last, exactly the reference's summation order.
#include <algorithm>

#include "kernels.h"
#include "rowdot.cuh"

namespace lb {

namespace {

constexpr int kThreads = 256;
constexpr int kMaxExperts = 1024;

// exp of a single-float as SBCL evaluates it (in double, rounded to single),
// then silu / sigmoid divide in double (llambda.lisp L926-930).
__device__ __forceinline__ float exp_single(float v) { return (float)exp((double)v); }
__device__ __forceinline__ float sigmoid_ref(float v) {
  return (float)(1.0 / (1.0 + (double)exp_single(-v)));
}
__device__ __forceinline__ float silu_ref(float v) {
  return (float)((double)v / (1.0 + (double)exp_single(-v)));
}
__device__ __forceinline__ float relu_sq_ref(float v) {
  const float x = v > 0.f ? v : 0.f;
  return __fmul_rn(x, x);
}

// ---------------------------------------------------------------- route
__global__ void __launch_bounds__(1024) route_kernel(MoeDevice m, MoeWork w, int T) {
  __shared__ int s_count[kMaxExperts];
  __shared__ int s_offset[kMaxExperts + 1];
  const int E = m.experts, k = m.top_k;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int ld = E + 1;
  // Top-k and weights, one warp per token.
  for (int t = warp; t < T; t += nwarps) {
    const float* L = w.logits + (long)t * ld;
    const int per_lane = (E + 31) / 32;  // <= 32
    uint32_t taken = 0;
    float wsum = 0.f;
    float wk[32];
    int ik[32];
    for (int j = 0; j < k; ++j) {
      float best = -3.40282347e38f;  // most-negative-single-float: never selected
      int bi = -1;
      for (int q = 0; q < per_lane; ++q) {
        const int i = lane + 32 * q;
        if (i >= E || ((taken >> q) & 1u)) continue;
        float v = L[i];
        if (m.router_bias) v = v + m.router_bias[i];
        if (v > best) { best = v; bi = i; }  // strict: lower index wins ties
      }
      // warp arg-max, ties to the lower index
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi >= 0 && (bi < 0 || ob > best || (ob == best && oi < bi))) { best = ob; bi = oi; }
      }
      if (bi >= 0 && (bi & 31) == lane) taken |= 1u << (bi >> 5);
      ik[j < 32 ? j : 31] = bi;
      wk[j < 32 ? j : 31] = best;
    }
    if (lane == 0) {
      int bad = 0;
      for (int j = 0; j < k; ++j) {
        const float wv = sigmoid_ref(wk[j]);
        wk[j] = wv;
        wsum = wsum + wv;
        bad |= ik[j] < 0;
      }
      if (m.arch == 0 || m.weights_norm) {
        if (!(wsum > 0.f)) bad = 1;
        for (int j = 0; j < k; ++j) wk[j] = wk[j] / wsum;
      }
      if (m.arch == 1)
        for (int j = 0; j < k; ++j) wk[j] = __fmul_rn(m.weight_scale, wk[j]);
      for (int j = 0; j < k; ++j) {
        w.sel[t * k + j] = ik[j];
        w.wts[t * k + j] = wk[j];
      }
      w.shw[t] = (m.arch == 0) ? sigmoid_ref(L[E]) : 1.0f;
      if (bad) atomicOr(w.status, 1);
    }
  }
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_count[e] = 0;
  __syncthreads();
  // Stable grouping of entries (token-major, rank-minor) by owned expert.
  const int n = T * k;
  if (warp == 0) {
    const unsigned lt_mask = (1u << lane) - 1u;
    for (int c = 0; c < n; c += 32) {
      const int id = c + lane;
      int e = id < n ? w.sel[id] : -1;
      const bool own = e >= m.expert_begin && e < m.expert_end;
      const unsigned act = __ballot_sync(0xffffffffu, own);
      int rank = 0;
      unsigned grp = 0;
      if (own) {
        grp = __match_any_sync(act, e);
        rank = __popc(grp & lt_mask);
      }
      int base = own ? s_count[e] : 0;
      __syncwarp();
      if (own && rank == 0) s_count[e] = base + __popc(grp);
      __syncwarp();
      if (id < n) w.entries[id] = own ? (base + rank) : -1;  // position, fixed below
    }
    // exclusive scan over experts, active list in increasing expert id
    int run = 0, nact = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const int cnt = e < E ? s_count[e] : 0;
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (e < E) s_offset[e] = run + incl - cnt;
      const unsigned nz = __ballot_sync(0xffffffffu, cnt > 0);
      if (cnt > 0) w.active[nact + __popc(nz & lt_mask)] = e;
      nact += __popc(nz);
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      s_offset[E] = run;
      w.active[E] = nact;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    w.counts[e] = s_count[e];
    w.offsets[e] = s_offset[e];
  }
  if (threadIdx.x == 0) w.offsets[E] = s_offset[E];
  __syncthreads();
  // Scatter entry ids into their expert-grouped slots (second half of entries;
  // the first half holds each entry's position within its expert).
  for (int id = threadIdx.x; id < n; id += blockDim.x) {
    const int pos = w.entries[id];
    if (pos >= 0) w.entries[T * k + s_offset[w.sel[id]] + pos] = id;
  }
}

// ---------------------------------------------------------------- up
template <int GT, int UT, int NT>
__global__ void __launch_bounds__(kThreads) up_kernel(MoeDevice m, MoeWork w, const float* x,
                                                      int T, int chunk, int chunk_sh) {
  extern __shared__ float4 smem4[];
  __shared__ int s_rows[NT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int k = m.top_k;
  const int inter_max = max(m.inter, m.inter_sh);
  const int nact = w.active[m.experts];
  const int per = (m.inter + chunk - 1) / chunk;
  const int per_sh = m.inter_sh ? (m.inter_sh + chunk_sh - 1) / chunk_sh : 0;
  const int total = nact * per + (m.shared_here ? per_sh : 0);
  for (int item = blockIdx.x; item < total; item += gridDim.x) {
    int e, row0, rows_end, ntok, K;
    const int* list = nullptr;
    const uint8_t *Wg, *Wu;
    size_t grb, urb;
    if (item < nact * per) {
      const int a = item / per;
      e = w.active[a];
      row0 = (item - a * per) * chunk;
      rows_end = min(row0 + chunk, m.inter);
      ntok = w.counts[e];
      list = w.entries + T * k + w.offsets[e];
      K = m.k_in;
      grb = m.gate_rb;
      urb = m.up_rb;
      Wg = m.gate_exps ? m.gate_exps + (size_t)e * m.inter * grb : nullptr;
      Wu = m.up_exps + (size_t)e * m.inter * urb;
    } else {
      e = -1;
      row0 = (item - nact * per) * chunk_sh;
      rows_end = min(row0 + chunk_sh, m.inter_sh);
      ntok = T;
      K = m.k_in_sh;
      grb = m.gate_sh_rb;
      urb = m.up_sh_rb;
      Wg = m.gate_sh;
      Wu = m.up_sh;
    }
    const int tasks = K >> 6;
    const int lpr = lanes_per_row(tasks), rpw = 32 / lpr, lt = lane % lpr;
    float4* xs = smem4;
    float* sx = reinterpret_cast<float*>(smem4 + NT * 16 * tasks);
    const XView xv{xs, sx, tasks, K / group_size<UT>()};
    for (int t0 = 0; t0 < ntok; t0 += NT) {
      const int nt = min(NT, ntok - t0);
      __syncthreads();
      if (threadIdx.x < nt) {
        const int id = list ? list[t0 + threadIdx.x] : (t0 + threadIdx.x);
        s_rows[threadIdx.x] = list ? id / k : id;
      }
      __syncthreads();
      stage_x<UT>(xs, sx, x, m.hidden, s_rows, nt, K, m.hidden);
      __syncthreads();
      for (int r = row0 + warp * rpw; r < rows_end; r += nwarps * rpw) {
        const int row = r + lane / lpr;
        const bool ok = row < rows_end;
        const int rr = ok ? row : row0;
        float u[NT];
        row_dot<UT, NT>(Wu + (size_t)rr * urb, ok, xv, nt, lt, lpr, u);
        float g[NT];
        if (m.arch == 0) row_dot<GT, NT>(Wg + (size_t)rr * grb, ok, xv, nt, lt, lpr, g);
        if (lt == 0 && ok) {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            if (t < nt) {
              const int id = list ? list[t0 + t] : (T * k + t0 + t);
              const float hv = (m.arch == 0) ? __fmul_rn(silu_ref(g[t]), u[t]) : relu_sq_ref(u[t]);
              w.hbuf[(long)id * inter_max + row] = hv;
            }
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------- down
template <int DT, int NT>
__global__ void __launch_bounds__(kThreads) down_kernel(MoeDevice m, MoeWork w, int T, int chunk) {
  extern __shared__ float4 smem4[];
  __shared__ int s_ids[NT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int k = m.top_k, H = m.hidden;
  const int inter_max = max(m.inter, m.inter_sh);
  const int nact = w.active[m.experts];
  const int per = (H + chunk - 1) / chunk;
  const int total = nact * per + ((m.shared_here && m.inter_sh) ? per : 0);
  for (int item = blockIdx.x; item < total; item += gridDim.x) {
    int row0, ntok, K, n_valid;
    const int* list = nullptr;
    const uint8_t* Wd;
    size_t rb;
    if (item < nact * per) {
      const int a = item / per;
      const int e = w.active[a];
      row0 = (item - a * per) * chunk;
      ntok = w.counts[e];
      list = w.entries + T * k + w.offsets[e];
      K = m.k_down;
      n_valid = m.inter;
      rb = m.down_rb;
      Wd = m.down_exps + (size_t)e * H * rb;
    } else {
      row0 = (item - nact * per) * chunk;
      ntok = T;
      K = m.k_down_sh;
      n_valid = m.inter_sh;
      rb = m.down_sh_rb;
      Wd = m.down_sh;
    }
    const int rows_end = min(row0 + chunk, H);
    const int tasks = K >> 6;
    const int lpr = lanes_per_row(tasks), rpw = 32 / lpr, lt = lane % lpr;
    float4* xs = smem4;
    float* sx = reinterpret_cast<float*>(smem4 + NT * 16 * tasks);
    const XView xv{xs, sx, tasks, K / group_size<DT>()};
    for (int t0 = 0; t0 < ntok; t0 += NT) {
      const int nt = min(NT, ntok - t0);
      __syncthreads();
      if (threadIdx.x < nt) s_ids[threadIdx.x] = list ? list[t0 + threadIdx.x] : (T * k + t0 + threadIdx.x);
      __syncthreads();
      stage_x<DT>(xs, sx, w.hbuf, inter_max, s_ids, nt, K, n_valid);
      __syncthreads();
      for (int r = row0 + warp * rpw; r < rows_end; r += nwarps * rpw) {
        const int row = r + lane / lpr;
        const bool ok = row < rows_end;
        float y[NT];
        row_dot<DT, NT>(Wd + (size_t)(ok ? row : row0) * rb, ok, xv, nt, lt, lpr, y);
        if (lt == 0 && ok) {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            if (t < nt) {
              const int id = s_ids[t];
              // routed entry id = token*k + rank -> slot (token, rank);
              // shared entry T*k + token -> slot (token, k)
              const int tok = id < T * k ? id / k : id - T * k;
              const int slot = id < T * k ? id - tok * k : k;
              w.partial[((long)tok * (k + 1) + slot) * H + row] = y[t];
            }
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------- norm
// rms-norm-into (llambda.lisp L859-879): scale = 1/sqrt(mean(x^2) + eps),
// dest = (x * weight) * scale.  One block per token.
__global__ void rms_norm_kernel(const float* __restrict__ x, const float* __restrict__ wgt,
                                float eps, int H, float* __restrict__ out) {
  __shared__ float s_part[32];
  const float* xt = x + (long)blockIdx.x * H;
  float acc = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) acc = fmaf(xt[i], xt[i], acc);
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? s_part[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) s_part[0] = v;
  }
  __syncthreads();
  const float ms = __fdiv_rn(s_part[0], (float)H);
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
  for (int i = threadIdx.x; i < H; i += blockDim.x)
    out[(long)blockIdx.x * H + i] = __fmul_rn(__fmul_rn(xt[i], wgt[i]), scale);
}

// ---------------------------------------------------------------- combine
__global__ void combine_kernel(MoeDevice m, MoeWork w, int T, const float* x, float* out) {
  const int H = m.hidden, k = m.top_k;
  const long n = (long)T * H;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const int t = (int)(i / H), h = (int)(i - (long)t * H);
    const float* p = w.partial + (long)t * (k + 1) * H + h;
    float acc = 0.f;
    for (int j = 0; j < k; ++j) {
      const int e = w.sel[t * k + j];
      if (e >= m.expert_begin && e < m.expert_end)
        acc = __fadd_rn(acc, __fmul_rn(w.wts[t * k + j], p[(long)j * H]));
    }
    if (m.shared_here && m.inter_sh) {
      const float s = p[(long)k * H];
      acc = (m.arch == 0) ? __fadd_rn(acc, __fmul_rn(w.shw[t], s)) : __fadd_rn(acc, s);
    }
    // vector-add-into x x ffn-output (L5746) when the layer carries the residual
    out[i] = m.add_residual ? __fadd_rn(x[i], acc) : acc;
  }
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

template <typename F>
cudaError_t prep(F kern, size_t smem) {
  if (smem > 48 * 1024)
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  return cudaSuccess;
}

template <int GT, int UT, int NT>
cudaError_t launch_up_t(const MoeDevice& m, const MoeWork& w, const float* x, int T,
                        cudaStream_t s) {
  const int K = std::max(m.k_in, m.k_in_sh);
  const size_t smem = stage_bytes<UT>(NT, K);
  auto kern = up_kernel<GT, UT, NT>;
  cudaError_t e = prep(kern, smem);
  if (e != cudaSuccess) return e;
  const int chunk = 16, chunk_sh = 16;
  kern<<<sm_count() * 4, kThreads, smem, s>>>(m, w, x, T, chunk, chunk_sh);
  return cudaGetLastError();
}

template <int DT, int NT>
cudaError_t launch_down_t(const MoeDevice& m, const MoeWork& w, int T, cudaStream_t s) {
  const int K = std::max(m.k_down, m.k_down_sh);
  const size_t smem = stage_bytes<DT>(NT, K);
  auto kern = down_kernel<DT, NT>;
  cudaError_t e = prep(kern, smem);
  if (e != cudaSuccess) return e;
  const int chunk = 32;
  kern<<<sm_count() * 4, kThreads, smem, s>>>(m, w, T, chunk);
  return cudaGetLastError();
}

int tile_for(int T) { return T >= 8 ? 8 : T >= 4 ? 4 : T >= 2 ? 2 : 1; }

}  // namespace

size_t moe_work_bytes(const MoeDevice& m, int T) {
  MoeWork w;
  moe_work_carve(m, T, nullptr, &w);
  return w.bytes;
}

void moe_work_carve(const MoeDevice& m, int T, void* base, MoeWork* w) {
  const int E = m.experts, k = m.top_k;
  const int inter_max = std::max(m.inter, m.inter_sh);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return base ? static_cast<char*>(base) + o : nullptr;
  };
  w->max_tokens = T;
  w->logits = reinterpret_cast<float*>(take((size_t)T * (E + 1) * 4));
  w->sel = reinterpret_cast<int*>(take((size_t)T * k * 4));
  w->wts = reinterpret_cast<float*>(take((size_t)T * k * 4));
  w->shw = reinterpret_cast<float*>(take((size_t)T * 4));
  w->counts = reinterpret_cast<int*>(take((size_t)E * 4));
  w->offsets = reinterpret_cast<int*>(take((size_t)(E + 1) * 4));
  w->entries = reinterpret_cast<int*>(take((size_t)T * k * 2 * 4));
  w->active = reinterpret_cast<int*>(take((size_t)(E + 1) * 4));
  w->status = reinterpret_cast<int*>(take(4));
  w->hbuf = reinterpret_cast<float*>(take((size_t)(T * k + T) * inter_max * 4));
  w->partial = reinterpret_cast<float*>(take((size_t)T * (k + 1) * m.hidden * 4));
  w->xnorm = reinterpret_cast<float*>(take(m.input_norm ? (size_t)T * m.hidden * 4 : 4));
  w->bytes = off;
}

cudaError_t launch_moe(const MoeDevice& m, const MoeWork& w, const float* x, int T, float* out,
                       cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  if (T > w.max_tokens || m.experts > kMaxExperts || m.top_k > 32 || T * m.top_k > 4 * 1024)
    return cudaErrorInvalidValue;
  const int E = m.experts;
  const int router_rows = E + (m.arch == 0 && !m.router_extra_row ? 1 : 0);
  const float* x_in = x;
  cudaError_t e;
  if (m.input_norm) {
    rms_norm_kernel<<<T, 256, 0, s>>>(x, m.input_norm, m.norm_epsilon, m.hidden, w.xnorm);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    x = w.xnorm;
  }
  if (m.arch == 0 && m.router_extra_row) {  // shared-expert gate logit into column E
    e = launch_gemv(LB_TYPE_F32, m.router_extra_row, (size_t)m.hidden * 4, 1, m.hidden, x,
                    m.hidden, m.hidden, T, w.logits + E, E + 1, s);
    if (e != cudaSuccess) return e;
  }
  e = launch_gemv(LB_TYPE_F32, m.router, (size_t)m.hidden * 4, router_rows, m.hidden,
                              x, m.hidden, m.hidden, T, w.logits, E + 1, s);
  if (e != cudaSuccess) return e;
  route_kernel<<<1, 1024, 0, s>>>(m, w, T);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  const int nt = tile_for(T);
  // gate/up: qwen3next gate and up share a type in practice; both Q4_K here.
  if (m.up_type == LB_TYPE_Q4_K && (m.arch == 1 || m.gate_type == LB_TYPE_Q4_K)) {
    switch (nt) {
      case 1: e = launch_up_t<LB_TYPE_Q4_K, LB_TYPE_Q4_K, 1>(m, w, x, T, s); break;
      case 2: e = launch_up_t<LB_TYPE_Q4_K, LB_TYPE_Q4_K, 2>(m, w, x, T, s); break;
      case 4: e = launch_up_t<LB_TYPE_Q4_K, LB_TYPE_Q4_K, 4>(m, w, x, T, s); break;
      default: e = launch_up_t<LB_TYPE_Q4_K, LB_TYPE_Q4_K, 8>(m, w, x, T, s); break;
    }
  } else if (m.up_type == LB_TYPE_Q6_K && (m.arch == 1 || m.gate_type == LB_TYPE_Q6_K)) {
    switch (nt) {
      case 1: e = launch_up_t<LB_TYPE_Q6_K, LB_TYPE_Q6_K, 1>(m, w, x, T, s); break;
      case 2: e = launch_up_t<LB_TYPE_Q6_K, LB_TYPE_Q6_K, 2>(m, w, x, T, s); break;
      case 4: e = launch_up_t<LB_TYPE_Q6_K, LB_TYPE_Q6_K, 4>(m, w, x, T, s); break;
      default: e = launch_up_t<LB_TYPE_Q6_K, LB_TYPE_Q6_K, 8>(m, w, x, T, s); break;
    }
  } else {
    return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) return e;
  if (m.down_type == LB_TYPE_Q6_K) {
    switch (nt) {
      case 1: e = launch_down_t<LB_TYPE_Q6_K, 1>(m, w, T, s); break;
      case 2: e = launch_down_t<LB_TYPE_Q6_K, 2>(m, w, T, s); break;
      case 4: e = launch_down_t<LB_TYPE_Q6_K, 4>(m, w, T, s); break;
      default: e = launch_down_t<LB_TYPE_Q6_K, 8>(m, w, T, s); break;
    }
  } else if (m.down_type == LB_TYPE_Q4_K) {
    switch (nt) {
      case 1: e = launch_down_t<LB_TYPE_Q4_K, 1>(m, w, T, s); break;
      case 2: e = launch_down_t<LB_TYPE_Q4_K, 2>(m, w, T, s); break;
      case 4: e = launch_down_t<LB_TYPE_Q4_K, 4>(m, w, T, s); break;
      default: e = launch_down_t<LB_TYPE_Q4_K, 8>(m, w, T, s); break;
    }
  } else {
    return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) return e;
  const long n = (long)T * m.hidden;
  const int grid = (int)std::min<long>((n + 255) / 256, (long)sm_count() * 8);
  combine_kernel<<<std::max(grid, 1), 256, 0, s>>>(m, w, T, x_in, out);
  return cudaGetLastError();
}

}  // namespace lb
