// Routed-MoE feed-forward layer (qwen3next and nemotron_h_moe) for a batch of
// tokens on device-resident raw GGUF expert tensors.
//
// Reference: qwen3next-moe-into (llambda.lisp L5321-5426) and
// nemotron-h-moe-ffn-into (L5827-5949).  The reference runs one token at a
// time and, per selected expert, three (or two) separate row-parallel GEMVs.
// Here one layer call runs over the whole batch:
//   1. prep: optional rms-norm, router input, prepared gate/up input;
//   2. router GEMV (F32) for every token, plus the qwen3next shared-gate row;
//   3. route: top-k per token (select-top-k-logits-into, L5265-5292),
//      sigmoid weights with the reference's normalisation rules, and a stable
//      grouping of (token, rank) entries by expert;
//   4. up (routed, then shared): TMA-staged units of gate/up rows of one
//      expert for all of its tokens, SwiGLU (silu(gate) * up) or ReLU^2 in
//      registers, written into the down projection's prepared input;
//   5. down (routed, then shared): TMA-staged units of down rows;
//   6. combine: weight * down added in rank order (vector-add-scaled-in-place,
//      L3465) and the shared expert last, the reference's summation order.
// In 4 and 5 every warp takes a contiguous run of units, so the expert's
// routing metadata and the token's activations stay in registers across the
// expert's units.
#include <algorithm>

#include "engine.cuh"
#include "kernels.h"

namespace lb {

namespace {

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
// Top-k and weights: one warp (block) per token.  Lane l holds logits l,
// l+32, ... (biased for nemotron, L5892) and its best remaining candidate;
// each rank is a warp arg-max (ties to the lower index, as the strict > of
// select-top-k-logits-into keeps the earlier logit) after which only the
// winning lane rescans its candidates.
__global__ void __launch_bounds__(32) topk_kernel(MoeDevice m, MoeWork w, int T) {
  const int t = blockIdx.x, lane = threadIdx.x;
  const int E = m.experts, k = m.top_k;
  const float* L = w.logits + (long)t * (E + 1);
  const int per = (E + 31) / 32;
  float lv[32];
  uint32_t taken = 0;  // bit q: candidate q of this lane is used or absent
#pragma unroll
  for (int q = 0; q < 32; ++q) {
    const int i = lane + 32 * q;
    float v = 0.f;
    if (q < per && i < E) {
      v = L[i];
      if (m.router_bias) v = v + m.router_bias[i];
    } else {
      taken |= 1u << q;
    }
    lv[q] = v;
  }
  auto local_best = [&](float& bv, int& bi) {
    bv = -3.40282347e38f;  // most-negative-single-float: never selected
    bi = -1;
#pragma unroll
    for (int q = 0; q < 32; ++q)
      if (!((taken >> q) & 1u) && lv[q] > bv) {  // strict: lower index wins ties
        bv = lv[q];
        bi = lane + 32 * q;
      }
  };
  float bv;
  int bi;
  local_best(bv, bi);
  int my_i = -1;  // lane j keeps rank j's expert and logit
  float my_v = 0.f;
  for (int j = 0; j < k; ++j) {
    float gv = bv;
    int gi = bi;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, gv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, gi, o);
      if (oi >= 0 && (gi < 0 || ov > gv || (ov == gv && oi < gi))) {
        gv = ov;
        gi = oi;
      }
    }
    if (lane == j) {
      my_i = gi;
      my_v = gv;
    }
    if (gi >= 0 && (gi & 31) == lane) {
      taken |= 1u << (gi >> 5);
      local_best(bv, bi);
    }
  }
  // sigmoid per rank in parallel; the sum runs in rank order, as in L5367-5372
  float wv = lane < k ? sigmoid_ref(my_v) : 0.f;
  float wsum = 0.f;
  for (int j = 0; j < k; ++j) wsum = wsum + __shfl_sync(0xffffffffu, wv, j);
  int bad = __any_sync(0xffffffffu, lane < k && my_i < 0);
  if (m.arch == 0 || m.weights_norm) {
    if (!(wsum > 0.f)) bad = 1;
    wv = wv / wsum;
  }
  if (m.arch == 1) wv = __fmul_rn(m.weight_scale, wv);
  if (lane < k) {
    w.sel[t * k + lane] = my_i;
    w.wts[t * k + lane] = wv;
  }
  if (lane == 0) {
    w.shw[t] = (m.arch == 0) ? sigmoid_ref(L[E]) : 1.0f;
    if (bad) atomicOr(w.status, 1);
  }
}

// Groups the (token, rank) entries by owned expert, stably.
__global__ void __launch_bounds__(256) route_kernel(MoeDevice m, MoeWork w, int T) {
  __shared__ int s_count[kMaxExperts];
  __shared__ int s_offset[kMaxExperts + 1];
  const int E = m.experts, k = m.top_k;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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

// ---------------------------------------------------------------- prep
// Per token: optional rms-norm (rms-norm-into, llambda.lisp L859-879:
// scale = 1/sqrt(mean(x^2) + eps), dest = (x * weight) * scale), then the
// router input (natural layout) and the prepared gate/up input (weight-type
// layout with sub-block sums, zero-padded from H to k_in).
template <int UT>
__global__ void __launch_bounds__(256) moe_prep_kernel(MoeDevice m, MoeWork w,
                                                       const float* __restrict__ x) {
  __shared__ float s_part[8];
  const int H = m.hidden, K = m.k_in, tasks = K >> 6;
  const float* xt = x + (long)blockIdx.x * H;
  float scale = 1.f;
  if (m.input_norm) {
    float acc = 0.f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) acc = fmaf(xt[i], xt[i], acc);
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = acc;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += s_part[i];
    const float ms = __fdiv_rn(tot, (float)H);
    scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, m.norm_epsilon)));
  }
  float* xn = w.xn + (long)blockIdx.x * H;
  float* xp = w.xp_up + (long)blockIdx.x * xp_stride(K);
  for (int base = 0; base < K; base += 4 * blockDim.x) {
    const int e = base + 4 * threadIdx.x;
    float v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int i = e + q;
      float val = 0.f;
      if (i < H) {
        val = xt[i];
        if (m.input_norm) {
          val = __fmul_rn(__fmul_rn(val, m.input_norm[i]), scale);
          xn[i] = val;
        }
      }
      v[q] = val;
    }
    if (e < K) {  // K is a multiple of 256, so whole warps agree here
      *reinterpret_cast<float4*>(xp + xp_index<UT>(e, tasks)) = make_float4(v[0], v[1], v[2], v[3]);
      if (UT == LB_TYPE_Q4_K) {
        float part = (v[0] + v[1]) + (v[2] + v[3]);
        part += __shfl_xor_sync(0xffffffffu, part, 1);
        part += __shfl_xor_sync(0xffffffffu, part, 2);
        part += __shfl_xor_sync(0xffffffffu, part, 4);
        if ((threadIdx.x & 7) == 0) xp[K + (e >> 5)] = part;
      }
    }
  }
}

// Routing metadata of the expert owning a run of units, cached per warp.
struct ExpertView {
  int a = -1;            // active-list index
  int e = -1;            // expert id
  int ntok = 0;          // tokens routed to it
  const int* list = nullptr;  // their entry ids
};

__device__ __forceinline__ void view_expert(const MoeDevice& m, const MoeWork& w, int T, int a,
                                            ExpertView& v) {
  if (v.a == a) return;
  v.a = a;
  v.e = w.active[a];
  v.ntok = w.counts[v.e];
  v.list = w.entries + T * m.top_k + w.offsets[v.e];
}

// ---------------------------------------------------------------- up
// gate/up rows (qwen3next: silu(gate) * up; nemotron: relu(up)^2) for all
// tokens of the unit, written straight into the down input's prepared
// layout of entry `id` (element = intermediate row).
template <int UT, int DT, int LPR, int RL, bool PAIR>
__global__ void __launch_bounds__(128) moe_up_kernel(MoeDevice m, MoeWork w, int T, int shared_pass,
                                                     int stages, int stage_bytes, int tchunk) {
  constexpr int RPP = 32 / LPR, RU = RL * RPP;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)nwarps * stages * stage_bytes);
  const WarpRing ring{smem + (size_t)warp * stages * stage_bytes, bars + warp * stages,
                      stage_bytes, stages};
  ring_init(ring, lane);
  const int k = m.top_k;
  const int rows_e = shared_pass ? m.inter_sh : m.inter;
  const int per = (rows_e + RU - 1) / RU;
  // shared-expert units are (token chunk, row block): all tokens meet it
  const int units = shared_pass ? (m.shared_here ? per * ((T + tchunk - 1) / tchunk) : 0)
                                : w.active[m.experts] * per;
  const int K = shared_pass ? m.k_in_sh : m.k_in;
  const int tasks = K >> 6;
  const int kd = shared_pass ? m.k_down_sh : m.k_down;
  const int tasks_d = kd >> 6;
  const long ld_up = xp_stride(m.k_in);
  const long ld_dn = xp_stride(max(m.k_down, m.k_down_sh));
  const size_t grb = shared_pass ? m.gate_sh_rb : m.gate_rb;
  const size_t urb = shared_pass ? m.up_sh_rb : m.up_rb;
  const int gw = blockIdx.x * nwarps + warp, total = gridDim.x * nwarps;
  const int chunk = (units + total - 1) / total;
  const int u0 = gw * chunk;
  const int n_my = max(0, min(units, u0 + chunk) - u0);

  ExpertView iv, cv;  // issuer's and consumer's cached expert
  auto sources = [&](int u, ExpertView& v, int& row0, const uint8_t*& g, const uint8_t*& up) {
    const int a = u / per;
    row0 = (u - a * per) * RU;
    if (shared_pass) {
      g = PAIR ? m.gate_sh + (size_t)row0 * grb : nullptr;
      up = m.up_sh + (size_t)row0 * urb;
    } else {
      view_expert(m, w, T, a, v);
      g = PAIR ? m.gate_exps + ((size_t)v.e * m.inter + row0) * grb : nullptr;
      up = m.up_exps + ((size_t)v.e * m.inter + row0) * urb;
    }
  };
  auto issue = [&](int idx) {
    int row0;
    const uint8_t *g, *up;
    sources(u0 + idx, iv, row0, g, up);
    const int nr = min(RU, rows_e - row0);
    if (PAIR)
      ring_issue(ring, idx % stages, g, (size_t)nr * grb, up, (size_t)nr * urb);
    else
      ring_issue(ring, idx % stages, up, (size_t)nr * urb, nullptr, 0);
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
    ok = __all_sync(0xffffffffu, mbar_wait(&ring.bars[i % stages], (i / stages) & 1, w.status));
    if (!ok) break;
    int row0;
    const uint8_t *g, *up;
    sources(u0 + i, cv, row0, g, up);
    const int nr = min(RU, rows_e - row0);
    uint8_t* st = ring.smem + (size_t)(i % stages) * stage_bytes;
    const uint8_t* grows = PAIR ? st + (reinterpret_cast<uintptr_t>(g) & 15) : nullptr;
    const uint8_t* urows =
        st + (PAIR ? widened(g, (size_t)nr * grb) : 0) + (reinterpret_cast<uintptr_t>(up) & 15);
    int t_begin = 0, t_end = cv.ntok;
    if (shared_pass) {
      t_begin = ((u0 + i) / per) * tchunk;
      t_end = min(T, t_begin + tchunk);
    }
    for (int t = t_begin; t < t_end; ++t) {
      const int id = shared_pass ? T * k + t : cv.list[t];  // routed entry id / shared slot
      const int tok = shared_pass ? t : id / k;
      float y0[RL], y1[RL];
      // PAIR: gate rows (matrix 0) and up rows (matrix 1) share the activations
      if (PAIR)
        unit_rows<UT, LPR, RL, true>(grows, (int)grb, urows, (int)urb, nr, tasks,
                                     w.xp_up + (long)tok * ld_up, tok, xc, lane, y0, y1);
      else
        unit_rows<UT, LPR, RL, false>(urows, (int)urb, nullptr, 0, nr, tasks,
                                      w.xp_up + (long)tok * ld_up, tok, xc, lane, y0, y1);
      float* hrow = w.xp_down + (long)id * ld_dn;
#pragma unroll
      for (int q = 0; q < RL; ++q) {
        const int r = grp + q * RPP;
        if (lt == q && r < nr) {
          const float hv = PAIR ? __fmul_rn(silu_ref(y0[q]), y1[q]) : relu_sq_ref(y0[q]);
          hrow[xp_index<DT>(row0 + r, tasks_d)] = hv;
        }
      }
      if (row0 + nr == rows_e)  // last block: zero the padding up to k_down
        for (int pe = rows_e + lane; pe < kd; pe += 32) hrow[xp_index<DT>(pe, tasks_d)] = 0.f;
    }
    __syncwarp();
  }
  if (!ok)
    for (int q = i + 1; q < issued; ++q) mbar_wait(&ring.bars[q % stages], (q / stages) & 1, nullptr);
}

// Q4_K down inputs need sub-block sums; Q6_K inputs do not.
__global__ void moe_down_sums_kernel(MoeDevice m, MoeWork w, int T) {
  const int k = m.top_k;
  const long ld_dn = xp_stride(max(m.k_down, m.k_down_sh));
  const int n_entries = T * k + T;
  for (int id = blockIdx.x; id < n_entries; id += gridDim.x) {
    const bool shared = id >= T * k;
    if (shared && !(m.shared_here && m.inter_sh)) continue;
    if (!shared) {
      const int e = w.sel[id];
      if (e < m.expert_begin || e >= m.expert_end) continue;
    }
    const int K = shared ? m.k_down_sh : m.k_down, tasks = K >> 6;
    float* xp = w.xp_down + (long)id * ld_dn;
    for (int g = threadIdx.x; g < K / 32; g += blockDim.x) {
      const int task = g >> 1, i0 = (g & 1) * 8;
      float s = 0.f;
      for (int i = 0; i < 8; ++i) {
        const float4 v = reinterpret_cast<const float4*>(xp)[(i0 + i) * tasks + task];
        s += (v.x + v.y) + (v.z + v.w);
      }
      xp[K + g] = s;
    }
  }
}

// ---------------------------------------------------------------- down
template <int DT, int LPR, int RL>
__global__ void __launch_bounds__(128) moe_down_kernel(MoeDevice m, MoeWork w, int T,
                                                       int shared_pass, int stages,
                                                       int stage_bytes, int tchunk) {
  constexpr int RPP = 32 / LPR, RU = RL * RPP;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)nwarps * stages * stage_bytes);
  const WarpRing ring{smem + (size_t)warp * stages * stage_bytes, bars + warp * stages,
                      stage_bytes, stages};
  ring_init(ring, lane);
  const int k = m.top_k, H = m.hidden;
  const int per = (H + RU - 1) / RU;
  const int units = shared_pass
                        ? ((m.shared_here && m.inter_sh) ? per * ((T + tchunk - 1) / tchunk) : 0)
                        : w.active[m.experts] * per;
  const int K = shared_pass ? m.k_down_sh : m.k_down;
  const int tasks = K >> 6;
  const long ld_dn = xp_stride(max(m.k_down, m.k_down_sh));
  const size_t rb = shared_pass ? m.down_sh_rb : m.down_rb;
  const int gw = blockIdx.x * nwarps + warp, total = gridDim.x * nwarps;
  const int chunk = (units + total - 1) / total;
  const int u0 = gw * chunk;
  const int n_my = max(0, min(units, u0 + chunk) - u0);
  ExpertView iv, cv;
  auto source = [&](int u, ExpertView& v, int& row0) -> const uint8_t* {
    const int a = u / per;
    row0 = (u - a * per) * RU;
    if (shared_pass) return m.down_sh + (size_t)row0 * rb;
    view_expert(m, w, T, a, v);
    return m.down_exps + ((size_t)v.e * H + row0) * rb;
  };
  auto issue = [&](int idx) {
    int row0;
    const uint8_t* src = source(u0 + idx, iv, row0);
    ring_issue(ring, idx % stages, src, (size_t)min(RU, H - row0) * rb, nullptr, 0);
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
    ok = __all_sync(0xffffffffu, mbar_wait(&ring.bars[i % stages], (i / stages) & 1, w.status));
    if (!ok) break;
    int row0;
    const uint8_t* src = source(u0 + i, cv, row0);
    const int nr = min(RU, H - row0);
    const uint8_t* rows =
        ring.smem + (size_t)(i % stages) * stage_bytes + (reinterpret_cast<uintptr_t>(src) & 15);
    int t_begin = 0, t_end = cv.ntok;
    if (shared_pass) {
      t_begin = ((u0 + i) / per) * tchunk;
      t_end = min(T, t_begin + tchunk);
    }
    for (int t = t_begin; t < t_end; ++t) {
      const int id = shared_pass ? T * k + t : cv.list[t];
      const int tok = shared_pass ? t : id / k;
      const int slot = shared_pass ? k : id - tok * k;
      float y0[RL], unused[RL];
      unit_rows<DT, LPR, RL, false>(rows, (int)rb, nullptr, 0, nr, tasks,
                                    w.xp_down + (long)id * ld_dn, id, xc, lane, y0, unused);
      float* out = w.partial + ((long)tok * (k + 1) + slot) * H + row0;
#pragma unroll
      for (int q = 0; q < RL; ++q) {
        const int r = grp + q * RPP;
        if (lt == q && r < nr) out[r] = y0[q];
      }
    }
    __syncwarp();
  }
  if (!ok)
    for (int q = i + 1; q < issued; ++q) mbar_wait(&ring.bars[q % stages], (q / stages) & 1, nullptr);
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

template <typename Kern>
cudaError_t launch_persistent(Kern kern, const UnitPlan& p, cudaStream_t s, MoeDevice m, MoeWork w,
                              int T, int shared_pass) {
  const size_t smem = (size_t)p.warps * p.stages * (p.stage_bytes + 8);
  const int occ = prepared_occupancy(kern, p.warps * 32, smem);
  if (occ < 0) return cudaErrorUnknown;
  // shared-expert passes: enough token chunks to give every warp a unit
  const int warps = sm_count() * std::max(occ, 1) * p.warps;
  const int tchunk = std::max(1, std::min(T, 4));
  (void)warps;
  kern<<<sm_count() * std::max(occ, 1), p.warps * 32, smem, s>>>(m, w, T, shared_pass, p.stages,
                                                                 p.stage_bytes, tchunk);
  return cudaGetLastError();
}

template <int UT, int DT>
cudaError_t launch_up(const MoeDevice& m, const MoeWork& w, int T, int shared_pass,
                      cudaStream_t s) {
  const size_t rb = shared_pass ? m.up_sh_rb : m.up_rb;
  const int K = shared_pass ? m.k_in_sh : m.k_in;
  const bool pair = m.arch == 0;
  const UnitPlan p = plan_units(rb, K / 64, pair ? 2 : 1);
#define LB_UP(L, RR)                                                                              \
  if (p.lpr == L && p.rl == RR)                                                                   \
    return pair ? launch_persistent(moe_up_kernel<UT, DT, L, RR, true>, p, s, m, w, T, shared_pass) \
                : launch_persistent(moe_up_kernel<UT, DT, L, RR, false>, p, s, m, w, T, shared_pass);
  LB_UP(8, 1) LB_UP(8, 2) LB_UP(8, 4) LB_UP(16, 1) LB_UP(16, 2) LB_UP(16, 4)
  LB_UP(32, 1) LB_UP(32, 2) LB_UP(32, 4)
#undef LB_UP
  return cudaErrorInvalidValue;
}

template <int DT>
cudaError_t launch_down(const MoeDevice& m, const MoeWork& w, int T, int shared_pass,
                        cudaStream_t s) {
  const size_t rb = shared_pass ? m.down_sh_rb : m.down_rb;
  const int K = shared_pass ? m.k_down_sh : m.k_down;
  const UnitPlan p = plan_units(rb, K / 64, 1);
#define LB_DN(L, RR) \
  if (p.lpr == L && p.rl == RR) return launch_persistent(moe_down_kernel<DT, L, RR>, p, s, m, w, T, shared_pass);
  LB_DN(8, 1) LB_DN(8, 2) LB_DN(8, 4) LB_DN(16, 1) LB_DN(16, 2) LB_DN(16, 4)
  LB_DN(32, 1) LB_DN(32, 2) LB_DN(32, 4)
#undef LB_DN
  return cudaErrorInvalidValue;
}

template <int UT, int DT>
cudaError_t launch_expert_passes(const MoeDevice& m, const MoeWork& w, int T, cudaStream_t s) {
  cudaError_t e = launch_up<UT, DT>(m, w, T, 0, s);
  if (e == cudaSuccess && m.shared_here && m.inter_sh) e = launch_up<UT, DT>(m, w, T, 1, s);
  if (e != cudaSuccess) return e;
  if (DT == LB_TYPE_Q4_K) {
    moe_down_sums_kernel<<<std::min(T * m.top_k + T, sm_count() * 4), 128, 0, s>>>(m, w, T);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  e = launch_down<DT>(m, w, T, 0, s);
  if (e == cudaSuccess && m.shared_here && m.inter_sh) e = launch_down<DT>(m, w, T, 1, s);
  return e;
}

}  // namespace

size_t moe_work_bytes(const MoeDevice& m, int T) {
  MoeWork w;
  moe_work_carve(m, T, nullptr, &w);
  return w.bytes;
}

void moe_work_carve(const MoeDevice& m, int T, void* base, MoeWork* w) {
  const int E = m.experts, k = m.top_k;
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
  w->xn = reinterpret_cast<float*>(take(m.input_norm ? (size_t)T * m.hidden * 4 : 4));
  w->xp_up = reinterpret_cast<float*>(take((size_t)T * xp_stride(m.k_in) * 4));
  w->xp_down = reinterpret_cast<float*>(
      take((size_t)(T * k + T) * xp_stride(std::max(m.k_down, m.k_down_sh)) * 4));
  w->partial = reinterpret_cast<float*>(take((size_t)T * (k + 1) * m.hidden * 4));
  w->bytes = off;
}

cudaError_t launch_moe(const MoeDevice& m, const MoeWork& w, const float* x, int T, float* out,
                       cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  if (T > w.max_tokens || m.experts > kMaxExperts || m.top_k > 32 || T * m.top_k > 4 * 1024)
    return cudaErrorInvalidValue;
  if (m.inter_sh && m.k_in_sh != m.k_in) return cudaErrorInvalidValue;
  const int E = m.experts;
  const int router_rows = E + (m.arch == 0 && !m.router_extra_row ? 1 : 0);
  cudaError_t e;
  if (m.up_type == LB_TYPE_Q4_K)
    moe_prep_kernel<LB_TYPE_Q4_K><<<T, 256, 0, s>>>(m, w, x);
  else
    moe_prep_kernel<LB_TYPE_Q6_K><<<T, 256, 0, s>>>(m, w, x);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  const float* xr = m.input_norm ? w.xn : x;
  if (m.arch == 0 && m.router_extra_row) {  // shared-expert gate logit into column E
    e = launch_gemv_f32(m.router_extra_row, 1, m.hidden, xr, m.hidden, T, w.logits + E, E + 1, s);
    if (e != cudaSuccess) return e;
  }
  e = launch_gemv_f32(m.router, router_rows, m.hidden, xr, m.hidden, T, w.logits, E + 1, s);
  if (e != cudaSuccess) return e;
  topk_kernel<<<T, 32, 0, s>>>(m, w, T);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  route_kernel<<<1, 256, 0, s>>>(m, w, T);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  const bool gate_ok = m.arch == 1 || m.gate_type == m.up_type;
  if (!gate_ok) return cudaErrorInvalidValue;
  if (m.up_type == LB_TYPE_Q4_K && m.down_type == LB_TYPE_Q6_K)
    e = launch_expert_passes<LB_TYPE_Q4_K, LB_TYPE_Q6_K>(m, w, T, s);
  else if (m.up_type == LB_TYPE_Q4_K && m.down_type == LB_TYPE_Q4_K)
    e = launch_expert_passes<LB_TYPE_Q4_K, LB_TYPE_Q4_K>(m, w, T, s);
  else if (m.up_type == LB_TYPE_Q6_K && m.down_type == LB_TYPE_Q6_K)
    e = launch_expert_passes<LB_TYPE_Q6_K, LB_TYPE_Q6_K>(m, w, T, s);
  else if (m.up_type == LB_TYPE_Q6_K && m.down_type == LB_TYPE_Q4_K)
    e = launch_expert_passes<LB_TYPE_Q6_K, LB_TYPE_Q4_K>(m, w, T, s);
  else
    return cudaErrorInvalidValue;
  if (e != cudaSuccess) return e;
  const long n = (long)T * m.hidden;
  const int grid = (int)std::min<long>((n + 255) / 256, (long)sm_count() * 8);
  combine_kernel<<<std::max(grid, 1), 256, 0, s>>>(m, w, T, x, out);
  return cudaGetLastError();
}

}  // namespace lb
