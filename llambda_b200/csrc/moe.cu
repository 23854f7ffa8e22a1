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
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "engine.cuh"
#include "kernels.h"
#include "mma.cuh"

namespace lb {

namespace {

constexpr int kMaxExperts = 1024;
constexpr int kSlabMaxStages = 10;

// Floats per token of the prepared gate/up input: room for either layout
// (Q4_K: the tensor-core layout of mma.cuh; Q6_K: the warp engine's).
__host__ __device__ __forceinline__ long up_ld_floats(int K) {
  const long a = xp_stride(K), b = (long)(mx_bytes(K) / 4);
  return a > b ? a : b;
}

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
// pass_nt: tokens per pass of the up kernel; pass_off counts passes.
__global__ void __launch_bounds__(256) route_kernel(MoeDevice m, MoeWork w, int T, int pass_nt) {
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
    // exclusive scans over experts (entries and token passes), active list in
    // increasing expert id
    int run = 0, nact = 0, prun = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const int cnt = e < E ? s_count[e] : 0;
      const int pc = (cnt + pass_nt - 1) / pass_nt;
      int incl = cnt, pincl = pc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        const int pv = __shfl_up_sync(0xffffffffu, pincl, o);
        if (lane >= o) {
          incl += v;
          pincl += pv;
        }
      }
      if (e < E) s_offset[e] = run + incl - cnt;
      const unsigned nz = __ballot_sync(0xffffffffu, cnt > 0);
      if (cnt > 0) {
        const int a = nact + __popc(nz & lt_mask);
        w.active[a] = e;
        w.pass_off[a] = prun + pincl - pc;
      }
      nact += __popc(nz);
      run += __shfl_sync(0xffffffffu, incl, 31);
      prun += __shfl_sync(0xffffffffu, pincl, 31);
    }
    if (lane == 0) {
      s_offset[E] = run;
      w.active[E] = nact;
      w.pass_off[nact] = prun;
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
  float* xp = w.xp_up + (long)blockIdx.x * up_ld_floats(K);
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
      if (UT == LB_TYPE_Q4_K)  // tensor-core layout (mma.cuh)
        mx_store4(reinterpret_cast<uint8_t*>(xp), K, e, make_float4(v[0], v[1], v[2], v[3]));
      else
        *reinterpret_cast<float4*>(xp + xp_index<UT>(e, tasks)) =
            make_float4(v[0], v[1], v[2], v[3]);
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
  const long ld_up = up_ld_floats(m.k_in);
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

// ---------------------------------------------------------------- up (slabs)
// Q4_K gate/up rows on the tensor cores, K-sliced: a unit is a slab of RU
// rows of each matrix (gate and up: RU = 16 * CW / 2; up only: 16 * CW) of
// one routed expert, or of the shared expert for a chunk of tokens.  Consumer
// warp w owns row block w (16 rows of one matrix) across the whole K, so its
// sums stay in registers; a pipeline stage is one super-block column slice of
// the slab: CW boxes of 16 rows x 144 bytes, loaded by 2-D tensor copies
// (rows 144 bytes apart in shared memory: the 8 row groups of a fragment load
// fall in different bank groups).  Warp CW is the producer: it waits until
// all consumer warps released a stage (empty barrier) before refilling it.
// With gate and up, the up warps hand their row sums to the gate warps once
// per slab through a double-buffered exchange guarded by two more barriers.
// Every wait is bounded; a timeout raises a CTA-wide abort flag.
struct SlabSync {
  uint64_t full[kSlabMaxStages];
  uint64_t empty[kSlabMaxStages];
  uint64_t xfull[2];
  uint64_t xempty[2];
  int abort;
  int pad[3];
};

template <int NT, bool PAIR, int DT, int CW>
__global__ void __launch_bounds__((CW + 1) * 32, 1)
    moe_up_slab_kernel(MoeDevice m, MoeWork w, int T, int stages, long map_row_base,
                       const __grid_constant__ CUtensorMap tm_gate,
                       const __grid_constant__ CUtensorMap tm_up,
                       const __grid_constant__ CUtensorMap tm_gate_sh,
                       const __grid_constant__ CUtensorMap tm_up_sh) {
  constexpr int MATS = PAIR ? 2 : 1;
  constexpr int RBM = CW / MATS;       // row blocks per matrix
  constexpr int RU = RBM * kTileRows;  // rows per matrix per slab
  constexpr int BOX = kTileRows * LB_Q4K;
  constexpr int STAGE = CW * BOX;
  extern __shared__ __align__(128) uint8_t smem[];
  SlabSync* sync = reinterpret_cast<SlabSync*>(smem + (size_t)stages * STAGE);
  float* xch = reinterpret_cast<float*>(sync + 1);  // [2][RU][NT] up-row sums
  volatile int* abort = &sync->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&sync->full[s], 1);
      mbar_init(&sync->empty[s], CW);
    }
    for (int p = 0; p < 2; ++p) {
      mbar_init(&sync->xfull[p], RBM);
      mbar_init(&sync->xempty[p], RBM);
    }
    sync->abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const int k = m.top_k;
  const int per_r = (m.inter + RU - 1) / RU;
  const int per_s = (m.inter_sh + RU - 1) / RU;
  const int passes_s = (T + NT - 1) / NT;
  const int nact = w.active[m.experts];
  // work items: (slab, pass of up to NT tokens), all of one cost; routed ones
  // expert-major (passes of expert a: pass_off[a] ..), then slab, then pass
  const int n_routed = w.pass_off[nact] * per_r;
  const int n_shared = (m.shared_here && m.inter_sh) ? per_s * passes_s : 0;
  const int units = n_routed + n_shared;
  const int u0 = (int)((long)blockIdx.x * units / gridDim.x);
  const int n_my = (int)((long)(blockIdx.x + 1) * units / gridDim.x) - u0;
  const int nsb = m.k_in >> 8;

  struct Unit {
    int row0, rows_e, t_begin, t_end;
    long map_row;  // row of the slab's first row in its tensor map
    bool shared;
  };
  ExpertView view;
  int a_hint = 0;  // active index of the previous item (items are visited in order)
  auto unit_at = [&](int u) {
    Unit x;
    if (u < n_routed) {
      int a = a_hint;  // first a with pass_off[a + 1] * per_r > u, searched from the hint
      if (w.pass_off[a] * per_r > u) a = 0;
      int hi = nact;
      while (hi - a > 1) {
        const int mid = (a + hi) >> 1;
        if (w.pass_off[mid] * per_r <= u) a = mid; else hi = mid;
      }
      a_hint = a;
      view_expert(m, w, T, a, view);
      const int np = w.pass_off[a + 1] - w.pass_off[a];
      const int local = u - w.pass_off[a] * per_r, slab = local / np, p = local - slab * np;
      x.shared = false;
      x.rows_e = m.inter;
      x.row0 = slab * RU;
      x.t_begin = p * NT;
      x.t_end = min(view.ntok, x.t_begin + NT);
      x.map_row = (long)view.e * m.inter - map_row_base + x.row0;
    } else {
      const int q = u - n_routed, slab = q / passes_s, p = q - slab * passes_s;
      x.shared = true;
      x.rows_e = m.inter_sh;
      x.row0 = slab * RU;
      x.t_begin = p * NT;
      x.t_end = min(T, x.t_begin + NT);
      x.map_row = x.row0;
    }
    return x;
  };

  if (warp == CW) {  // ---------------- producer
    if (lane == 0) {
      int q = 0;
      bool ok = true;
      for (int i = 0; i < n_my && ok; ++i) {
        const Unit x = unit_at(u0 + i);
        for (int t0 = x.t_begin; t0 < x.t_end && ok; t0 += NT) {
          for (int sb = 0; sb < nsb; ++sb, ++q) {
            const int s = q % stages;
            if (q >= stages &&
                !mbar_wait_or_abort(&sync->empty[s], ((q / stages) - 1) & 1, w.status, abort)) {
              ok = false;
              break;
            }
            mbar_expect_tx(&sync->full[s], STAGE);
            uint8_t* st = smem + (size_t)s * STAGE;
#pragma unroll
            for (int b = 0; b < CW; ++b) {
              const bool gate = PAIR && b < RBM;
              const CUtensorMap* tm = x.shared ? (gate ? &tm_gate_sh : &tm_up_sh)
                                               : (gate ? &tm_gate : &tm_up);
              tma_load_2d(st + b * BOX, tm, sb * LB_Q4K, (int)(x.map_row + (b % RBM) * kTileRows),
                          &sync->full[s]);
            }
          }
        }
      }
      // every copy issued must land before the CTA may exit
      for (int r = max(0, q - stages); r < q; ++r)
        mbar_wait(&sync->full[r % stages], (r / stages) & 1, nullptr);
    }
    return;
  }

  // ---------------- consumers
  const int mat = warp / RBM, rb = warp % RBM;
  const int g = lane >> 2, t = lane & 3;
  const long ld_up = up_ld_floats(m.k_in);
  const long ld_dn = xp_stride(max(m.k_down, m.k_down_sh));
  int q = 0, pass = 0;
  bool ok = true;
  for (int i = 0; i < n_my && ok; ++i) {
    const Unit x = unit_at(u0 + i);
    const int kd = x.shared ? m.k_down_sh : m.k_down, tasks_d = kd >> 6;
    for (int t0 = x.t_begin; t0 < x.t_end && ok; t0 += NT, ++pass) {
      const int nt = min(NT, x.t_end - t0);
      int ids[NT];
      const uint8_t* mxp[NT];
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const int tt = min(t0 + n, x.t_end - 1);
        ids[n] = x.shared ? T * k + tt : view.list[tt];
        const int tok = x.shared ? tt : ids[n] / k;
        mxp[n] = reinterpret_cast<const uint8_t*>(w.xp_up + tok * ld_up);
      }
      float2 acc[2][NT];
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int n = 0; n < NT; ++n) acc[r][n] = make_float2(0.f, 0.f);
      for (int sb = 0; sb < nsb; ++sb, ++q) {
        const int s = q % stages;
        if (!mbar_wait_or_abort(&sync->full[s], (q / stages) & 1, w.status, abort)) {
          ok = false;
          break;
        }
        const uint8_t* blk = smem + (size_t)s * STAGE + warp * BOX;
        q4k_sb_mma<NT>(blk + g * LB_Q4K, blk + (g + 8) * LB_Q4K, sb, mxp, nt, nsb, lane, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(&sync->empty[s]);
      }
      if (!ok) break;
      // row sums of rows g and g+8 of this block on lane t == 0 of each quad
      float v[2][NT];
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          float s = acc[r][n].x + acc[r][n].y;
          s += __shfl_xor_sync(0xffffffffu, s, 1);
          s += __shfl_xor_sync(0xffffffffu, s, 2);
          v[r][n] = s;
        }
      const int par = pass & 1, use = pass >> 1;
      float* xb = xch + (size_t)par * RU * NT;
      auto store_h = [&](float up_or_h, int r, int n, bool gated, float gate) {
        const int row = x.row0 + rb * kTileRows + g + 8 * r;
        if (row < x.rows_e && n < nt) {
          const float hv = gated ? __fmul_rn(silu_ref(gate), up_or_h) : relu_sq_ref(up_or_h);
          int id = ids[0];
#pragma unroll
          for (int n2 = 1; n2 < NT; ++n2)
            if (n2 == n) id = ids[n2];
          w.xp_down[(long)id * ld_dn + xp_index<DT>(row, tasks_d)] = hv;
        }
      };
      if (PAIR && mat == 1) {  // up warps: hand the sums to the gate warps
        if (use > 0 && !mbar_wait_or_abort(&sync->xempty[par], (use - 1) & 1, w.status, abort)) {
          ok = false;
          break;
        }
        if (t == 0)
#pragma unroll
          for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int n = 0; n < NT; ++n) xb[(rb * kTileRows + g + 8 * r) * NT + n] = v[r][n];
        __syncwarp();
        if (lane == 0) mbar_arrive(&sync->xfull[par]);
      } else if (PAIR) {  // gate warps: silu(gate) * up
        if (!mbar_wait_or_abort(&sync->xfull[par], use & 1, w.status, abort)) {
          ok = false;
          break;
        }
        if (t == 0)
#pragma unroll
          for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int n = 0; n < NT; ++n)
              store_h(xb[(rb * kTileRows + g + 8 * r) * NT + n], r, n, true, v[r][n]);
        __syncwarp();
        if (lane == 0) mbar_arrive(&sync->xempty[par]);
      } else if (t == 0) {  // up only: relu(up)^2
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
          for (int n = 0; n < NT; ++n) store_h(v[r][n], r, n, false, 0.f);
      }
      if (warp == 0 && x.row0 + RU >= x.rows_e) {  // last slab: zero the padding up to kd
        const int pad = kd - x.rows_e;
        for (int qq = lane; qq < nt * pad; qq += 32) {
          const int nn = qq / pad, pe = x.rows_e + (qq - nn * pad);
          int id = ids[0];
#pragma unroll
          for (int n2 = 1; n2 < NT; ++n2)
            if (n2 == nn) id = ids[n2];
          w.xp_down[(long)id * ld_dn + xp_index<DT>(pe, tasks_d)] = 0.f;
        }
      }
    }
  }
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

// 2-D tensor map over `rows` Q4_K rows of `rb` bytes at `base`; one box is
// one super-block (144 bytes) of 16 rows.
bool q4k_rows_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t rb) {
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
  if (!encode || rows == 0) return false;
  const cuuint64_t dims[2] = {rb, rows};
  const cuuint64_t strides[1] = {rb};
  const cuuint32_t box[2] = {LB_Q4K, kTileRows};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct SlabMaps {
  CUtensorMap gate, up, gate_sh, up_sh;
  long row_base;  // global row (expert_begin * inter) of the routed maps' row 0
};

template <int NT, bool PAIR, int DT, int CW>
cudaError_t launch_up_slab_nt(const MoeDevice& m, const MoeWork& w, int T, const SlabMaps& mp,
                              cudaStream_t s) {
  auto kern = moe_up_slab_kernel<NT, PAIR, DT, CW>;
  constexpr int RU = CW / (PAIR ? 2 : 1) * kTileRows;
  const size_t stage = (size_t)CW * kTileRows * LB_Q4K;
  const size_t extra = sizeof(SlabSync) + (size_t)2 * RU * NT * 4;
  const int stages = (int)std::min<size_t>(kSlabMaxStages, (kTileSmemBudget - extra) / stage);
  if (stages < 2) return cudaErrorInvalidValue;
  const size_t smem = (size_t)stages * stage + extra;
  if (prepared_occupancy(kern, (CW + 1) * 32, smem) < 1) return cudaErrorUnknown;
  kern<<<sm_count(), (CW + 1) * 32, smem, s>>>(m, w, T, stages, mp.row_base, mp.gate,
                                                mp.up, mp.gate_sh, mp.up_sh);
  return cudaGetLastError();
}

// Tokens per pass (NT) of the tensor-core gate/up launch, from the expected
// tokens per active expert; the route kernel counts passes with the same NT.
int up_pass_tokens(const MoeDevice& m, int T) {
  if (m.up_type != LB_TYPE_Q4_K || T == 1) return 1;
  const long entries = (long)T * m.top_k;
  const long owned = std::max(1, m.expert_end - m.expert_begin);
  const double per_expert = (double)entries / (double)std::min(entries, owned);
  return per_expert < 2.5 ? 2 : 4;
}

// Routed and shared gate/up in one tensor-core launch.
template <int DT>
cudaError_t launch_up_mma(const MoeDevice& m, const MoeWork& w, int T, cudaStream_t s) {
  const bool pair = m.arch == 0;
  SlabMaps mp;
  mp.row_base = (long)m.expert_begin * m.inter;
  const uint64_t owned_rows = (uint64_t)std::max(0, m.expert_end - m.expert_begin) * m.inter;
  const bool shared = m.shared_here && m.inter_sh;
  if (shared) {
    if (!q4k_rows_map(&mp.up_sh, m.up_sh, m.inter_sh, m.up_sh_rb)) return cudaErrorInvalidValue;
    mp.gate_sh = mp.up_sh;
    if (pair && !q4k_rows_map(&mp.gate_sh, m.gate_sh, m.inter_sh, m.gate_sh_rb))
      return cudaErrorInvalidValue;
  }
  if (owned_rows) {
    const uint8_t* up0 = m.up_exps + (size_t)mp.row_base * m.up_rb;
    if (!q4k_rows_map(&mp.up, up0, owned_rows, m.up_rb)) return cudaErrorInvalidValue;
    mp.gate = mp.up;
    if (pair && !q4k_rows_map(&mp.gate, m.gate_exps + (size_t)mp.row_base * m.gate_rb,
                              owned_rows, m.gate_rb))
      return cudaErrorInvalidValue;
  } else if (shared) {  // no routed rows here: the routed maps are never used
    mp.up = mp.up_sh;
    mp.gate = mp.gate_sh;
  } else {
    return cudaSuccess;
  }
  if (!shared) {
    mp.up_sh = mp.up;
    mp.gate_sh = mp.gate;
  }
  switch (up_pass_tokens(m, T)) {
    case 1:
      return pair ? launch_up_slab_nt<1, true, DT, 8>(m, w, T, mp, s)
                  : launch_up_slab_nt<1, false, DT, 8>(m, w, T, mp, s);
    case 2:
      return pair ? launch_up_slab_nt<2, true, DT, 8>(m, w, T, mp, s)
                  : launch_up_slab_nt<2, false, DT, 8>(m, w, T, mp, s);
    default:
      return pair ? launch_up_slab_nt<4, true, DT, 8>(m, w, T, mp, s)
                  : launch_up_slab_nt<4, false, DT, 8>(m, w, T, mp, s);
  }
}

template <int UT, int DT>
cudaError_t launch_expert_passes(const MoeDevice& m, const MoeWork& w, int T, cudaStream_t s) {
  cudaError_t e;
  if constexpr (UT == LB_TYPE_Q4_K) {
    e = launch_up_mma<DT>(m, w, T, s);
  } else {
    e = launch_up<UT, DT>(m, w, T, 0, s);
    if (e == cudaSuccess && m.shared_here && m.inter_sh) e = launch_up<UT, DT>(m, w, T, 1, s);
  }
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
  w->pass_off = reinterpret_cast<int*>(take((size_t)(E + 1) * 4));
  w->status = reinterpret_cast<int*>(take(4));
  w->xn = reinterpret_cast<float*>(take(m.input_norm ? (size_t)T * m.hidden * 4 : 4));
  w->xp_up = reinterpret_cast<float*>(take((size_t)T * up_ld_floats(m.k_in) * 4));
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
  route_kernel<<<1, 256, 0, s>>>(m, w, T, up_pass_tokens(m, T));
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
