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
#include <cmath>
#include <mutex>

#include "engine.cuh"
#include "kernels.h"
#include "mma.cuh"

namespace lb {

namespace {

constexpr int kMaxExperts = 1024;
// (token, rank) entries of one layer call (prefill batches included)
constexpr int kMaxEntries = 64 * 1024;
// The routing CTA splits the grouping of entries over its warps from
// 8 * kRouteSplitChunks chunks of 32 entries on (decode batch 32 and up:
// the grouping walk of its 320 entries took 4.0 us on one warp, 2.0 split;
// at 80 entries the split's extra zeroing and fix-up cost more than they
// save), with per-warp expert counters in kRouteSplitSlots ints of shared
// memory.
constexpr int kRouteSplitChunks = 1;
constexpr int kTopkTokens = 8;  // tokens per CTA of the top-k launch (one per warp)
constexpr int kRouteSplitSlots = 8192;
constexpr int kSlabMaxStages = 10;
// Gate/up work items split over K: when a call has fewer (slab, pass) items
// than CTAs (decode batches of a token or two), each item's super-block
// columns are split over up to kUpMaxSplit CTAs and the last to finish sums
// the slices in slice order.  Buffers cover kUpSplitItems items.
constexpr int kUpMaxSplit = 4, kUpSplitItems = 160;
constexpr int kUpPartFloats = 32 * kTileRows;  // consumer warps x tokens per pass <= 32

__device__ __forceinline__ int up_split(int units, int grid, int nsb) {
  if (units <= 0 || units > kUpSplitItems) return 1;
  return max(1, min(min(kUpMaxSplit, nsb), grid / units));
}
// Rows of one 2-D tensor copy of the gate/up slabs (the slabs' rows per
// matrix are multiples of it).
constexpr int kUpBoxRows = 64;

// Bytes of one gate/up slab stage: CW boxes of 16 Q4_K rows x one super-block
// and NT tokens' activation slices (1024 fragment + 64 meta bytes each).
__host__ __device__ constexpr int up_stage_bytes(int cw, int nt) {
  return (cw * 16 * 144 + nt * 1088 + 127) & ~127;
}

// Floats per token of the prepared gate/up input: room for either layout
// (Q4_K: the tensor-core layout of mma.cuh; Q6_K: the warp engine's).
__host__ __device__ __forceinline__ long up_ld_floats(int K) {
  const long a = xp_stride(K), b = (long)(mx_bytes(K) / 4);
  return a > b ? a : b;
}

// Floats per entry of the prepared down input: room for the warp engine's
// layout and for the Q6_K tensor-core layout (i6, mma.cuh).
__host__ __device__ __forceinline__ long down_ld_floats(const MoeDevice& m) {
  const int K = m.k_down > m.k_down_sh ? m.k_down : m.k_down_sh;
  const long a = xp_stride(K), b = (long)(i6_bytes(K) / 4);
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
// Sortable key of a score: a larger float has a larger key.  0 marks what the
// reference's strict > against most-negative-single-float never selects
// (NaN, -inf, -most-positive); -0.0 and +0.0 compare equal there, so they
// share a key.
__device__ __forceinline__ uint32_t topk_key(float v) {
  if (!(v > -3.40282347e38f)) return 0u;
  const uint32_t u = __float_as_uint(v == 0.f ? 0.f : v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Inverse of topk_key for a selectable key (-0.0 comes back as +0.0, which
// every later use treats alike).
__device__ __forceinline__ float topk_value(uint32_t key) {
  return __uint_as_float((key & 0x80000000u) ? (key & 0x7FFFFFFFu) : ~key);
}

// The k best scores of one token, in the order the reference's repeated
// strict-> scan finds them (descending score, ties to the lower index), by k
// rounds of a warp-wide arg-max: every lane keeps the best of its own PER
// candidates (the lowest index among equal keys), a round's winner is the
// highest key (one warp max) held by one lane (a ballot; several lanes only
// on exactly equal scores, where a warp min picks the lowest index), and
// only the winning lane re-derives its best, by a tree over its candidates.
// PER: candidates per lane (E <= 32*PER); key 0 marks a score that is never
// selected (NaN, -inf, -FLT_MAX and below).  One warp per token t.
template <int PER>
__device__ __forceinline__ void topk_token(const MoeDevice& m, const MoeWork& w, int t,
                                           int lane, int* s_sel = nullptr) {
  const int E = m.experts, k = m.top_k;
  const float* L = w.logits + (long)t * (E + 1);
  // Every load goes out before any is used: addresses are clamped into the
  // row (E + 1 entries) rather than guarded, as a guarded load per candidate
  // would wait for the one before it.
  float lv[PER];
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    const float* p = L + min(lane + 32 * q, E);
    lv[q] = __ldg(p);
  }
  const float gate_logit = __ldg(L + E);
  if (m.router_bias) {
    float bs[PER];
#pragma unroll
    for (int q = 0; q < PER; ++q) bs[q] = __ldg(m.router_bias + min(lane + 32 * q, E - 1));
#pragma unroll
    for (int q = 0; q < PER; ++q) lv[q] = lv[q] + bs[q];
  }
  uint32_t key[PER];
#pragma unroll
  for (int q = 0; q < PER; ++q) key[q] = lane + 32 * q < E ? topk_key(lv[q]) : 0u;
  // this lane's best key and its slot, by a tree whose left halves hold the
  // lower slots (a strict > keeps the lower slot on equal keys)
  uint32_t bk = 0u;
  int bq = 0;
  auto best = [&]() {
    uint32_t kk[PER];
    int qq[PER];
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      kk[q] = key[q];
      qq[q] = q;
    }
#pragma unroll
    for (int h = 1; h < PER; h <<= 1)
#pragma unroll
      for (int q = 0; q < PER; q += 2 * h) {
        const bool take = kk[q + h] > kk[q];
        kk[q] = take ? kk[q + h] : kk[q];
        qq[q] = take ? qq[q + h] : qq[q];
      }
    bk = kk[0];
    bq = qq[0];
  };
  best();
  // round r: the highest key, and among lanes holding it the lowest index;
  // lane r keeps the round's expert and key (-1: fewer than k selectable)
  int my_i = -1;
  uint32_t my_k = 0u;
  for (int r = 0; r < k; ++r) {
    const uint32_t mk = __reduce_max_sync(0xffffffffu, bk);
    if (mk == 0u) break;  // uniform: no selectable score left
    const unsigned holders = __ballot_sync(0xffffffffu, bk == mk);
    int wl = __ffs(holders) - 1;
    if (holders & (holders - 1u))  // equal keys on several lanes (rare)
      wl = (int)(__reduce_min_sync(0xffffffffu,
                                   bk == mk ? (uint32_t)(lane + 32 * bq) : 0xffffffffu) & 31u);
    const int wq = __shfl_sync(0xffffffffu, bq, wl);
    if (lane == r) {
      my_i = wl + 32 * wq;
      my_k = mk;
    }
    if (lane == wl) {
#pragma unroll
      for (int q = 0; q < PER; ++q)
        if (q == bq) key[q] = 0u;
      best();
    }
  }
  // sigmoid per rank in parallel; the sum runs in rank order, as in L5367-5372.
  // Lane k (when k < 32) evaluates the shared-expert gate's sigmoid in the
  // same pass, so the token's chain holds one sigmoid instead of two.
  const bool rank_lane = lane < k && my_i >= 0;
  const float sig = sigmoid_ref(rank_lane ? topk_value(my_k) : gate_logit);
  const float gate_sig = __shfl_sync(0xffffffffu, sig, k < 32 ? k : 0);
  float wv = rank_lane ? sig : 0.f;
  float wsum = 0.f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float o = __shfl_sync(0xffffffffu, wv, j);
    if (j < k) wsum = wsum + o;
  }
  int bad = __any_sync(0xffffffffu, lane < k && my_i < 0);
  if (m.arch == 0 || m.weights_norm) {
    if (!(wsum > 0.f)) bad = 1;
    wv = wv / wsum;
  }
  if (m.arch == 1) wv = __fmul_rn(m.weight_scale, wv);
  if (lane < k) {
    w.sel[t * k + lane] = my_i;
    w.wts[t * k + lane] = wv;
    if (s_sel) s_sel[t * k + lane] = my_i;
  }
  if (lane == 0) {
    w.shw[t] = (m.arch == 0) ? (k < 32 ? gate_sig : sigmoid_ref(gate_logit)) : 1.0f;
    if (bad) atomicOr(w.status, 1);
  }
}

// Where route_block reads the selections: written by an earlier launch
// (read-only path), by other CTAs of the same launch (L2), or copied into
// shared memory by this CTA.
enum SelSrc { kSelEarlier = 0, kSelSameLaunch = 1, kSelShared = 2 };

template <int SRC>
__device__ __forceinline__ int sel_at(const MoeWork& w, const int* s_sel, int id) {
  if (SRC == kSelShared) return s_sel[id];
  if (SRC == kSelSameLaunch) return __ldcg(w.sel + id);
  return __ldg(w.sel + id);
}

// Declared here, defined with the routing below.
template <int SRC>
__device__ __forceinline__ void route_block(const MoeDevice& m, const MoeWork& w, int T,
                                            int pass_nt, int pass_dn, bool grouped_ids,
                                            const int* s_sel = nullptr);

// Top-k (one warp per token, kTopkTokens tokens per CTA) with the routing on
// the last CTA to finish (an arrival counter; its eight warps group the
// entries), so the grouping needs no launch of its own.  The counter is zero
// between launches: the last CTA resets it.
template <int PER>
__global__ void __launch_bounds__(256) topk_route_kernel(MoeDevice m, MoeWork w, int T,
                                                         int pass_nt, int pass_dn,
                                                         int grouped_ids) {
  __shared__ int s_last;
  griddep_wait();
  griddep_launch();
  {
    const int t = blockIdx.x * kTopkTokens + (threadIdx.x >> 5);
    if (t < T) topk_token<PER>(m, w, t, threadIdx.x & 31);
  }
  if (grouped_ids < 0) return;  // the caller groups the entries (token dispatch)
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(w.tickets, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();  // every CTA's selections are visible from here
  route_block<kSelSameLaunch>(m, w, T, pass_nt, pass_dn, grouped_ids != 0);
  if (threadIdx.x == 0) *w.tickets = 0;
  // the gate/up items' arrival tickets start at zero even after a launch
  // that gave up part-way (each is reset by its last arriver otherwise)
  if (w.up_tickets)
    for (int i = threadIdx.x; i < kUpSplitItems; i += blockDim.x) w.up_tickets[i] = 0;
}

// The grouping of route_block for at most 32 entries (decode batches of a
// token or three), by one warp with lane i on entry i: match_any gives each
// entry its expert's group, its position (entries of the group on lower
// lanes: the order stays stable) and the group's size; each group's leader
// (its lowest lane) finds its place among the groups in increasing expert
// id, and the entry, up-pass and down-pass offsets before it, by one pass
// over the leaders.  Only the active experts' counts and offsets are
// written: the decode passes read no others (every launch of the dense form
// writes them all).  This replaces a scan over every expert (1.5 us of the
// 3.1 us routing at one token and 512 experts).
__device__ __forceinline__ void route_sparse_warp(const MoeDevice& m, const MoeWork& w, int T,
                                                  int pass_nt, int pass_dn, bool grouped_ids,
                                                  const int* s_sel, int lane) {
  const int n = T * m.top_k;
  const int e = lane < n ? s_sel[lane] : -1;
  const bool own = e >= m.expert_begin && e < m.expert_end;
  const unsigned owners = __ballot_sync(0xffffffffu, own);
  const unsigned grp = __match_any_sync(0xffffffffu, own ? e : -1) & owners;
  const unsigned lt_mask = (1u << lane) - 1u;
  const int pos = __popc(grp & lt_mask), cnt = __popc(grp);
  const bool leader = own && pos == 0;
  const unsigned leaders = __ballot_sync(0xffffffffu, leader);
  // this leader's place among the groups and the offsets before it
  int a = 0, off = 0, poff = 0, doff = 0;
  for (unsigned rest = leaders; rest; rest &= rest - 1u) {
    const int j = __ffs(rest) - 1;
    const int ej = __shfl_sync(0xffffffffu, e, j), cj = __shfl_sync(0xffffffffu, cnt, j);
    if (ej < e) {
      ++a;
      off += cj;
      poff += (cj + pass_nt - 1) / pass_nt;
      doff += (cj + pass_dn - 1) / pass_dn;
    }
  }
  const int nact = __popc(leaders), n_own = __popc(owners);
  if (leader) {
    w.active[a] = e;
    w.pass_off[a] = poff;
    w.pass_off_dn[a] = doff;
    w.counts[e] = cnt;
    w.offsets[e] = off;
  }
  // the totals: the last group's offsets plus its own passes
  int tp = leader ? poff + (cnt + pass_nt - 1) / pass_nt : 0;
  int td = leader ? doff + (cnt + pass_dn - 1) / pass_dn : 0;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    tp = max(tp, __shfl_xor_sync(0xffffffffu, tp, o));
    td = max(td, __shfl_xor_sync(0xffffffffu, td, o));
  }
  if (lane == 0) {
    w.active[m.experts] = nact;
    w.pass_off[nact] = tp;
    w.pass_off_dn[nact] = td;
    w.offsets[m.experts] = n_own;
  }
  if (lane < n) w.entries[lane] = own ? pos : -1;
  if (grouped_ids && own) {
    const int lead = __ffs(grp) - 1;  // the group's offset is its leader's
    const int goff = __shfl_sync(grp, off, lead);
    w.entries[n + goff + pos] = lane;
  }
}

// Small decode batches (T <= 8, E <= 512): the top-k of every token (one
// warp each) and the routing in one CTA of 8 warps.  The selections meet in
// shared memory behind one CTA barrier, so the launch needs neither the
// arrival ticket of the multi-CTA form (a fence before it and after it) nor
// L2 round trips for the selections (batch 1: 13.5 -> 12.3 us per layer).
// Larger batches keep their tokens on several SMs: a token's top-k is a
// long dependent chain, and 32 of them on one SM took 24 us against 18.
constexpr int kTopkSmallTokens = 8;
template <int PER>
__global__ void __launch_bounds__(kTopkSmallTokens * 32) topk_route_small_kernel(
    MoeDevice m, MoeWork w, int T, int pass_nt, int pass_dn, int grouped_ids) {
  __shared__ int s_sel[kTopkSmallTokens * 32];  // [token][rank], top_k <= 32
  griddep_wait();
  griddep_launch();
  const int t = threadIdx.x >> 5;
  if (t < T) topk_token<PER>(m, w, t, threadIdx.x & 31, s_sel);
  if (grouped_ids < 0) return;  // the caller groups the entries (token dispatch)
  __syncthreads();
  if (T * m.top_k <= 32) {
    if (threadIdx.x < 32)
      route_sparse_warp(m, w, T, pass_nt, pass_dn, grouped_ids != 0, s_sel, threadIdx.x);
  } else {
    route_block<kSelShared>(m, w, T, pass_nt, pass_dn, grouped_ids != 0, s_sel);
  }
  if (w.up_tickets)
    for (int i = threadIdx.x; i < kUpSplitItems; i += blockDim.x) w.up_tickets[i] = 0;
}

// Groups the (token, rank) entries by owned expert, stably.  One CTA of up to
// 8 warps.  pass_nt / pass_dn: tokens per pass of the up / down kernel;
// pass_off / pass_off_dn count passes.  CG: the selections were written by other CTAs of the same launch
// (read through L2).
// The per-expert part of the routing, from the entries' per-expert counts in
// shared memory: exclusive scans over experts (entries, up passes, down
// passes) and the active list in increasing expert id, written with the
// counts and the offsets.  Whole CTA of up to 8 warps.
__device__ __forceinline__ void route_scan(const MoeDevice& m, const MoeWork& w, int pass_nt,
                                           int pass_dn, const int* s_count, int* s_offset) {
  const int E = m.experts;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Exclusive scans over experts (entries, up passes, down passes) and the
  // active list in increasing expert id: warp wp takes experts
  // [wp*per_w, (wp+1)*per_w); pass 1 sums each warp's range, pass 2 scans it
  // from the sum of the ranges before it.
  {
    __shared__ int s_tot[8][4];
    const int nw = blockDim.x >> 5;
    const int per_w = ((E + nw - 1) / nw + 31) & ~31;
    const int e_lo = warp * per_w, e_hi = min(E, e_lo + per_w);
    const unsigned lt_mask = (1u << lane) - 1u;
    int tot[4] = {0, 0, 0, 0};  // entries, active experts, up passes, down passes
    for (int e0 = e_lo; e0 < e_hi; e0 += 32) {
      const int e = e0 + lane;
      const int cnt = e < e_hi ? s_count[e] : 0;
      tot[0] += (int)__reduce_add_sync(0xffffffffu, (unsigned)cnt);
      tot[1] += __popc(__ballot_sync(0xffffffffu, cnt > 0));
      tot[2] += (int)__reduce_add_sync(0xffffffffu, (unsigned)((cnt + pass_nt - 1) / pass_nt));
      tot[3] += (int)__reduce_add_sync(0xffffffffu, (unsigned)((cnt + pass_dn - 1) / pass_dn));
    }
    if (lane < 4)  // (selects, not a register array indexed by the lane)
      s_tot[warp][lane] = lane == 0 ? tot[0] : lane == 1 ? tot[1] : lane == 2 ? tot[2] : tot[3];
    __syncthreads();
    int run = 0, nact = 0, prun = 0, drun = 0;
    for (int q = 0; q < warp; ++q) {
      run += s_tot[q][0];
      nact += s_tot[q][1];
      prun += s_tot[q][2];
      drun += s_tot[q][3];
    }
    for (int e0 = e_lo; e0 < e_hi; e0 += 32) {
      const int e = e0 + lane;
      const int cnt = e < e_hi ? s_count[e] : 0;
      const int pc = (cnt + pass_nt - 1) / pass_nt, dc = (cnt + pass_dn - 1) / pass_dn;
      int incl = cnt, pincl = pc, dincl = dc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        const int pv = __shfl_up_sync(0xffffffffu, pincl, o);
        const int dv = __shfl_up_sync(0xffffffffu, dincl, o);
        if (lane >= o) {
          incl += v;
          pincl += pv;
          dincl += dv;
        }
      }
      if (e < e_hi) s_offset[e] = run + incl - cnt;
      const unsigned nz = __ballot_sync(0xffffffffu, cnt > 0);
      if (cnt > 0) {
        const int a = nact + __popc(nz & lt_mask);
        w.active[a] = e;
        w.pass_off[a] = prun + pincl - pc;
        w.pass_off_dn[a] = drun + dincl - dc;
      }
      nact += __popc(nz);
      run += __shfl_sync(0xffffffffu, incl, 31);
      prun += __shfl_sync(0xffffffffu, pincl, 31);
      drun += __shfl_sync(0xffffffffu, dincl, 31);
    }
    if (warp == nw - 1 && lane == 0) {
      s_offset[E] = run;
      w.active[E] = nact;
      w.pass_off[nact] = prun;
      w.pass_off_dn[nact] = drun;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    w.counts[e] = s_count[e];
    w.offsets[e] = s_offset[e];
  }
  if (threadIdx.x == 0) w.offsets[E] = s_offset[E];
  __syncthreads();
}

template <int SRC>
__device__ __forceinline__ void route_block(const MoeDevice& m, const MoeWork& w, int T,
                                            int pass_nt, int pass_dn, bool grouped_ids,
                                            const int* s_sel) {
  __shared__ int s_count[kMaxExperts];
  __shared__ int s_offset[kMaxExperts + 1];
  const int E = m.experts, k = m.top_k;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  // Stable grouping of entries (token-major, rank-minor) by owned expert.
  // Small batches: warp 0 walks all entries.  Large batches: warp q walks
  // the q-th contiguous range of 32-entry chunks with its own per-expert
  // counters, and each entry's position is then offset by the entries the
  // warps before it gave the same expert, which keeps the order stable.
  const int n = T * k;
  const int nchunk = (n + 31) >> 5;
  const bool split = nchunk >= 8 * kRouteSplitChunks && E * nw <= kRouteSplitSlots;
  __shared__ int s_wcount[kRouteSplitSlots];  // [warp][expert] when split
  const int walkers = split ? nw : 1;
  int* my_count = split ? s_wcount + warp * E : s_count;
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_count[e] = 0;
  if (split)
    for (int i = threadIdx.x; i < E * nw; i += blockDim.x) s_wcount[i] = 0;
  __syncthreads();
  const int c_lo = (int)((long)nchunk * warp / walkers), c_hi = (int)((long)nchunk * (warp + 1) / walkers);
  if (warp < walkers) {
    const unsigned lt_mask = (1u << lane) - 1u;
    int ev[8];  // selections of the next 8 chunks, loaded ahead of the serial part
    for (int ci = c_lo; ci < c_hi; ++ci) {
      const int c = ci << 5;
      const int u = (ci - c_lo) & 7;
      if (u == 0)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int idj = c + 32 * j + lane;  // clamped, not guarded: the loads overlap
          const int v = sel_at<SRC>(w, s_sel, min(idj, n - 1));
          ev[j] = idj < n && ci + j < c_hi ? v : -1;
        }
      const int id = c + lane;
      int e = ev[0];
#pragma unroll
      for (int j = 1; j < 8; ++j)
        if (j == u) e = ev[j];
      const bool own = e >= m.expert_begin && e < m.expert_end;
      const unsigned act = __ballot_sync(0xffffffffu, own);
      int rank = 0;
      unsigned grp = 0;
      if (own) {
        grp = __match_any_sync(act, e);
        rank = __popc(grp & lt_mask);
      }
      int base = own ? my_count[e] : 0;
      __syncwarp();
      if (own && rank == 0) my_count[e] = base + __popc(grp);
      __syncwarp();
      if (id < n) w.entries[id] = own ? (base + rank) : -1;  // position, fixed below
    }
  }
  __syncthreads();
  if (split) {
    // per expert: the total, and each warp's start among the expert's entries
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      int run = 0;
      for (int q = 0; q < nw; ++q) {
        const int v = s_wcount[q * E + e];
        s_wcount[q * E + e] = run;
        run += v;
      }
      s_count[e] = run;
    }
    __syncthreads();
    if (warp > 0) {  // warp 0's positions already start at 0; 8 entries' loads in flight
      const int id_end = min(n, c_hi << 5);
      for (int id0 = (c_lo << 5) + lane; id0 < id_end; id0 += 8 * 32) {
        int pos[8], e[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int id = min(id0 + 32 * u, id_end - 1);
          pos[u] = w.entries[id];
          e[u] = sel_at<SRC>(w, s_sel, id);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int id = id0 + 32 * u;
          if (id < id_end && pos[u] >= 0) w.entries[id] = pos[u] + s_wcount[warp * E + e[u]];
        }
      }
    }
    __syncthreads();
  }
  route_scan(m, w, pass_nt, pass_dn, s_count, s_offset);
  // Scatter entry ids into their expert-grouped slots (second half of entries;
  // the first half holds each entry's position within its expert).  The
  // prefill path reads positions only and skips it.  Four entries' loads
  // per thread are in flight at once.
  if (!grouped_ids) return;
  for (int id0 = threadIdx.x; id0 < n; id0 += 4 * blockDim.x) {
    int pos[4], e[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int id = min(id0 + u * (int)blockDim.x, n - 1);
      pos[u] = w.entries[id];
      e[u] = sel_at<SRC>(w, s_sel, id);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int id = id0 + u * (int)blockDim.x;
      if (id < n && pos[u] >= 0) w.entries[T * k + s_offset[e[u]] + pos[u]] = id;
    }
  }
}


// Prefill batches: the top-k of every token (one warp each) and each owned
// entry's position within its expert, taken by an atomic increment of the
// expert's count (zeroed before the launch); the last CTA to finish (an
// arrival ticket) scans the counts.  Positions within an expert follow
// arrival, not entry order: the prefill passes compute every grouped row from
// its own token alone, so the order changes no value.  The one-CTA stable
// grouping it replaces walked all T * k entries (20480 at batch 2048) on the
// routing CTA.
template <int PER>
__global__ void __launch_bounds__(256) topk_count_kernel(MoeDevice m, MoeWork w, int T,
                                                         int pass_nt, int pass_dn) {
  __shared__ int s_last;
  __shared__ int s_count[kMaxExperts];
  __shared__ int s_offset[kMaxExperts + 1];
  griddep_wait();
  griddep_launch();
  const int lane = threadIdx.x & 31, k = m.top_k;
  const int t = blockIdx.x * kTopkTokens + (threadIdx.x >> 5);
  if (t < T) {
    topk_token<PER>(m, w, t, lane);
    if (lane < k) {
      const int e = w.sel[t * k + lane];  // this thread's own store
      const bool own = e >= m.expert_begin && e < m.expert_end;
      w.entries[t * k + lane] = own ? atomicAdd(w.counts + e, 1) : -1;
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(w.tickets, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();  // every CTA's counts are final from here
  for (int e = threadIdx.x; e < m.experts; e += blockDim.x) s_count[e] = __ldcg(w.counts + e);
  __syncthreads();
  route_scan(m, w, pass_nt, pass_dn, s_count, s_offset);
  if (threadIdx.x == 0) *w.tickets = 0;
  if (w.up_tickets)
    for (int i = threadIdx.x; i < kUpSplitItems; i += blockDim.x) w.up_tickets[i] = 0;
}

// ---------------------------------------------------------------- prep
// Per token: optional rms-norm (rms-norm-into, llambda.lisp L859-879:
// scale = 1/sqrt(mean(x^2) + eps), dest = (x * weight) * scale), then the
// router input (natural layout) and the prepared gate/up input (weight-type
// layout with sub-block sums, zero-padded from H to k_in).
template <int UT>
__global__ void __launch_bounds__(256) moe_prep_kernel(MoeDevice m, MoeWork w,
                                                       const float* __restrict__ x) {
  constexpr int kCached = 8;  // chunks of 1024 values kept in registers (K <= 8192)
  __shared__ float s_part[8];
  const int H = m.hidden, K = m.k_in, tasks = K >> 6;
  const float* xt = x + (long)blockIdx.x * H;
  const int nchunk = (K + 1023) >> 10;
  if (threadIdx.x == 0) {  // the router GEMV that follows finds its weights in L2
    const int rows = m.router_rows;
    const size_t bytes = (size_t)rows * H * sizeof(float);
    const size_t per = ((bytes + gridDim.x - 1) / gridDim.x + 15) & ~size_t(15);
    const size_t lo = (size_t)blockIdx.x * per;
    if (lo < bytes && (reinterpret_cast<uintptr_t>(m.router) & 15) == 0)
      prefetch_l2(reinterpret_cast<const uint8_t*>(m.router) + lo,
                  (uint32_t)(std::min(per, bytes - lo) & ~size_t(15)));
  }
  const bool vec = (H & 3) == 0 && (reinterpret_cast<uintptr_t>(xt) & 15) == 0;
  auto load4 = [&](int e) {  // x[e..e+3], zero past H
    if (vec && e + 3 < H) return __ldg(reinterpret_cast<const float4*>(xt + e));
    float4 r;
    r.x = e < H ? xt[e] : 0.f;
    r.y = e + 1 < H ? xt[e + 1] : 0.f;
    r.z = e + 2 < H ? xt[e + 2] : 0.f;
    r.w = e + 3 < H ? xt[e + 3] : 0.f;
    return r;
  };
  // one read of x: every chunk's four values are loaded before the reduction
  float4 v[kCached];
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < kCached; ++c) {
    v[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < nchunk) {
      v[c] = load4(c * 1024 + 4 * threadIdx.x);
      acc = fmaf(v[c].x, v[c].x, acc);
      acc = fmaf(v[c].y, v[c].y, acc);
      acc = fmaf(v[c].z, v[c].z, acc);
      acc = fmaf(v[c].w, v[c].w, acc);
    }
  }
  for (int c = kCached; c < nchunk; ++c) {
    const float4 u = load4(c * 1024 + 4 * threadIdx.x);
    acc = fmaf(u.x, u.x, fmaf(u.y, u.y, fmaf(u.z, u.z, fmaf(u.w, u.w, acc))));
  }
  float scale = 1.f;
  if (m.input_norm) {  // rms-norm-into, llambda.lisp L859-879
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
  auto emit = [&](int e, float4 u) {
    float val[4] = {u.x, u.y, u.z, u.w};
    if (m.input_norm) {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (e + q < H) {
          val[q] = __fmul_rn(__fmul_rn(val[q], m.input_norm[e + q]), scale);
          xn[e + q] = val[q];
        }
    }
    const float4 o = make_float4(val[0], val[1], val[2], val[3]);
    if (UT == LB_TYPE_Q4_K)  // tensor-core layout (mma.cuh)
      mx_store4(reinterpret_cast<uint8_t*>(xp), K, e, o);
    else
      *reinterpret_cast<float4*>(xp + xp_index<UT>(e, tasks)) = o;
  };
  // K is a multiple of 256 and blockDim 256, so whole warps agree on e < K
#pragma unroll
  for (int c = 0; c < kCached; ++c) {
    const int e = c * 1024 + 4 * threadIdx.x;
    if (c < nchunk && e < K) emit(e, v[c]);
  }
  for (int c = kCached; c < nchunk; ++c) {
    const int e = c * 1024 + 4 * threadIdx.x;
    if (e < K) emit(e, load4(e));
  }
}

// Prep and router in one kernel (Q4_K gate/up): a CTA takes 8 tokens and 16
// router rows, which arrive by two bulk copies; the token tile is
// rms-normalised in shared memory (rms-norm-into, L859-879), the warps of
// all row tiles share the writes of the tokens' prepared gate/up input (one
// super-block of one token each), and every CTA forms its 16 x 8 logits (dot-product-with-f32-tensor-data, L4096-4107) with
// packed fp32x2 FMAs and a 31-shuffle butterfly.  Row E of qwen3next (the
// shared-expert gate) comes from router_extra_row when it is kept apart.
// TOK: tokens per CTA, 8, or 4 where 8 tokens' and 16 rows' worth of the
// hidden size would not fit in shared memory (config 4, hidden 2688).
constexpr int kRouterRows = 16, kRouterWarps = 8;
template <int TOK>
__global__ void __launch_bounds__(kRouterWarps * 32) moe_router_kernel(
    MoeDevice m, MoeWork w, const float* __restrict__ x, int T, int router_rows) {
  constexpr int kRouterTok = TOK;
  extern __shared__ float4 rs4[];  // [8][H/4] tokens, then [16][H/4] router rows
  __shared__ __align__(8) uint64_t bar_x, bar_w;
  __shared__ float s_scale[kRouterTok];
  const int H = m.hidden, H4 = H >> 2, E = m.experts;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.y * kRouterTok, nt = min(kRouterTok, T - t0);
  const int crow0 = blockIdx.x * kRouterRows, crows = min(kRouterRows, router_rows - crow0);
  const int main_end = m.router_rows;  // rows of m.router; then router_extra_row
  const int main_rows = max(0, min(crows, main_end - crow0));
  float4* xs4 = rs4;
  float4* ws4 = rs4 + kRouterTok * H4;
  if (threadIdx.x == 0) {  // the token tile and the rows complete on separate barriers, so
    mbar_init(&bar_x, 1);  // the norm and the prepared input overlap the rows' copy
    mbar_init(&bar_w, 1);
    fence_mbar_init();
    const uint32_t rowb = (uint32_t)H * 4u;
    // the router rows do not depend on the kernel before: fetched first
    mbar_expect_tx(&bar_w, rowb * (uint32_t)crows);
    if (main_rows > 0) tma_load_1d(ws4, m.router + (size_t)crow0 * H, rowb * main_rows, &bar_w);
    if (main_rows < crows)  // row E, the last row of the last tile
      tma_load_1d(ws4 + (size_t)main_rows * H4, m.router_extra_row, rowb, &bar_w);
    griddep_wait();  // x is the previous kernel's output
    mbar_expect_tx(&bar_x, rowb * (uint32_t)nt);
    tma_load_1d(xs4, x + (long)t0 * H, rowb * nt, &bar_x);
  }
  griddep_launch();
  for (int i = nt * H4 + threadIdx.x; i < kRouterTok * H4; i += blockDim.x)
    xs4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncthreads();
  mbar_wait(&bar_x, 0, w.status);
  if (m.input_norm) {
    for (int tok = warp; tok < nt; tok += kRouterWarps) {
      float acc = 0.f;
      for (int c = lane; c < H4; c += 32) {
        const float4 v = xs4[tok * H4 + c];
        acc = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, acc))));
      }
      acc = warp_sum(acc);
      if (lane == 0) {
        const float ms = __fdiv_rn(acc, (float)H);
        s_scale[tok] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, m.norm_epsilon)));
      }
    }
    __syncthreads();
    const float4* nw4 = reinterpret_cast<const float4*>(m.input_norm);
    for (int i = threadIdx.x; i < nt * H4; i += blockDim.x) {
      const int tok = i / H4;
      const float sc = s_scale[tok];
      const float4 v = xs4[i], g = __ldg(nw4 + (i - tok * H4));
      xs4[i] = make_float4(__fmul_rn(__fmul_rn(v.x, g.x), sc), __fmul_rn(__fmul_rn(v.y, g.y), sc),
                           __fmul_rn(__fmul_rn(v.z, g.z), sc), __fmul_rn(__fmul_rn(v.w, g.w), sc));
    }
    __syncthreads();
  }
  {  // the experts' prepared input (zero-padded from H to k_in): the row tiles'
     // warps share the tokens' (token, super-block) items
    const int K = m.k_in, nsb = K >> 8;
    const long ld_up = up_ld_floats(K);
    for (int it = blockIdx.x * kRouterWarps + warp; it < nt * nsb;
         it += gridDim.x * kRouterWarps) {
      const int tok = it / nsb, sb = it - tok * nsb;
      uint8_t* mx = reinterpret_cast<uint8_t*>(w.xp_up + (long)(t0 + tok) * ld_up);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int e = sb * 256 + h * 128 + lane * 4;
        mx_store4(mx, K, e, e < H ? xs4[tok * H4 + (e >> 2)] : make_float4(0.f, 0.f, 0.f, 0.f));
      }
    }
  }
  mbar_wait(&bar_w, 0, w.status);
  constexpr int R = kRouterRows / kRouterWarps;  // this warp's rows of the tile
  const int row0 = warp * R;
  if (row0 >= crows) return;
  float2 acc[R][kRouterTok / 2];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int p = 0; p < kRouterTok / 2; ++p) acc[r][p] = make_float2(0.f, 0.f);
  const float4* wr[R];
#pragma unroll
  for (int r = 0; r < R; ++r) wr[r] = ws4 + (size_t)min(row0 + r, crows - 1) * H4;
  for (int c = lane; c < H4; c += 32) {
    float4 wv[R];
#pragma unroll
    for (int r = 0; r < R; ++r) wv[r] = wr[r][c];
#pragma unroll
    for (int p = 0; p < kRouterTok / 2; ++p) {
      const float4 xa = xs4[(2 * p) * H4 + c], xb = xs4[(2 * p + 1) * H4 + c];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        acc[r][p] = __ffma2_rn(make_float2(wv[r].x, wv[r].x), make_float2(xa.x, xb.x), acc[r][p]);
        acc[r][p] = __ffma2_rn(make_float2(wv[r].y, wv[r].y), make_float2(xa.y, xb.y), acc[r][p]);
        acc[r][p] = __ffma2_rn(make_float2(wv[r].z, wv[r].z), make_float2(xa.z, xb.z), acc[r][p]);
        acc[r][p] = __ffma2_rn(make_float2(wv[r].w, wv[r].w), make_float2(xa.w, xb.w), acc[r][p]);
      }
    }
  }
  // transpose-reduce of the warp's NV = R * TOK sums over the 32 lanes: each
  // halving step keeps half of a lane's values (the upper lanes the upper
  // half) and adds the partner's, so value r * TOK + n ends on the lanes
  // whose bits above the low LS bits spell its index; the low bits are summed
  // last
  constexpr int NV = R * kRouterTok;
  static_assert(NV == 16 || NV == 8, "two rows of eight or four tokens per warp");
  constexpr int LS = NV == 16 ? 1 : 2;
  float v[NV];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int p = 0; p < kRouterTok / 2; ++p) {
      v[r * kRouterTok + 2 * p] = acc[r][p].x;
      v[r * kRouterTok + 2 * p + 1] = acc[r][p].y;
    }
#pragma unroll
  for (int h = 16, cnt = NV / 2; cnt >= 1; h >>= 1, cnt >>= 1) {
    const bool upper = (lane & h) != 0;
#pragma unroll
    for (int i = 0; i < cnt; ++i) {
      const float send = upper ? v[i] : v[i + cnt];
      const float keep = upper ? v[i + cnt] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, h);
    }
  }
#pragma unroll
  for (int h = 1 << (LS - 1); h >= 1; h >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], h);
  const int idx = (lane >> LS) & (NV - 1), r = idx / kRouterTok, n = idx % kRouterTok;
  if ((lane & ((1 << LS) - 1)) == 0 && row0 + r < crows && n < nt)
    w.logits[(long)(t0 + n) * (E + 1) + crow0 + row0 + r] = v[0];
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
  const long ld_dn = down_ld_floats(m);
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
// A gate/up work item as the producer publishes it with the item's first
// stage (before it arms that stage's barrier): the slab's first row, the
// matrix's rows, the pass's entries and their ids.
struct __align__(16) UpUnit {
  int row0, rows_e, nt, shared;
  int ids[4];
};

struct SlabSync {
  uint64_t full[kSlabMaxStages];
  uint64_t empty[kSlabMaxStages];
  uint64_t xfull[2];
  uint64_t xempty[2];
  UpUnit unit[kSlabMaxStages];
  int abort;
  int pad[3];
  uint4 zero[2];  // the B source of the threads whose column cannot be non-zero
};

// DL: the layout the gate/up epilogue writes the down input in: 0 the
// warp-engine layout (xp_index), 1 i6 (Q6_K sub-block slots, for passes of
// one or two entries), 2 m6 (four entries per mma, for passes of four).
enum DownLayout { kDownPlain = 0, kDownI6 = 1, kDownM6 = 2 };

template <int NT, bool PAIR, int DT, int DL, int CW>
__global__ void __launch_bounds__((CW + 1) * 32, 1)
    moe_up_slab_kernel(MoeDevice m, MoeWork w, int T, int stages, long map_row_base,
                       const __grid_constant__ CUtensorMap tm_gate,
                       const __grid_constant__ CUtensorMap tm_up,
                       const __grid_constant__ CUtensorMap tm_gate_sh,
                       const __grid_constant__ CUtensorMap tm_up_sh) {
  constexpr int MATS = PAIR ? 2 : 1;
  constexpr int RBM = CW / MATS;       // row blocks per matrix
  constexpr int RU = RBM * kTileRows;  // rows per matrix per slab
  static_assert(RU % kUpBoxRows == 0, "slab rows must be whole copy boxes");
  constexpr int BOX = kTileRows * LB_Q4K;
  constexpr int STAGE_W = CW * BOX;  // weights; then NT activation slices of 1088 bytes
  constexpr int STAGE = up_stage_bytes(CW, NT);
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
    sync->zero[0] = sync->zero[1] = make_uint4(0, 0, 0, 0);
    fence_mbar_init();
  }
  __syncthreads();
  griddep_wait();  // the routing and prepared inputs of the kernels before
  griddep_launch();
  const int k = m.top_k;
  const int per_r = (m.inter + RU - 1) / RU;
  const int per_s = (m.inter_sh + RU - 1) / RU;
  int sh_t0, sh_t1;
  shared_tokens(m, T, sh_t0, sh_t1);
  const int passes_s = (sh_t1 - sh_t0 + NT - 1) / NT;
  const int nact = w.active[m.experts];
  // work items: (slab, pass of up to NT tokens), all of one cost; routed ones
  // expert-major (passes of expert a: pass_off[a] ..), then slab, then pass
  const int n_routed = w.pass_off[nact] * per_r;
  const int n_shared = (m.shared_here && m.inter_sh) ? per_s * passes_s : 0;
  const int units = n_routed + n_shared;
  const int nsb = m.k_in >> 8;
  // with few items (one-token passes: decode batch 1), each is cut into nks
  // slices of its super-block columns; other pass sizes keep whole items
  constexpr bool kSplit = NT == 1;
  const int nks = kSplit && w.up_part ? up_split(units, gridDim.x, nsb) : 1;
  const int u0 = (int)((long)blockIdx.x * units * nks / gridDim.x);
  const int n_my = (int)((long)(blockIdx.x + 1) * units * nks / gridDim.x) - u0;

  struct Unit {
    int row0, rows_e, t_begin, t_end;
    long map_row;  // row of the slab's first row in its tensor map
    bool shared;
  };
  ExpertView view;
  int a_hint = -1;  // active index of the previous item (items are visited in order)
  auto unit_at = [&](int u) {
    Unit x;
    if (u < n_routed) {
      // the active expert a with pass_off[a] * per_r <= u < pass_off[a + 1] * per_r:
      // items come in order, so step on from the previous item's expert; the
      // first item of a CTA searches
      int a = a_hint;
      if (a < 0) {
        a = 0;
        int hi = nact;
        while (hi - a > 1) {
          const int mid = (a + hi) >> 1;
          if (w.pass_off[mid] * per_r <= u) a = mid; else hi = mid;
        }
      } else {
        while (w.pass_off[a + 1] * per_r <= u) ++a;
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
      x.t_begin = sh_t0 + p * NT;
      x.t_end = min(sh_t1, x.t_begin + NT);
      x.map_row = x.row0;
    }
    return x;
  };

  const long ld_up = up_ld_floats(m.k_in);
  if (warp == CW) {  // ---------------- producer
    if (lane == 0) {
      int q = 0;
      RingPos rp;
      bool ok = true;
      for (int i = 0; i < n_my && ok; ++i) {
        const int ub = (u0 + i) / nks, ks = (u0 + i) - ub * nks;
        const Unit x = unit_at(ub);
        const int sb_lo = ks * nsb / nks, sb_hi = (ks + 1) * nsb / nks;
        for (int t0 = x.t_begin; t0 < x.t_end && ok; t0 += NT) {
          for (int sb = sb_lo; sb < sb_hi; ++sb, ++q, rp.next(stages)) {
            const int s = rp.s;
            if (q >= stages && !mbar_wait_or_abort(&sync->empty[s], rp.phase ^ 1u, w.status, abort)) {
              ok = false;
              break;
            }
            const int nt = min(NT, x.t_end - t0);
            if (sb == sb_lo) {  // the item's rows and entries travel with its first stage
              UpUnit& uu = sync->unit[s];
              uu.row0 = x.row0;
              uu.rows_e = x.rows_e;
              uu.nt = nt;
              uu.shared = x.shared ? 1 : 0;
              for (int n = 0; n < NT; ++n) {
                const int tt = min(t0 + n, x.t_end - 1);
                uu.ids[n] = x.shared ? T * k + tt : view.list[tt];
              }
            }
            mbar_expect_tx(&sync->full[s], STAGE_W + nt * 1088);
            uint8_t* st = smem + (size_t)s * STAGE;
            // one box of kUpBoxRows rows per copy (the slab's blocks lie
            // back to back, 144 bytes per row, in the stage as in the matrix)
#pragma unroll
            for (int mt = 0; mt < MATS; ++mt)
#pragma unroll
              for (int b = 0; b < RU / kUpBoxRows; ++b) {
                const bool gate = PAIR && mt == 0;
                const CUtensorMap* tm = x.shared ? (gate ? &tm_gate_sh : &tm_up_sh)
                                                 : (gate ? &tm_gate : &tm_up);
                tma_load_2d(st + (mt * RU + b * kUpBoxRows) * LB_Q4K, tm, sb * LB_Q4K,
                            (int)(x.map_row + b * kUpBoxRows), &sync->full[s]);
              }
            // the pass's tokens' activation slices for this super-block
            for (int n = 0; n < nt; ++n) {
              const int tok = x.shared ? t0 + n : view.list[t0 + n] / k;
              const uint8_t* mx = reinterpret_cast<const uint8_t*>(w.xp_up + tok * ld_up);
              tma_load_1d(st + STAGE_W + n * 1088, mx + (size_t)sb * 1024, 1024, &sync->full[s]);
              tma_load_1d(st + STAGE_W + n * 1088 + 1024, mx + (size_t)nsb * 1024 + sb * 64, 64,
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
  const long ld_dn = down_ld_floats(m);
  RingPos rp;
  int pass = 0;  // items whose epilogue this CTA ran (the exchange's parity)
  bool ok = true;
  __shared__ int s_last;
  for (int i = 0; i < n_my && ok; ++i) {
    const int ub = (u0 + i) / nks, ks = (u0 + i) - ub * nks;
    const int sb_lo = ks * nsb / nks, sb_hi = (ks + 1) * nsb / nks;
    UpUnit x;  // read with the item's first stage
    int nt = 0;
    float2 acc[NT][2];
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int r = 0; r < 2; ++r) acc[n][r] = make_float2(0.f, 0.f);
    for (int sb = sb_lo; sb < sb_hi; ++sb, rp.next(stages)) {
      const int s = rp.s;
      if (!mbar_wait_or_abort(&sync->full[s], rp.phase, w.status, abort)) {
        ok = false;
        break;
      }
      if (sb == sb_lo) {  // the item, as the producer published it with this stage
        x = sync->unit[s];
        nt = x.nt;
      }
      const uint8_t* st = smem + (size_t)s * STAGE;
      const uint8_t* blk = st + warp * BOX;
      BSlice bs[NT];
#pragma unroll
      for (int n = 0; n < NT; ++n)
        bs[n] = BSlice{st + STAGE_W + n * 1088, st + STAGE_W + n * 1088 + 1024};
      q4k_sb_mma_n<NT, true>(nt, blk + g * LB_Q4K, blk + (g + 8) * LB_Q4K, bs,
                             reinterpret_cast<const uint8_t*>(sync->zero), lane, acc);
      __syncwarp();
      if (lane == 0) mbar_arrive(&sync->empty[s]);
    }
    if (!ok) break;
    const int kd = x.shared ? m.k_down_sh : m.k_down, tasks_d = kd >> 6;
    // row sums of rows g and g+8 of this block on lane t == 0 of each quad
    float v[2][NT];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        float s = acc[n][r].x + acc[n][r].y;
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        v[r][n] = s;
      }
    if (kSplit && nks > 1) {
      // this slice's row sums to the item's slot; the last of the item's
      // CTAs to arrive sums all slices in slice order and runs the epilogue
      float* part = w.up_part + (size_t)ub * kUpMaxSplit * kUpPartFloats;
      if (t == 0)
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
          for (int n = 0; n < NT; ++n)
            part[(size_t)ks * kUpPartFloats + (warp * kTileRows + g + 8 * r) * NT + n] = v[r][n];
      __threadfence();
      named_bar_sync(1, CW * 32);  // every consumer warp's slice is stored
      if (threadIdx.x == 0) s_last = atomicAdd(&w.up_tickets[ub], 1) == nks - 1;
      named_bar_sync(1, CW * 32);
      if (!s_last) continue;  // another CTA finishes this item
      __threadfence();
      // every lane of a quad holds its rows' sums (the gate warps use all four)
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            float sum = 0.f;
            for (int q = 0; q < nks; ++q)
              sum += q == ks ? v[r][n]
                             : __ldcg(part + (size_t)q * kUpPartFloats +
                                      (warp * kTileRows + g + 8 * r) * NT + n);
            v[r][n] = sum;
          }
      if (threadIdx.x == 0) w.up_tickets[ub] = 0;  // zero for the next launch
    }
    const int par = pass & 1, use = pass >> 1;
    ++pass;
    float* xb = xch + (size_t)par * RU * NT;
    auto id_of = [&](int nn) {  // ids[nn] without indexing registers dynamically
      int id = x.ids[0];
#pragma unroll
      for (int n2 = 1; n2 < NT; ++n2)
        if (n2 == nn) id = x.ids[n2];
      return id;
    };
    // h = silu(gate) * up or relu(up)^2 of rows g, g+8 (zero past rows_e),
    // on lane t == 0 of each quad; zero elsewhere
    float hv[2][NT];
    bool writer = !PAIR;
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
      // the quad's 2 * NT values (all four lanes hold every sum) are shared
      // out: lane t takes pairs (r, n) with 2n + r = t, t + 4, ..., and the
      // products come back to lane t == 0
      constexpr int PER_LANE = (2 * NT + 3) / 4;
      float hq[PER_LANE];
#pragma unroll
      for (int i = 0; i < PER_LANE; ++i) {
        const int pr = t + 4 * i, r = pr & 1, n = pr >> 1;
        float gv = v[0][0];
#pragma unroll
        for (int r2 = 0; r2 < 2; ++r2)
#pragma unroll
          for (int n2 = 0; n2 < NT; ++n2)
            if (r2 == r && n2 == n) gv = v[r2][n2];
        const int row = x.row0 + rb * kTileRows + g + 8 * r;
        const bool live = n < NT && n < nt && row < x.rows_e;
        const float uv = xb[(rb * kTileRows + g + 8 * r) * NT + min(n, NT - 1)];
        hq[i] = live ? __fmul_rn(silu_ref(gv), uv) : 0.f;
      }
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          const int pr = 2 * n + r;
          const float o = __shfl_sync(0xffffffffu, hq[pr >> 2], (lane & ~3) | (pr & 3));
          hv[r][n] = t == 0 ? o : 0.f;
        }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sync->xempty[par]);
      writer = true;
    }
    if (!PAIR) {  // up only: relu(up)^2
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          const int row = x.row0 + rb * kTileRows + g + 8 * r;
          hv[r][n] = (t == 0 && row < x.rows_e && n < nt) ? relu_sq_ref(v[r][n]) : 0.f;
        }
    }
    if (writer) {
      if (DL != kDownPlain) {  // the block's 16 rows are one Q6_K sub-block of the down input
        const int s_glob = (x.row0 + rb * kTileRows) >> 4;
#pragma unroll
        for (int n = 0; n < NT; ++n)
          if (n < nt) {
            uint8_t* dst = reinterpret_cast<uint8_t*>(w.xp_down + (long)id_of(n) * ld_dn);
            if (DL == kDownM6)
              m6_store_subblock(dst, s_glob, hv[0][n], hv[1][n], lane);
            else
              i6_store_subblock(dst, s_glob, hv[0][n], hv[1][n], lane);
          }
      } else if (t == 0) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int row = x.row0 + rb * kTileRows + g + 8 * r;
#pragma unroll
          for (int n = 0; n < NT; ++n)
            if (row < x.rows_e && n < nt)
              w.xp_down[(long)id_of(n) * ld_dn + xp_index<DT>(row, tasks_d)] = hv[r][n];
        }
      }
    }
    if (warp == 0 && x.row0 + RU >= x.rows_e) {  // last slab: zero the padding up to kd
      if (DL != kDownPlain) {  // sub-blocks past the slab (the slab's own are written above)
        const int s_from = (x.row0 + RU) >> 4, s_to = kd >> 4;
        for (int qq = lane >> 4; qq < nt * (s_to - s_from); qq += 2) {
          const int nn = qq / (s_to - s_from), sg = s_from + (qq - nn * (s_to - s_from));
          uint8_t* dst = reinterpret_cast<uint8_t*>(w.xp_down + (long)id_of(nn) * ld_dn);
          if (DL == kDownM6)
            m6_zero_subblock(dst, sg, lane & 15);
          else
            i6_zero_subblock(dst, sg, lane & 15);
        }
      } else {
        const int pad = kd - x.rows_e;
        for (int qq = lane; qq < nt * pad; qq += 32) {
          const int nn = qq / pad, pe = x.rows_e + (qq - nn * pad);
          w.xp_down[(long)id_of(nn) * ld_dn + xp_index<DT>(pe, tasks_d)] = 0.f;
        }
      }
    }
  }
}

// ---------------------------------------------------------------- down (slabs)
// Q6_K down rows on the tensor cores (mma.cuh, Q6_K rows in sub-block slots,
// one mma per entry and k-step): a work item is a
// slab of RU = 16 * CW / KSPLIT rows of one routed expert's down matrix (or
// the shared expert's) for one pass of up to 4 entries.  A stage holds the
// slab's 16-row blocks whole (16 rows x row bytes is a multiple of 16 bytes,
// so each block is one aligned 1-D bulk copy); consumer warp w takes block
// w / KSPLIT and super-blocks part w % KSPLIT of K.  With KSPLIT > 1 the
// other parts' sums reach the part-0 warp through shared memory, guarded by
// a per-stage barrier.  Lane (g, t) ends with rows g, g+8 of its block for
// the pass's entry t and writes them to `partial`.
// What a stage holds, written by the producer before it arms the stage's
// barrier (whose arrive releases it to the consumers): the slab's first row
// and, per entry of the pass, its prepared-input id and output row of
// `partial` (token * (k + 1) + slot).
struct __align__(16) DownUnit {
  int row0, nt, pad[2];
  int id[8];
  int orow[8];
};

struct DownSync {
  uint64_t full[kSlabMaxStages];
  uint64_t empty[kSlabMaxStages];
  uint64_t red[kSlabMaxStages];
  DownUnit unit[kSlabMaxStages];
  int abort;
  int pad[3];
  uint4 zero[2];  // the B source of the threads without a column of their own
};

// SB: the pass's entries' prepared inputs are staged with the weights (at
// stage_w, i6_bytes(K) each) instead of being read through L1.
// M6: the inputs are in the m6 layout (one mma per k-step serves four
// entries of a pass) instead of i6 (one mma per entry and k-step).
// NTD: entries per pass, 4, or 8 in m6 (two groups of four per k-step, so an
// expert with five to eight entries streams its rows once).
// shared_pass: 0 the routed experts' slabs, 1 the shared expert's, 2 both in
// one launch (routed units first; the shared down rows must then have the
// routed rows' width).
template <int KSPLIT, int CW, bool SB, bool M6, int NTD>
__global__ void __launch_bounds__((CW + 1) * 32, 1)
    moe_down_slab_kernel(MoeDevice m, MoeWork w, int T, int stages, int stage_bytes,
                         int stage_w, int shared_pass) {
  constexpr int NB = CW / KSPLIT;  // 16-row blocks per slab
  constexpr int RU = NB * kTileRows;
  constexpr int NT = NTD;
  constexpr int NG = NTD / 4;  // groups of four entries
  static_assert(NTD == 4 || (NTD == 8 && M6), "eight entries per pass in m6 only");
  extern __shared__ __align__(128) uint8_t smem[];
  DownSync* sync = reinterpret_cast<DownSync*>(smem + (size_t)stages * stage_bytes);
  float2* red = reinterpret_cast<float2*>(sync + 1);  // [stages][CW][32][NG]
  volatile int* abort = &sync->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&sync->full[s], 1);
      mbar_init(&sync->empty[s], CW);
      mbar_init(&sync->red[s], CW - NB);
    }
    sync->abort = 0;
    sync->zero[0] = sync->zero[1] = make_uint4(0, 0, 0, 0);
    fence_mbar_init();
  }
  __syncthreads();
  griddep_wait();  // the routing and the gate/up pass's output
  griddep_launch();
  const int k = m.top_k, H = m.hidden;
  const int per = (H + RU - 1) / RU;
  const int K = shared_pass == 1 ? m.k_down_sh : m.k_down;
  const int nsb = K >> 8;
  const size_t rb = shared_pass == 1 ? m.down_sh_rb : m.down_rb;
  const long ld_dn = down_ld_floats(m);
  const uint32_t xib = (uint32_t)i6_bytes(K);

  if (warp == CW) {  // ---------------- producer: enumerates the units, stages them
    if (lane == 0) {
      int sh_t0, sh_t1;
      shared_tokens(m, T, sh_t0, sh_t1);
      const int passes_s = (sh_t1 - sh_t0 + NT - 1) / NT;
      const int nact = w.active[m.experts];
      const int n_routed = shared_pass == 1 ? 0 : w.pass_off_dn[nact] * per;
      const int n_shared = (shared_pass && m.shared_here && m.inter_sh) ? per * passes_s : 0;
      const int units = n_routed + n_shared;
      const int u0 = (int)((long)blockIdx.x * units / gridDim.x);
      const int n_my = (int)((long)(blockIdx.x + 1) * units / gridDim.x) - u0;
      ExpertView view;
      int a = -1;
      int q = 0;
      RingPos rp;
      for (int i = 0; i < n_my; ++i, ++q, rp.next(stages)) {
        const int u = u0 + i;
        const bool sh_u = u >= n_routed;  // a shared-expert unit
        int row0, t_begin, t_end;
        const uint8_t* src;
        if (!sh_u) {
          if (a < 0) {  // search once, then step on
            a = 0;
            int hi = nact;
            while (hi - a > 1) {
              const int mid = (a + hi) >> 1;
              if (w.pass_off_dn[mid] * per <= u) a = mid; else hi = mid;
            }
          } else {
            while (w.pass_off_dn[a + 1] * per <= u) ++a;
          }
          view_expert(m, w, T, a, view);
          const int np = w.pass_off_dn[a + 1] - w.pass_off_dn[a];
          const int local = u - w.pass_off_dn[a] * per, slab = local / np, p = local - slab * np;
          row0 = slab * RU;
          t_begin = p * NT;
          t_end = min(view.ntok, t_begin + NT);
          src = m.down_exps + ((size_t)view.e * H + row0) * rb;
        } else {
          const int us = u - n_routed, slab = us / passes_s, p = us - slab * passes_s;
          row0 = slab * RU;
          t_begin = sh_t0 + p * NT;
          t_end = min(sh_t1, t_begin + NT);
          src = m.down_sh + (size_t)row0 * rb;
        }
        const int s = rp.s;
        if (q >= stages && !mbar_wait_or_abort(&sync->empty[s], rp.phase ^ 1u, w.status, abort))
          break;
        const int nblk = min(NB, (H - row0) / kTileRows);  // H % 16 == 0
        const int nt = t_end - t_begin;
        DownUnit& du = sync->unit[s];
        du.row0 = row0;
        du.nt = nt;
        for (int n = 0; n < NT; ++n) {
          const int tt = t_begin + min(n, nt - 1);
          const int id = sh_u ? T * k + tt : view.list[tt];
          const int tok = sh_u ? tt : id / k;
          du.id[n] = id;
          du.orow[n] = tok * (k + 1) + (sh_u ? k : id - tok * k);
        }
        mbar_expect_tx(&sync->full[s], (uint32_t)(nblk * kTileRows * rb) + (SB ? nt * xib : 0u));
        uint8_t* st = smem + (size_t)s * stage_bytes;
        // the slab's blocks are contiguous rows: one copy
        tma_load_1d(st, src, (uint32_t)(nblk * kTileRows * rb), &sync->full[s]);
        if (SB)
          for (int n = 0; n < nt; ++n)
            tma_load_1d(st + stage_w + n * xib, w.xp_down + du.id[n] * ld_dn, xib, &sync->full[s]);
      }
      for (int r = max(0, q - stages); r < q; ++r)
        mbar_wait(&sync->full[r % stages], (r / stages) & 1, nullptr);
    }
    return;
  }

  // ---------------- consumers: the same units, in the same order
  int units_c;
  {
    int sh_t0, sh_t1;
    shared_tokens(m, T, sh_t0, sh_t1);
    const int passes_s = (sh_t1 - sh_t0 + NT - 1) / NT;
    const int n_routed = shared_pass == 1 ? 0 : w.pass_off_dn[w.active[m.experts]] * per;
    const int n_shared = (shared_pass && m.shared_here && m.inter_sh) ? per * passes_s : 0;
    units_c = n_routed + n_shared;
  }
  const int u0 = (int)((long)blockIdx.x * units_c / gridDim.x);
  const int n_my = (int)((long)(blockIdx.x + 1) * units_c / gridDim.x) - u0;
  const int b = warp / KSPLIT, kp = warp % KSPLIT;
  const int sb0 = kp * nsb / KSPLIT, sb1 = (kp + 1) * nsb / KSPLIT;
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* bz = SB ? reinterpret_cast<const uint8_t*>(sync->zero) : kZero32;
  RingPos rp;
  for (int i = 0; i < n_my; ++i, rp.next(stages)) {
    const int s = rp.s;
    if (!mbar_wait_or_abort(&sync->full[s], rp.phase, w.status, abort)) break;
    const DownUnit du = sync->unit[s];
    const int nt = du.nt;
    const int row_blk = du.row0 + b * kTileRows;
    const uint8_t* xin[NT];
#pragma unroll
    for (int n = 0; n < NT; ++n)
      xin[n] = SB ? smem + (size_t)s * stage_bytes + stage_w + min(n, nt - 1) * xib
                  : reinterpret_cast<const uint8_t*>(w.xp_down + (long)du.id[n] * ld_dn);
    float2 y[NG];
#pragma unroll
    for (int grp = 0; grp < NG; ++grp) y[grp] = make_float2(0.f, 0.f);
    if (row_blk < H && M6) {
      const uint8_t* blk = smem + (size_t)s * stage_bytes + (size_t)b * kTileRows * rb;
      for (int sb = sb0; sb < sb1; ++sb)
        q6k_sb_mma<SB, NG>(blk + g * rb + sb * LB_Q6K, blk + (g + 8) * rb + sb * LB_Q6K, sb, xin,
                           nt, lane, y);
    } else if (row_blk < H) {
      const uint8_t* blk = smem + (size_t)s * stage_bytes + (size_t)b * kTileRows * rb;
      if (nt == 1) {
        q6i_block<SB, 1>(blk, rb, sb0, sb1, xin, bz, lane, 0, y[0]);
      } else if (nt == 2 || CW > 8) {  // at most two entries per decode (registers)
        q6i_block<SB, 2>(blk, rb, sb0, sb1, xin, bz, lane, 0, y[0]);
        if (nt == 3) q6i_block<SB, 1>(blk, rb, sb0, sb1, xin + 2, bz, lane, 2, y[0]);
        if (nt == 4) q6i_block<SB, 2>(blk, rb, sb0, sb1, xin + 2, bz, lane, 2, y[0]);
      } else if (nt == 3) {
        q6i_block<SB, 3>(blk, rb, sb0, sb1, xin, bz, lane, 0, y[0]);
      } else {
        q6i_block<SB, 4>(blk, rb, sb0, sb1, xin, bz, lane, 0, y[0]);
      }
    }
    if (KSPLIT > 1) {
      float2* rs = red + ((size_t)s * CW) * 32 * NG;
      if (kp != 0) {
#pragma unroll
        for (int grp = 0; grp < NG; ++grp) rs[(warp * 32 + lane) * NG + grp] = y[grp];
        __syncwarp();
        if (lane == 0) mbar_arrive(&sync->red[s]);
      } else {
        if (!mbar_wait_or_abort(&sync->red[s], rp.phase, w.status, abort)) break;
#pragma unroll
        for (int p = 1; p < KSPLIT; ++p)
#pragma unroll
          for (int grp = 0; grp < NG; ++grp) {
            const float2 o = rs[((warp + p) * 32 + lane) * NG + grp];
            y[grp].x += o.x;
            y[grp].y += o.y;
          }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sync->empty[s]);
#pragma unroll
    for (int grp = 0; grp < NG; ++grp) {
      const int n = 4 * grp + t;  // this lane's entry of the group
      if (kp == 0 && row_blk < H && n < nt) {
        int orow = du.orow[0];
#pragma unroll
        for (int n2 = 1; n2 < NT; ++n2)
          if (n2 == n) orow = du.orow[n2];
        float* out = w.partial + (long)orow * H + row_blk;
        out[g] = y[grp].x;
        out[g + 8] = y[grp].y;
      }
    }
  }
}

// Q4_K down inputs need sub-block sums; Q6_K inputs do not.
__global__ void moe_down_sums_kernel(MoeDevice m, MoeWork w, int T) {
  const int k = m.top_k;
  const long ld_dn = down_ld_floats(m);
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
  const long ld_dn = down_ld_floats(m);
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
// VEC: four hidden values per thread (H % 4 == 0, x / out 16-byte aligned).
// KMAX >= top_k: the rank loop is unrolled whole over clamped (not guarded)
// addresses, so all of a thread's loads are in flight at once.
template <bool VEC, int KMAX>
__global__ void __launch_bounds__(128) combine_kernel(MoeDevice m, MoeWork w, int T,
                                                      const float* x, float* out) {
  constexpr int V = VEC ? 4 : 1;
  griddep_wait();
  griddep_launch();
  const int H = m.hidden, k = m.top_k, HV = H / V;
  const long n = (long)T * HV;
  const bool shared = m.shared_here && m.inter_sh;
  int sh_t0, sh_t1;
  shared_tokens(m, T, sh_t0, sh_t1);
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const int t = (int)(i / HV), h = (int)(i - (long)t * HV) * V;
    const float* p = w.partial + (long)t * (k + 1) * H + h;
    float acc[V];
#pragma unroll
    for (int c = 0; c < V; ++c) acc[c] = 0.f;
#pragma unroll
    for (int j = 0; j < KMAX; ++j) {
      const int jc = min(j, k - 1);
      const int es = w.sel[t * k + jc];
      const int e = j < k ? es : -1;
      const float wt = w.wts[t * k + jc];
      float pv[V];  // loaded unconditionally (a valid address), so all loads go out at once
      if (VEC) {
        const float4 q = *reinterpret_cast<const float4*>(p + (long)jc * H);
        pv[0] = q.x;
        pv[V > 1 ? 1 : 0] = q.y;
        pv[V > 2 ? 2 : 0] = q.z;
        pv[V > 3 ? 3 : 0] = q.w;
      } else {
        pv[0] = p[(long)jc * H];
      }
      // experts of other devices add +0.0, which leaves a sum that starts at
      // +0.0 unchanged (it can never be -0.0)
      const bool own = e >= m.expert_begin && e < m.expert_end;
#pragma unroll
      for (int c = 0; c < V; ++c) acc[c] = __fadd_rn(acc[c], own ? __fmul_rn(wt, pv[c]) : 0.f);
    }
    if (shared && t >= sh_t0 && t < sh_t1) {
      const float sw = m.arch == 0 ? w.shw[t] : 1.0f;
#pragma unroll
      for (int c = 0; c < V; ++c) {
        const float sv = p[(long)k * H + c];
        acc[c] = m.arch == 0 ? __fadd_rn(acc[c], __fmul_rn(sw, sv)) : __fadd_rn(acc[c], sv);
      }
    }
    // vector-add-into x x ffn-output (L5746) when the layer carries the residual
    const long o = (long)t * H + h;
#pragma unroll
    for (int c = 0; c < V; ++c) out[o + c] = m.add_residual ? __fadd_rn(x[o + c], acc[c]) : acc[c];
  }
}


// Flags between ranks: one system-scope fence orders a CTA's data stores
// (made visible to thread 0 by the barrier before it) ahead of every flag
// store that follows, so the flags themselves are relaxed stores; a
// release store per flag would wait for the previous remote store to be
// acknowledged each time, one NVLink round trip per peer.  The waiting side
// polls with relaxed loads and fences once, after every flag it needs.
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// Expert-parallel combine with the cross-rank reduction fused in, over peer
// memory.  CTA c owns a fixed chunk of the T x H outputs on every rank:
//   1. it forms this rank's partial (its routed experts in rank order, the
//      shared expert if here) and stores it into slot `rank` of every rank's
//      buffer (plain stores over NVLink, half of the slots by epoch parity);
//   2. it raises its flag on every rank (system-scope release after a
//      fence) and waits, with a bounded spin, for every rank's flag;
//   3. it sums the slots in rank order, plus the residual when the layer
//      carries it, so every rank ends with the whole layer output.
// Epochs are per-CTA counters in device memory, so the kernel can be replayed
// from a CUDA graph.  A rank can be at most one epoch ahead of another (to
// push epoch e+2 it needs every flag of e+1, raised only after that rank's
// sum of e), so two parities of slots suffice.
__global__ void __launch_bounds__(256) combine_ep_kernel(MoeDevice m, MoeWork w, int T,
                                                         const float* __restrict__ x,
                                                         float* __restrict__ out) {
  __shared__ uint32_t s_epoch;
  griddep_wait();
  griddep_launch();
  const int H = m.hidden, k = m.top_k, world = m.ep_world, rank = m.ep_rank;
  const int H4 = H >> 2;
  uint8_t* self = static_cast<uint8_t*>(m.ep_peers[rank]);
  if (threadIdx.x == 0) {
    uint32_t* epochs = reinterpret_cast<uint32_t*>(self);
    s_epoch = epochs[blockIdx.x] + 1u;
    epochs[blockIdx.x] = s_epoch;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  // phase stamps of CTA 0 (kernel timing only): start, pushed, peers seen, end
  unsigned long long* stamps = blockIdx.x == 0 && threadIdx.x == 0 ? m.ep_stamps : nullptr;
  if (stamps) stamps[0] = global_ns();
  const size_t slot = (size_t)m.ep_max_tokens * H;  // floats per (parity, rank)
  const size_t par = (size_t)(epoch & 1u) * world * slot;
  const long n4 = (long)T * H4;
  const long c0 = (long)blockIdx.x * n4 / gridDim.x, c1 = (long)(blockIdx.x + 1) * n4 / gridDim.x;
  const bool shared = m.shared_here && m.inter_sh;
  int sh_t0, sh_t1;
  shared_tokens(m, T, sh_t0, sh_t1);
  for (long i = c0 + threadIdx.x; i < c1; i += blockDim.x) {
    const int t = (int)(i / H4), h = (int)(i - (long)t * H4) * 4;
    const float* p = w.partial + (long)t * (k + 1) * H + h;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int j = 0; j < k; ++j) {
      const int e = w.sel[t * k + j];
      const float wt = w.wts[t * k + j];
      const float4 q = *reinterpret_cast<const float4*>(p + (long)j * H);
      const bool own = e >= m.expert_begin && e < m.expert_end;
      acc[0] = __fadd_rn(acc[0], own ? __fmul_rn(wt, q.x) : 0.f);
      acc[1] = __fadd_rn(acc[1], own ? __fmul_rn(wt, q.y) : 0.f);
      acc[2] = __fadd_rn(acc[2], own ? __fmul_rn(wt, q.z) : 0.f);
      acc[3] = __fadd_rn(acc[3], own ? __fmul_rn(wt, q.w) : 0.f);
    }
    if (shared && t >= sh_t0 && t < sh_t1) {
      const float sw = m.arch == 0 ? w.shw[t] : 1.0f;
      const float4 q = *reinterpret_cast<const float4*>(p + (long)k * H);
      const float sv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int c = 0; c < 4; ++c)
        acc[c] = m.arch == 0 ? __fadd_rn(acc[c], __fmul_rn(sw, sv[c])) : __fadd_rn(acc[c], sv[c]);
    }
    const float4 v = make_float4(acc[0], acc[1], acc[2], acc[3]);
    const size_t off = par + (size_t)rank * slot + (size_t)t * H + h;
    for (int q = 0; q < world; ++q)
      *reinterpret_cast<float4*>(static_cast<uint8_t*>(m.ep_peers[q]) + 8192 + off * 4) = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // the CTA's pushes before any of its flags
    for (int q = 0; q < world; ++q)
      st_relaxed_sys(reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(m.ep_peers[q]) + 4096) +
                         rank * kEpGrid + blockIdx.x,
                     epoch);
    const uint32_t* flags = reinterpret_cast<const uint32_t*>(self + 4096);
    const uint64_t t_start = global_ns();
    if (stamps) stamps[1] = t_start;
    bool late = false;
    for (int q = 0; q < world && !late; ++q) {
      while ((int)(ld_relaxed_sys(flags + q * kEpGrid + blockIdx.x) - epoch) < 0) {
        if (global_ns() - t_start > 2000000000ull) {  // bounded: two seconds
          late = true;
          break;
        }
        __nanosleep(32);
      }
    }
    fence_acq_rel_sys();  // every rank's slot stores before the reads below
    if (late) atomicOr(w.status, 4);  // a peer never arrived: the output is not valid
    if (stamps) stamps[2] = global_ns();
  }
  __syncthreads();
  const float* slots = reinterpret_cast<const float*>(self + 8192) + par;
  for (long i = c0 + threadIdx.x; i < c1; i += blockDim.x) {
    const int t = (int)(i / H4), h = (int)(i - (long)t * H4) * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < world; ++q) {  // rank order; L2 reads (peers wrote them)
      const float4 v = __ldcg(reinterpret_cast<const float4*>(slots + (size_t)q * slot +
                                                              (size_t)t * H + h));
      acc.x = __fadd_rn(acc.x, v.x);
      acc.y = __fadd_rn(acc.y, v.y);
      acc.z = __fadd_rn(acc.z, v.z);
      acc.w = __fadd_rn(acc.w, v.w);
    }
    const long o = (long)t * H + h;
    if (m.add_residual) {
      const float4 xv = *reinterpret_cast<const float4*>(x + o);
      acc = make_float4(__fadd_rn(xv.x, acc.x), __fadd_rn(xv.y, acc.y), __fadd_rn(xv.z, acc.z),
                        __fadd_rn(xv.w, acc.w));
    }
    *reinterpret_cast<float4*>(out + o) = acc;
  }
  if (blockIdx.x == 0 && m.ep_stamps) {
    __syncthreads();
    if (threadIdx.x == 0) m.ep_stamps[3] = global_ns();
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
  const cuuint32_t box[2] = {LB_Q4K, kUpBoxRows};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NT, bool PAIR, int DT, int DL, int CW>
cudaError_t launch_up_slab_cw(const MoeDevice& m, const MoeWork& w, int T, const SlabMaps& mp,
                              cudaStream_t s) {
  auto kern = moe_up_slab_kernel<NT, PAIR, DT, DL, CW>;
  constexpr int RU = CW / (PAIR ? 2 : 1) * kTileRows;
  const size_t stage = up_stage_bytes(CW, NT);
  const size_t extra = sizeof(SlabSync) + (size_t)2 * RU * NT * 4;
  const int stages = (int)std::min<size_t>(kSlabMaxStages, (kTileSmemBudget - extra) / stage);
  if (stages < 2) return cudaErrorInvalidValue;
  const size_t smem = (size_t)stages * stage + extra;
  if (prepared_occupancy(kern, (CW + 1) * 32, smem) < 1) return cudaErrorUnknown;
  return launch_pdl(kern, dim3(sm_count()), dim3((CW + 1) * 32), smem, s, m, w, T, stages,
                    mp.row_base, mp.gate, mp.up, mp.gate_sh, mp.up_sh);
}

// Shape of the Q6_K down slabs for rows of rb bytes: the most 16-row blocks
// (8, 4, 2 or 1) whose stage fits 56 KiB, K split over 8 / blocks warps.
struct DownPlan {
  int nb, stages, stage_bytes, stage_w;
  bool staged;  // entries' inputs staged with the weights
};
constexpr int kDownWarps = 8;

bool down_plan(size_t rb, int K, DownPlan* p, int ntd = 4) {
  const size_t block = (size_t)kTileRows * rb;
  int nb = 8;
  while (nb > 1 && nb * block > 56 * 1024) nb >>= 1;
  p->nb = nb;
  p->stage_w = (int)((nb * block + 127) & ~size_t(127));
  // the entries' inputs ride in the stage when three stages still fit
  const size_t red = nb < kDownWarps ? (size_t)kDownWarps * 32 * sizeof(float2) * (ntd / 4) : 0;
  const size_t room = kTileSmemBudget - sizeof(DownSync);
  p->staged = 4 * i6_bytes(K) <= 24 * 1024 &&
              room / (p->stage_w + ntd * i6_bytes(K) + red) >= 3;
  p->stage_bytes = p->stage_w + (p->staged ? (int)(ntd * i6_bytes(K)) : 0);
  const size_t per_stage = (size_t)p->stage_bytes + red;
  p->stages = (int)std::min<size_t>(kSlabMaxStages, room / per_stage);
  return p->stages >= 2;
}

// The down input is written in the i6 layout and the down pass runs on the
// Q6_K tensor-core slabs when the gate/up pass is the tensor-core one, the
// down rows are Q6_K, the hidden size is a multiple of 16 and the slabs fit.
double tokens_per_active_expert(const MoeDevice& m, int T);

// Where experts expect 2.5 or more tokens the down input is written in m6 and
// the down slabs (passes of four entries) take each k-step of all four in
// one mma; with fewer, most passes hold one or two entries and i6 gives each
// its own mma.
bool down_uses_m6(const MoeDevice& m, int T) {
  return m.up_type == LB_TYPE_Q4_K && T > 1 && tokens_per_active_expert(m, T) >= 2.5;
}

// Entries per down pass: 8 (two m6 groups per k-step) in a launch of the
// shared expert's slabs alone, which sees every token (config 4, batch 64:
// 60 -> 50 us); 4 for the routed experts, whose passes of eight were slower
// (223 -> 252 us: most experts hold four or fewer entries, and the second
// group's registers and mma cost every pass).
int down_pass_tokens(const MoeDevice& m, int T, int shared_pass) {
  return shared_pass == 1 && down_uses_m6(m, T) ? 8 : 4;
}

bool down_uses_i6(const MoeDevice& m) {
  DownPlan p;
  if (m.up_type != LB_TYPE_Q4_K || m.down_type != LB_TYPE_Q6_K || m.hidden % kTileRows) return false;
  if (!down_plan(m.down_rb, m.k_down, &p)) return false;
  return !(m.shared_here && m.inter_sh) || down_plan(m.down_sh_rb, m.k_down_sh, &p);
}

template <int KSPLIT, bool SB, bool M6, int NTD = 4>
cudaError_t launch_down_slab_k(const MoeDevice& m, const MoeWork& w, int T, int shared_pass,
                               const DownPlan& p, cudaStream_t s) {
  auto kern = moe_down_slab_kernel<KSPLIT, kDownWarps, SB, M6, NTD>;
  const size_t smem =
      (size_t)p.stages * p.stage_bytes + sizeof(DownSync) +
      (KSPLIT > 1 ? (size_t)p.stages * kDownWarps * 32 * sizeof(float2) * (NTD / 4) : 0);
  if (prepared_occupancy(kern, (kDownWarps + 1) * 32, smem) < 1) return cudaErrorUnknown;
  return launch_pdl(kern, dim3(sm_count()), dim3((kDownWarps + 1) * 32), smem, s, m, w, T,
                    p.stages, p.stage_bytes, p.stage_w, shared_pass);
}

cudaError_t launch_down_slab(const MoeDevice& m, const MoeWork& w, int T, int shared_pass,
                             cudaStream_t s) {
  DownPlan p;
  const int ntd = down_pass_tokens(m, T, shared_pass);
  if (!down_plan(shared_pass == 1 ? m.down_sh_rb : m.down_rb,
                 shared_pass == 1 ? m.k_down_sh : m.k_down, &p, ntd))
    return cudaErrorInvalidValue;
  const bool m6 = down_uses_m6(m, T);
#define LB_DOWN_SLAB(KS)                                                                     \
  if (ntd == 8)                                                                             \
    return p.staged ? launch_down_slab_k<KS, true, true, 8>(m, w, T, shared_pass, p, s)        \
                    : launch_down_slab_k<KS, false, true, 8>(m, w, T, shared_pass, p, s);      \
  return p.staged ? (m6 ? launch_down_slab_k<KS, true, true>(m, w, T, shared_pass, p, s)       \
                        : launch_down_slab_k<KS, true, false>(m, w, T, shared_pass, p, s))      \
                  : (m6 ? launch_down_slab_k<KS, false, true>(m, w, T, shared_pass, p, s)      \
                        : launch_down_slab_k<KS, false, false>(m, w, T, shared_pass, p, s));
  switch (kDownWarps / p.nb) {
    case 1: LB_DOWN_SLAB(1)
    case 2: LB_DOWN_SLAB(2)
    case 4: LB_DOWN_SLAB(4)
    default: LB_DOWN_SLAB(8)
  }
#undef LB_DOWN_SLAB
}

template <int NT, int DT>
cudaError_t launch_up_slab_nt(const MoeDevice& m, const MoeWork& w, int T, const SlabMaps& mp,
                              cudaStream_t s) {
  // 16 consumer warps where their registers fit (96 each), else 8
  constexpr int CW = NT <= 2 ? 16 : 8;
  const bool pair = m.arch == 0;
  if constexpr (NT > 1) {  // the down pass takes passes of four in m6
    if (DT == LB_TYPE_Q6_K && down_uses_i6(m) && down_uses_m6(m, T))
      return pair ? launch_up_slab_cw<NT, true, DT, kDownM6, CW>(m, w, T, mp, s)
                  : launch_up_slab_cw<NT, false, DT, kDownM6, CW>(m, w, T, mp, s);
  }
  if (DT == LB_TYPE_Q6_K && down_uses_i6(m))
    return pair ? launch_up_slab_cw<NT, true, DT, kDownI6, CW>(m, w, T, mp, s)
                : launch_up_slab_cw<NT, false, DT, kDownI6, CW>(m, w, T, mp, s);
  return pair ? launch_up_slab_cw<NT, true, DT, kDownPlain, CW>(m, w, T, mp, s)
              : launch_up_slab_cw<NT, false, DT, kDownPlain, CW>(m, w, T, mp, s);
}

// Tokens per pass (NT) of the tensor-core gate/up launch, from the expected
// tokens per active expert; the route kernel counts passes with the same NT.
// With T*k entries spread over E experts, about E * (1 - exp(-T*k / E))
// experts are hit, each by T*k / that many tokens on average; an expert-
// parallel rank sees the same ratio on its share of the experts and entries.
double tokens_per_active_expert(const MoeDevice& m, int T) {
  const double entries = (double)T * m.top_k, E = std::max(1, m.experts);
  const double hit = E * -std::expm1(-entries / E);
  return entries / std::max(1.0, hit);
}

// Two-token passes (16 consumer warps of 96 registers) up to 8 expected
// tokens per expert: at 4.8 (config 4, batch 64) they beat four-token passes
// (8 warps of 160 registers) by 15% although the weights are decoded twice
// as often.
int up_pass_tokens(const MoeDevice& m, int T) {
  if (m.up_type != LB_TYPE_Q4_K || T == 1) return 1;
  return tokens_per_active_expert(m, T) < 8.0 ? 2 : 4;
}

// Routed and shared gate/up in one tensor-core launch.
template <int DT>
cudaError_t launch_up_mma(const MoeDevice& m, const MoeWork& w, int T, const SlabMaps* cached,
                          cudaStream_t s) {
  SlabMaps local;
  if (!cached) {
    const cudaError_t e = moe_maps_build(m, &local);
    if (e != cudaSuccess) return e;
    cached = &local;
  }
  const SlabMaps& mp = *cached;
  if (!mp.ready) return cudaSuccess;  // nothing owned here
  switch (up_pass_tokens(m, T)) {
    case 1:
      return launch_up_slab_nt<1, DT>(m, w, T, mp, s);
    case 2:
      return launch_up_slab_nt<2, DT>(m, w, T, mp, s);
    default:
      return launch_up_slab_nt<4, DT>(m, w, T, mp, s);
  }
}

}  // namespace

cudaError_t moe_maps_build(const MoeDevice& m_in, SlabMaps* out) {
  // a latent layer's gate/up matrices are those of its routed sub-layer
  const MoeDevice m = m_in.latent_dim > 0 ? latent_routed_view(m_in) : m_in;
  SlabMaps& mp = *out;
  mp.ready = 0;
  if (m.up_type != LB_TYPE_Q4_K) return cudaSuccess;
  const bool pair = m.arch == 0;
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
  mp.ready = 1;
  return cudaSuccess;
}

namespace {

template <int UT, int DT>
cudaError_t launch_expert_passes(const MoeDevice& m, const MoeWork& w, int T,
                                 const SlabMaps* maps, cudaStream_t s, const cudaEvent_t* marks) {
  cudaError_t e;
  auto mark = [&](int i) { return marks ? cudaEventRecord(marks[i], s) : cudaSuccess; };
  if ((e = mark(0)) != cudaSuccess) return e;
  if constexpr (UT == LB_TYPE_Q4_K) {
    e = launch_up_mma<DT>(m, w, T, maps, s);
  } else {
    e = launch_up<UT, DT>(m, w, T, 0, s);
    if (e == cudaSuccess && m.shared_here && m.inter_sh) e = launch_up<UT, DT>(m, w, T, 1, s);
  }
  if (e != cudaSuccess || (e = mark(1)) != cudaSuccess) return e;
  if (DT == LB_TYPE_Q4_K) {
    moe_down_sums_kernel<<<std::min(T * m.top_k + T, sm_count() * 4), 128, 0, s>>>(m, w, T);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (DT == LB_TYPE_Q6_K && down_uses_i6(m)) {
    // When this device computes the shared expert for a few tokens only
    // (expert-parallel ranks, or small batches), its down slabs ride in the
    // routed launch: one launch less on the layer's critical path (decode
    // batch 1 on one B200: 469 -> 515 tokens/s).  For larger batches on one
    // device its own launch overlaps the routed tail better (measured at 32
    // tokens), so it stays apart there.
    const bool ride = (m.ep_world > 1 || T <= 8) && m.shared_here && m.inter_sh &&
                      m.k_down_sh == m.k_down && m.down_sh_rb == m.down_rb;
    e = launch_down_slab(m, w, T, ride ? 2 : 0, s);
    if (e == cudaSuccess) e = mark(2);
    if (e == cudaSuccess && !ride && m.shared_here && m.inter_sh)
      e = launch_down_slab(m, w, T, 1, s);
    return e;
  }
  e = launch_down<DT>(m, w, T, 0, s);
  if (e == cudaSuccess) e = mark(2);
  if (e == cudaSuccess && m.shared_here && m.inter_sh) e = launch_down<DT>(m, w, T, 1, s);
  return e;
}

}  // namespace

size_t moe_work_bytes(const MoeDevice& m, int T) {
  MoeWork w;
  moe_work_carve(m, T, nullptr, &w);
  return w.bytes;
}

MoeDevice latent_routed_view(const MoeDevice& m) {
  MoeDevice r = m;
  r.hidden = m.latent_dim;
  r.latent_dim = 0;
  r.input_norm = nullptr;
  r.add_residual = 0;
  r.shared_here = 0;
  r.inter_sh = 0;
  r.router_rows = 0;
  r.router_extra_row = nullptr;
  r.logits_ready = 1;
  r.ep_world = 0;
  r.ep_peers = nullptr;
  return r;
}

void moe_work_carve(const MoeDevice& m, int T, void* base, MoeWork* w) {
  if (m.latent_dim > 0) {
    // the routed sub-layer's buffers first, then the latent path's own
    const MoeDevice r = latent_routed_view(m);
    moe_work_carve(r, T, base, w);
    size_t off = w->bytes;
    auto take = [&](size_t bytes) {
      size_t o = off;
      off += (bytes + 255) & ~size_t(255);
      return base ? reinterpret_cast<float*>(static_cast<char*>(base) + o) : nullptr;
    };
    const size_t H = m.hidden, L = m.latent_dim, Ish = m.shared_here ? m.inter_sh : 0;
    w->lat_xr = take(m.input_norm ? (size_t)T * H * 4 : 4);
    w->lat_x = take((size_t)T * L * 4);
    w->lat_y = take((size_t)T * L * 4);
    w->lat_u = take((size_t)T * H * 4);
    w->lat_s1 = take(std::max<size_t>((size_t)T * Ish * 4, 4));
    w->lat_s2 = take(std::max<size_t>((size_t)T * (Ish ? H : 1) * 4, 4));
    size_t xp = 1;
    auto kq = [](int t) { return t == LB_TYPE_Q4_K || t == LB_TYPE_Q6_K; };
    if (kq(m.lat_down_type)) xp = std::max(xp, xprep_floats(m.k_lat_down, T));
    if (kq(m.lat_up_type)) xp = std::max(xp, xprep_floats(m.k_lat_up, T));
    if (Ish && kq(m.up_sh_type)) xp = std::max(xp, xprep_floats(m.k_in_sh, T));
    if (Ish && kq(m.down_sh_type)) xp = std::max(xp, xprep_floats(m.k_down_sh, T));
    w->lat_xp = take(xp * 4);
    w->bytes = off;
    return;
  }
  const int E = m.experts, k = m.top_k;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return base ? static_cast<char*>(base) + o : nullptr;
  };
  w->lat_xr = w->lat_x = w->lat_y = w->lat_u = w->lat_s1 = w->lat_s2 = w->lat_xp = nullptr;
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
  w->pass_off_dn = reinterpret_cast<int*>(take((size_t)(E + 1) * 4));
  w->status = reinterpret_cast<int*>(take(8));  // the status word, then the ticket
  w->tickets = w->status ? w->status + 1 : nullptr;
  w->xn = reinterpret_cast<float*>(take(m.input_norm ? (size_t)T * m.hidden * 4 : 4));
  w->xp_up = reinterpret_cast<float*>(take((size_t)T * up_ld_floats(m.k_in) * 4));
  w->xp_down = reinterpret_cast<float*>(
      take((size_t)(T * k + T) * down_ld_floats(m) * 4));
  w->partial = reinterpret_cast<float*>(take((size_t)T * (k + 1) * m.hidden * 4));
  // K-split gate/up items (decode): per item its slices' row sums, and an
  // arrival ticket per item (zero between launches)
  w->up_part = reinterpret_cast<float*>(
      take((size_t)kUpSplitItems * kUpMaxSplit * kUpPartFloats * 4));
  w->up_tickets = reinterpret_cast<int*>(take((size_t)kUpSplitItems * 4));
  size_t pf[6];
  if (prefill_work_bytes(m, T, pf)) {
    w->pf_xs = reinterpret_cast<uint16_t*>(take(pf[0]));
    w->pf_hs = reinterpret_cast<uint16_t*>(take(pf[1]));
    w->pf_prow = reinterpret_cast<int*>(take(pf[2]));
    w->pf_tiles = reinterpret_cast<int4*>(take(pf[3]));
    w->pf_count = reinterpret_cast<int*>(take(pf[4]));
    w->pf_rlog = reinterpret_cast<float*>(take(pf[5]));
    w->pf_max_up = prefill_max_up_tiles(m, T);
  } else {
    w->pf_xs = w->pf_hs = nullptr;
    w->pf_prow = w->pf_count = nullptr;
    w->pf_tiles = nullptr;
    w->pf_rlog = nullptr;
    w->pf_max_up = 0;
  }
  w->bytes = off;
}

namespace {

// rms-norm-into (llambda.lisp L859-879) of each token (one CTA per token):
// scale = 1 / sqrt(mean(x^2) + eps), dest = (x * weight) * scale.
__global__ void __launch_bounds__(256) latent_norm_kernel(MoeDevice m, const float* __restrict__ x,
                                                          float* __restrict__ xn) {
  __shared__ float s_part[8];
  const int H = m.hidden;
  const float* xt = x + (long)blockIdx.x * H;
  float acc = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) acc = fmaf(xt[i], xt[i], acc);
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = acc;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += s_part[i];
  const float scale =
      __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)H), m.norm_epsilon)));
  for (int i = threadIdx.x; i < H; i += blockDim.x)
    xn[(long)blockIdx.x * H + i] = __fmul_rn(__fmul_rn(xt[i], m.input_norm[i]), scale);
}

// apply-relu-squared-into (L938-940, L945-979) in place.
__global__ void relu_sq_kernel(float* __restrict__ v, long n) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    v[i] = relu_sq_ref(v[i]);
}

// dest = latent_up . moe-output (L5933-5938), plus the shared expert's down
// output (vector-add-bias-in-place, L5949), plus x when the layer carries
// the residual (vector-add-into, L5746): out = x + (lu + sh).
__global__ void latent_out_kernel(const float* __restrict__ x, const float* __restrict__ lu,
                                  const float* __restrict__ sh, float* __restrict__ out, long n,
                                  int residual) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
       i += (long)gridDim.x * blockDim.x) {
    float v = lu[i];
    if (sh) v = __fadd_rn(v, sh[i]);
    out[i] = residual ? __fadd_rn(x[i], v) : v;
  }
}

cudaError_t launch_moe_latent(const MoeDevice& m, const MoeWork& w, const float* x, int T,
                              float* out, const SlabMaps* maps, cudaStream_t s,
                              const cudaEvent_t* marks) {
  const int H = m.hidden, L = m.latent_dim, E = m.experts;
  cudaError_t e;
  const float* xr = x;
  if (m.input_norm) {
    latent_norm_kernel<<<T, 256, 0, s>>>(m, x, w.lat_xr);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    xr = w.lat_xr;
  }
  // the router sees x itself (L5889-5892); its logits feed the routed sub-layer
  e = launch_gemv_f32(m.router, E, H, xr, H, T, w.logits, E + 1, s);
  if (e != cudaSuccess) return e;
  e = launch_projection(m.lat_down_type, m.lat_down, m.lat_down_rb, L, m.k_lat_down, xr, H, H, T,
                        w.lat_x, L, w.lat_xp, w.status, s);
  if (e != cudaSuccess) return e;
  const MoeDevice r = latent_routed_view(m);
  if ((e = launch_moe(r, w, w.lat_x, T, w.lat_y, maps, s, marks)) != cudaSuccess) return e;
  e = launch_projection(m.lat_up_type, m.lat_up, m.lat_up_rb, H, m.k_lat_up, w.lat_y, L, L, T,
                        w.lat_u, H, w.lat_xp, w.status, s);
  if (e != cudaSuccess) return e;
  const bool shared = m.shared_here && m.inter_sh;
  if (shared) {  // the shared expert on x (L5939-5949)
    const int I = m.inter_sh;
    e = launch_projection(m.up_sh_type, m.up_sh, m.up_sh_rb, I, m.k_in_sh, xr, H, H, T, w.lat_s1,
                          I, w.lat_xp, w.status, s);
    if (e != cudaSuccess) return e;
    const long n = (long)T * I;
    relu_sq_kernel<<<(int)std::min<long>((n + 255) / 256, sm_count() * 8L), 256, 0, s>>>(w.lat_s1, n);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    e = launch_projection(m.down_sh_type, m.down_sh, m.down_sh_rb, H, m.k_down_sh, w.lat_s1, I, I,
                          T, w.lat_s2, H, w.lat_xp, w.status, s);
    if (e != cudaSuccess) return e;
  }
  const long n = (long)T * H;
  latent_out_kernel<<<(int)std::min<long>((n + 255) / 256, sm_count() * 8L), 256, 0, s>>>(
      x, w.lat_u, shared ? w.lat_s2 : nullptr, out, n, m.add_residual);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_moe(const MoeDevice& m, const MoeWork& w, const float* x, int T, float* out,
                       const SlabMaps* maps, cudaStream_t s, const cudaEvent_t* marks) {
  if (T <= 0) return cudaSuccess;
  if (m.latent_dim > 0) {
    if (T > w.max_tokens || m.arch != 1 || m.ep_world > 1 || m.dx_world > 1)
      return cudaErrorInvalidValue;
    return launch_moe_latent(m, w, x, T, out, maps, s, marks);
  }
  if (m.dx_world > 1) {  // token dispatch across ranks for prefill batches
    if (T >= prefill_min_tokens()) return launch_moe_dispatch(m, w, x, T, out, s, marks);
    // smaller calls hold the tokens of every rank and need the peer reduction
    if (m.ep_world <= 1) return cudaErrorInvalidValue;
  }
  if (T > w.max_tokens || m.experts > kMaxExperts || m.top_k > 32 || T * m.top_k > kMaxEntries)
    return cudaErrorInvalidValue;
  if (m.inter_sh && m.k_in_sh != m.k_in) return cudaErrorInvalidValue;
  const int E = m.experts;
  cudaError_t e;
  // the router's CTA tile: 8 tokens, or 4 where 8 do not fit beside the rows
  const size_t router_smem8 = (size_t)(8 + kRouterRows) * m.hidden * sizeof(float);
  const int router_tok = router_smem8 <= 192 * 1024 ? 8 : 4;
  const size_t router_smem = (size_t)(router_tok + kRouterRows) * m.hidden * sizeof(float);
  auto router_kern = router_tok == 8 ? moe_router_kernel<8> : moe_router_kernel<4>;
  const uintptr_t align =
      reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(m.router) |
      reinterpret_cast<uintptr_t>(m.router_extra_row) | reinterpret_cast<uintptr_t>(m.input_norm);
  const int all_rows = m.router_rows + (m.router_extra_row ? 1 : 0);  // column E: shared gate
  const bool prefill = prefill_applies(m, w, T);
  auto mark = [&](int i) { return marks ? cudaEventRecord(marks[i], s) : cudaSuccess; };
  if ((e = mark(3)) != cudaSuccess) return e;
  if (m.logits_ready) {  // the routed sub-layer of a latent layer: no router
    if (!prefill) {
      if (m.up_type == LB_TYPE_Q4_K)
        moe_prep_kernel<LB_TYPE_Q4_K><<<T, 256, 0, s>>>(m, w, x);
      else
        moe_prep_kernel<LB_TYPE_Q6_K><<<T, 256, 0, s>>>(m, w, x);
      if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
  } else if (prefill) {
    if ((e = launch_prefill_router(m, w, x, T, s)) != cudaSuccess) return e;
  } else if (m.up_type == LB_TYPE_Q4_K && (m.hidden & 3) == 0 && (align & 15) == 0 &&
      router_smem <= 224 * 1024 &&
      prepared_occupancy(router_kern, kRouterWarps * 32, router_smem) >= 1) {
    dim3 grid((all_rows + kRouterRows - 1) / kRouterRows, (T + router_tok - 1) / router_tok);
    e = launch_pdl(router_kern, grid, dim3(kRouterWarps * 32), router_smem, s, m, w, x, T,
                   all_rows);
    if (e != cudaSuccess) return e;
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  } else {
    if (m.up_type == LB_TYPE_Q4_K)
      moe_prep_kernel<LB_TYPE_Q4_K><<<T, 256, 0, s>>>(m, w, x);
    else
      moe_prep_kernel<LB_TYPE_Q6_K><<<T, 256, 0, s>>>(m, w, x);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const float* xr = m.input_norm ? w.xn : x;
    if (m.arch == 0 && m.router_extra_row) {  // shared-expert gate logit into column E
      e = launch_gemv_f32(m.router_extra_row, 1, m.hidden, xr, m.hidden, T, w.logits + E, E + 1,
                          s);
      if (e != cudaSuccess) return e;
    }
    e = launch_gemv_f32(m.router, m.router_rows, m.hidden, xr, m.hidden, T, w.logits, E + 1, s);
    if (e != cudaSuccess) return e;
  }
  if ((e = mark(6)) != cudaSuccess) return e;
  // top-k per token, the routing on the last CTA
  if ((e = launch_topk(m, w, T, prefill ? 0 : 1, s)) != cudaSuccess) return e;
  const bool gate_ok = m.arch == 1 || m.gate_type == m.up_type;
  if (!gate_ok) return cudaErrorInvalidValue;
  if (prefill)
    e = launch_prefill_passes(m, w, x, T, s, marks);
  else if (m.up_type == LB_TYPE_Q4_K && m.down_type == LB_TYPE_Q6_K)
    e = launch_expert_passes<LB_TYPE_Q4_K, LB_TYPE_Q6_K>(m, w, T, maps, s, marks);
  else if (m.up_type == LB_TYPE_Q4_K && m.down_type == LB_TYPE_Q4_K)
    e = launch_expert_passes<LB_TYPE_Q4_K, LB_TYPE_Q4_K>(m, w, T, maps, s, marks);
  else if (m.up_type == LB_TYPE_Q6_K && m.down_type == LB_TYPE_Q6_K)
    e = launch_expert_passes<LB_TYPE_Q6_K, LB_TYPE_Q6_K>(m, w, T, maps, s, marks);
  else if (m.up_type == LB_TYPE_Q6_K && m.down_type == LB_TYPE_Q4_K)
    e = launch_expert_passes<LB_TYPE_Q6_K, LB_TYPE_Q4_K>(m, w, T, maps, s, marks);
  else
    return cudaErrorInvalidValue;
  if (e != cudaSuccess || (e = mark(4)) != cudaSuccess) return e;
  const bool vec = (m.hidden & 3) == 0 &&
                   ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  if (m.ep_world > 1) {  // every rank's partial meets here (peer memory, NVLink)
    if (!vec || T > m.ep_max_tokens) return cudaErrorInvalidValue;
    e = launch_pdl(combine_ep_kernel, dim3(kEpGrid), dim3(256), 0, s, m, w, T, x, out);
  } else {
    e = launch_combine(m, w, T, x, out, s);
  }
  return e != cudaSuccess ? e : mark(5);
}

cudaError_t launch_topk(const MoeDevice& m, const MoeWork& w, int T, int grouped_ids,
                        cudaStream_t s) {
  const int per = (m.experts + 31) / 32, pnt = up_pass_tokens(m, T);
  const int pdn = down_pass_tokens(m, T, 0);  // the routed down passes
  if (T <= kTopkSmallTokens && per <= 16) {
    auto small = per <= 1 ? topk_route_small_kernel<1> : per <= 2 ? topk_route_small_kernel<2>
               : per <= 4 ? topk_route_small_kernel<4> : per <= 8 ? topk_route_small_kernel<8>
               : topk_route_small_kernel<16>;
    cudaError_t e = launch_pdl(small, dim3(1), dim3(32 * kTopkSmallTokens), 0, s, m, w, T, pnt,
                               pdn, grouped_ids);
    return e != cudaSuccess ? e : cudaGetLastError();
  }
  if (grouped_ids == 0) {  // prefill: positions by atomic counts, no stable walk
    cudaError_t e = cudaMemsetAsync(w.counts, 0, (size_t)m.experts * sizeof(int), s);
    if (e != cudaSuccess) return e;
    auto cnt = per <= 1 ? topk_count_kernel<1> : per <= 2 ? topk_count_kernel<2>
             : per <= 4 ? topk_count_kernel<4> : per <= 8 ? topk_count_kernel<8>
             : per <= 16 ? topk_count_kernel<16> : topk_count_kernel<32>;
    e = launch_pdl(cnt, dim3((T + kTopkTokens - 1) / kTopkTokens), dim3(256), 0, s, m, w, T, pnt,
                   pdn);
    return e != cudaSuccess ? e : cudaGetLastError();
  }
  auto kern = per <= 1 ? topk_route_kernel<1> : per <= 2 ? topk_route_kernel<2>
            : per <= 4 ? topk_route_kernel<4> : per <= 8 ? topk_route_kernel<8>
            : per <= 16 ? topk_route_kernel<16> : topk_route_kernel<32>;
  cudaError_t e = launch_pdl(kern, dim3((T + kTopkTokens - 1) / kTopkTokens), dim3(256), 0, s, m,
                             w, T, pnt, pdn, grouped_ids);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_combine(const MoeDevice& m, const MoeWork& w, int T, const float* x, float* out,
                           cudaStream_t s) {
  const bool vec = (m.hidden & 3) == 0 &&
                   ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  const long n = (long)T * m.hidden / (vec ? 4 : 1);
  const int grid = std::max(1, (int)std::min<long>((n + 127) / 128, (long)sm_count() * 16));
  auto kern = vec && m.top_k <= 16 ? combine_kernel<true, 16>
              : vec ? combine_kernel<true, 32> : combine_kernel<false, 32>;
  return launch_pdl(kern, dim3(grid), dim3(128), 0, s, m, w, T, x, out);
}

}  // namespace lb
