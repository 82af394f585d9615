// er_plan.cu -- K2: group the routed (token, slot) pairs by expert.
//
// Reference: runtime/qwen_moe.py:341-344. The reference loops over
// np.unique(selected) (ascending expert id) and, per expert, takes
// np.nonzero(selected == e): the (token, slot) pairs in row-major order.
// This kernel produces the same grouping as one expert-sorted array: the
// pairs of expert 0 first, then expert 1, ..., each expert's pairs in
// row-major (token, slot) order. It also lays out the work items of the
// grouped expert kernels over the active experts (and the shared expert).
#include "er_internal.cuh"

namespace er {

constexpr int kPlanThreads = 1024;
constexpr int kPlanWarps = kPlanThreads / 32;

// One CTA. Warp w owns the contiguous entries [w * span, (w + 1) * span) of the
// row-major (token, slot) list. (1) each warp counts its entries per expert;
// (2) per expert, an exclusive prefix over the warps; per-expert offsets and
// the work-item schedules; (3) each warp walks its entries again and places
// entry i at offsets[e] + (entries of e in earlier warps) + (earlier entries
// of e in this warp): the same stable order as np.nonzero per expert.
__global__ void __launch_bounds__(kPlanThreads) plan_kernel(const int32_t* __restrict__ idx,
                                                            const float* __restrict__ w, int n, int k, int E,
                                                            int H, int I, int Is, SchedSpec s0, SchedSpec s1,
                                                            Plan* __restrict__ plan,
                                                            int32_t* __restrict__ perm_token,
                                                            float* __restrict__ perm_w,
                                                            int32_t* __restrict__ pos_of) {
  __shared__ int cnt[kPlanWarps][kMaxExperts];  // per-warp counts, then running bases
  __shared__ int hist[kMaxExperts];
  __shared__ int base[kMaxExperts];
  __shared__ int act[kMaxExperts + 1];
  __shared__ int bad;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nk = n * k;
  const int span = (nk + kPlanWarps * 32 - 1) / (kPlanWarps * 32) * 32;
  const int beg = warp * span, end = min(nk, beg + span);
  for (int i = tid; i < kPlanWarps * kMaxExperts; i += kPlanThreads) cnt[i / kMaxExperts][i % kMaxExperts] = 0;
  if (tid == 0) bad = 0;
  __syncthreads();
  // the warp's entries are fetched kBatch rows of 32 at a time with independent
  // loads, so a batch costs one memory round trip
  constexpr int kBatch = 16;
  for (int b0 = beg; b0 < end; b0 += 32 * kBatch) {
    int ev[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int i = b0 + 32 * j + lane;
      ev[j] = i < end ? __ldg(idx + i) : -1;
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int i = b0 + 32 * j + lane;
      int e = ev[j];
      if (i < end && (e < 0 || e >= E)) {
        bad = 1;
        e = -1;
      }
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      if (e >= 0 && (__ffs(peers) - 1) == lane) cnt[warp][e] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();
  for (int e = tid; e < E; e += kPlanThreads) {
    int run = 0;
    for (int w2 = 0; w2 < kPlanWarps; ++w2) {
      const int c = cnt[w2][e];
      cnt[w2][e] = run;
      run += c;
    }
    hist[e] = run;
  }
  __syncthreads();
  if (warp == 0) {
    // Warp 0 builds the offsets, the active list and the schedules with
    // warp scans (lane l owns entries 9l .. 9l+8, enough for E + 2 <= 258).
    constexpr int kPer = 9;
    auto warp_excl_scan = [&](int v) {  // exclusive prefix of v over the lanes; also returns the total
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      return incl - v;
    };
    int sum = 0, nact = 0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int e = lane * kPer + j;
      if (e < E) {
        sum += hist[e];
        nact += hist[e] > 0;
      }
    }
    int off = warp_excl_scan(sum), pos = warp_excl_scan(nact);
    const int na_routed = __shfl_sync(0xffffffffu, pos + nact, 31);
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int e = lane * kPer + j;
      if (e < E) {
        base[e] = off;
        off += hist[e];
        if (hist[e] > 0) act[pos++] = e;
      }
    }
    const int na = na_routed + (n > 0 ? 1 : 0);
    if (lane == 0 && n > 0) act[na_routed] = E;
    __syncwarp();
    for (int a = lane; a < na; a += 32) plan->active[a] = act[a];
    const SchedSpec specs[kNumSched] = {s0, s1};
#pragma unroll
    for (int s = 0; s < kNumSched; ++s) {
      const SchedSpec sp = specs[s];
      int items[kPer], local = 0;
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int a = lane * kPer + j;
        items[j] = 0;
        if (a < na) {
          const int g = act[a];
          const int rows = g == E ? n : hist[g];
          const int units = sp.which == 0 ? (g == E ? Is : I) : H;
          const int mt = sp.bm > 0 ? (rows + sp.bm - 1) / sp.bm : 1;
          items[j] = mt * ((units + sp.bn - 1) / sp.bn);
        }
        local += items[j];
      }
      int start_a = warp_excl_scan(local);
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int a = lane * kPer + j;
        if (a <= na) plan->item_start[s][a] = bad ? 0 : start_a;
        start_a += items[j];
      }
    }
    if (lane == 0) {
      plan->n = n;
      plan->E = E;
      plan->k = k;
      plan->nk = nk;
      plan->error = bad;
      plan->sched[0] = s0;
      plan->sched[1] = s1;
      // no work items at all when an expert id was out of range: nothing
      // downstream may read the unfilled permutation
      plan->num_active = bad ? 0 : na;
    }
  }
  __syncthreads();
  for (int e = tid; e <= E; e += kPlanThreads) {
    plan->counts[e] = e < E ? hist[e] : n;
    plan->offsets[e] = e < E ? base[e] : 0;
  }
  if (bad) return;
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int b0 = beg; b0 < end; b0 += 32 * kBatch) {
    int ev[kBatch];
    float wv[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int i = b0 + 32 * j + lane;
      ev[j] = i < end ? __ldg(idx + i) : -1;
      wv[j] = i < end ? __ldg(w + i) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int i = b0 + 32 * j + lane;
      const int e = ev[j];
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      int p = 0;
      if (e >= 0) p = base[e] + cnt[warp][e] + __popc(peers & lt_mask);
      __syncwarp();
      if (e >= 0 && (__ffs(peers) - 1) == lane) cnt[warp][e] += __popc(peers);
      __syncwarp();
      if (e >= 0) {
        perm_token[p] = i / k;
        perm_w[p] = wv[j];
        pos_of[i] = p;
      }
    }
  }
}

long long sched_items_bound(const SchedSpec& s, int n, int k, int E, int H, int I, int Is) {
  const long long nk = (long long)n * k;
  const long long active = nk < E ? nk : E;  // routed groups with at least one token
  long long routed_rows_tiles, shared_tiles;
  if (s.bm > 0) {
    routed_rows_tiles = (nk + s.bm - 1) / s.bm + active;  // sum over groups of ceil(rows / bm)
    shared_tiles = (n + s.bm - 1) / s.bm;
  } else {
    routed_rows_tiles = active;
    shared_tiles = n > 0 ? 1 : 0;
  }
  const long long nt_r = s.which == 0 ? (I + s.bn - 1) / s.bn : (H + s.bn - 1) / s.bn;
  const long long nt_s = s.which == 0 ? (Is + s.bn - 1) / s.bn : (H + s.bn - 1) / s.bn;
  return routed_rows_tiles * nt_r + shared_tiles * nt_s;
}

int launch_plan(const int32_t* idx, const float* w, int n, int k, int E, int H, int I, int Is,
                const SchedSpec* specs, Plan* plan, int32_t* perm_token, float* perm_w, int32_t* pos_of,
                cudaStream_t st) {
  plan_kernel<<<1, kPlanThreads, 0, st>>>(idx, w, n, k, E, H, I, Is, specs[0], specs[1], plan, perm_token, perm_w,
                                          pos_of);
  return launch_check("plan_kernel");
}

}  // namespace er
