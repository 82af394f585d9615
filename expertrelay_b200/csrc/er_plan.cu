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

__global__ void __launch_bounds__(kPlanThreads) plan_kernel(const int32_t* __restrict__ idx,
                                                            const float* __restrict__ w, int n, int k, int E,
                                                            int H, int I, int Is, SchedSpec s0, SchedSpec s1,
                                                            Plan* __restrict__ plan,
                                                            int32_t* __restrict__ perm_token,
                                                            float* __restrict__ perm_w,
                                                            int32_t* __restrict__ pos_of) {
  __shared__ int hist[kMaxExperts];
  __shared__ int base[kMaxExperts];
  __shared__ int chunk_total[kMaxExperts];
  __shared__ int wcount[kPlanThreads / 32][kMaxExperts];
  __shared__ int bad;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nk = n * k;
  for (int e = tid; e < kMaxExperts; e += kPlanThreads) hist[e] = 0;
  if (tid == 0) bad = 0;
  __syncthreads();
  // warp-aggregated histogram: one shared-memory atomic per distinct expert per warp
  for (int i0 = 0; i0 < nk; i0 += kPlanThreads) {
    const int i = i0 + tid;
    int e = i < nk ? idx[i] : -1;
    if (i < nk && (e < 0 || e >= E)) {
      bad = 1;
      e = -1;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0 && (__ffs(peers) - 1) == lane) atomicAdd(&hist[e], __popc(peers));
  }
  __syncthreads();
  if (tid == 0) {
    plan->n = n;
    plan->E = E;
    plan->k = k;
    plan->nk = nk;
    plan->error = bad;
    plan->sched[0] = s0;
    plan->sched[1] = s1;
    int off = 0, na = 0;
    for (int e = 0; e < E; ++e) {
      plan->counts[e] = hist[e];
      plan->offsets[e] = off;
      base[e] = off;
      off += hist[e];
      if (hist[e] > 0) plan->active[na++] = e;
    }
    plan->counts[E] = n;
    plan->offsets[E] = 0;
    if (n > 0) plan->active[na++] = E;
    plan->num_active = na;
    const SchedSpec specs[kNumSched] = {s0, s1};
    for (int s = 0; s < kNumSched; ++s) {
      const SchedSpec sp = specs[s];
      int acc = 0;
      for (int a = 0; a < na; ++a) {
        plan->item_start[s][a] = acc;
        const int g = plan->active[a];
        const int rows = plan->counts[g];
        const int units = sp.which == 0 ? (g == E ? Is : I) : H;
        const int mt = sp.bm > 0 ? (rows + sp.bm - 1) / sp.bm : 1;
        const int nt = (units + sp.bn - 1) / sp.bn;
        acc += mt * nt;
      }
      plan->item_start[s][na] = acc;
    }
    if (bad) {  // no work items: nothing downstream may read the unfilled permutation
      plan->num_active = 0;
      for (int s = 0; s < kNumSched; ++s) plan->item_start[s][0] = 0;
    }
  }
  __syncthreads();
  if (bad) return;
  // stable expert-sorted positions, one chunk of kPlanThreads pairs at a time
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int c0 = 0; c0 < nk; c0 += kPlanThreads) {
    const int i = c0 + tid;
    const int e = (i < nk) ? idx[i] : -1;
    for (int x = lane; x < E; x += 32) wcount[warp][x] = 0;
    __syncthreads();
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & lt_mask);
    if (e >= 0 && rank == 0) wcount[warp][e] = __popc(peers);
    __syncthreads();
    for (int x = tid; x < E; x += kPlanThreads) {  // exclusive prefix over warps
      int run = 0;
      for (int w2 = 0; w2 < kPlanThreads / 32; ++w2) {
        const int c = wcount[w2][x];
        wcount[w2][x] = run;
        run += c;
      }
      chunk_total[x] = run;
    }
    __syncthreads();
    if (e >= 0) {
      const int p = base[e] + wcount[warp][e] + rank;
      perm_token[p] = i / k;
      perm_w[p] = w[i];
      pos_of[i] = p;
    }
    __syncthreads();
    for (int x = tid; x < E; x += kPlanThreads) base[x] += chunk_total[x];
    __syncthreads();
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
