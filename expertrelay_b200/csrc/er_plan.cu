// er_plan.cu -- K2: group the routed (token, slot) pairs by expert.
//
// Reference: runtime/qwen_moe.py:341-344. The reference loops over
// np.unique(selected) (ascending expert id) and, per expert, takes
// np.nonzero(selected == e): the (token, slot) pairs routed to it. Here the
// pairs of each expert occupy one contiguous range of an expert-sorted array
// (expert 0's range first), laid out in two launches:
//   per-expert counts, tallied by the top-k kernel (or tally_kernel) ->
//   dispatch_kernel: each CTA derives the experts' ranges from the counts
//                   (CTA 0 also writes the active groups and the work-item
//                   schedules); one warp per token claims a position in each
//                   of its k experts' ranges (an atomic count per expert) and,
//                   for the tensor-core path, slices the token's h row once
//                   into the int8 operand rows of those positions and of the
//                   shared expert's row nk + t.
// The order of the pairs inside one expert's range follows the atomics, not
// the token order; nothing downstream depends on it: every output element is
// computed from its own token's row alone, and the combine sums each token's
// slots in ascending expert id through pos_of.
#include "er_select.cuh"

namespace er {

// Exclusive prefix of v over the CTA (every thread calls; `tmp` holds one
// int per warp); *total receives the sum over the CTA.
__device__ __forceinline__ int cta_excl_scan(int v, int* tmp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) tmp[warp] = incl;
  __syncthreads();
  int base = 0, tot = 0;
  for (int w = 0; w < nw; ++w) {
    const int x = tmp[w];
    base += w < warp ? x : 0;
    tot += x;
  }
  __syncthreads();  // tmp is reused by the next scan
  *total = tot;
  return base + incl - v;
}

// The record addresses thread `tid` hands plan_scan (experts 2 tid, 2 tid + 1;
// zero unless this CTA writes the plan), loaded at a kernel's start so their
// latency hides behind its other work.
__device__ __forceinline__ void plan_records(const uint64_t* records, bool write_plan, int E, uint64_t& r0,
                                             uint64_t& r1) {
  const int e = 2 * (int)threadIdx.x;
  r0 = (write_plan && records && e < E) ? records[e] : 0ull;
  r1 = (write_plan && records && e + 1 < E) ? records[e + 1] : 0ull;
}

// The plan from the per-expert tallies, by the whole CTA (at least 256
// threads; thread i owns entries 2i, 2i+1 of the per-expert and per-group
// lists, enough for E + 2 <= 258). Every caller gets the expert ranges' first
// positions in `offs` (shared memory) and whether the tallies are consistent;
// with write_plan it also writes the plan's groups, ranges and work-item
// schedules for the expert kernels. Ends with a __syncthreads.
__device__ void plan_scan(Plan* __restrict__ plan, int n, int k, int E, int H, int I, int Is, SchedSpec s0,
                          SchedSpec s1, int shared, bool write_plan, int* hist, int* offs, int* act, int* bad_out,
                          int* tmp, const int* tally = nullptr, uint64_t rec0 = 0ull, uint64_t rec1 = 0ull) {
  const int tid = threadIdx.x;
  const int nk = n * k;
  int cnt[2], on[2];
  // rec0 / rec1: the record addresses of experts 2 tid and 2 tid + 1 (loaded
  // by the caller early, see plan_records), copied into the plan by active position
  const uint64_t rec[2] = {rec0, rec1};
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int e = 2 * tid + j;
    cnt[j] = e < E ? (tally ? tally[e] : __ldcg(&plan->tally[e])) : 0;  // plan->tally: counted at L2 by atomics
    on[j] = cnt[j] > 0;
    if (e < E) hist[e] = cnt[j];
  }
  int total, na_routed;
  // the shared expert, when it runs, is the first active group: its work
  // items come first in every schedule (decode launches prefetch its weights
  // before the routing is known)
  const int first = (shared && n > 0) ? 1 : 0;
  int off = cta_excl_scan(cnt[0] + cnt[1], tmp, &total);
  int pos = cta_excl_scan(on[0] + on[1], tmp, &na_routed) + first;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int e = 2 * tid + j;
    if (e < E) {
      offs[e] = off;
      if (write_plan) {
        plan->counts[e] = cnt[j];
        plan->offsets[e] = off;
        if (on[j]) {
          plan->act_rows[pos] = cnt[j];
          plan->act_off[pos] = off;
          plan->act_rec[pos] = rec[j];
        }
      }
      off += cnt[j];
      if (on[j]) act[pos++] = e;
    }
  }
  // every pair lands in some expert's range: the counts must add up to n * k
  const bool bad = total != nk;
  if (tid == 0) *bad_out = bad;
  if (!write_plan) {
    __syncthreads();
    return;
  }
  const int na = na_routed + first;
  if (tid == 0) {
    if (first) {
      act[0] = E;
      plan->act_rows[0] = n;
      plan->act_off[0] = 0;
      plan->act_rec[0] = 0ull;
    }
    plan->counts[E] = n;
    plan->offsets[E] = 0;
  }
  __syncthreads();
  for (int a = tid; a < na; a += blockDim.x) plan->active[a] = act[a];
#pragma unroll 1
  for (int s = 0; s < kNumSched; ++s) {
    const SchedSpec sp = s == 0 ? s0 : s1;
    int items[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int a = 2 * tid + j;
      items[j] = 0;
      if (a < na) {
        const int g = act[a];
        const int rows = g == E ? n : hist[g];
        const int units = sp.which == 0 ? (g == E ? Is : I) : H;
        const int mt = sp.bm > 0 ? (rows + sp.bm - 1) / sp.bm : 1;
        const int parts = (g == E && sp.which == 1 && sp.ks > 1) ? sp.ks : 1;
        items[j] = mt * ((units + sp.bn - 1) / sp.bn) * parts;
      }
    }
    int sum;
    int start = cta_excl_scan(items[0] + items[1], tmp, &sum);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int a = 2 * tid + j;
      if (a <= na) plan->item_start[s][a] = bad ? 0 : start;
      start += items[j];
    }
  }
  if (tid == 0) {
    plan->n = n;
    plan->E = E;
    plan->k = k;
    plan->nk = nk;
    if (bad) atomicOr(&plan->error, 2);
    plan->sched[0] = s0;
    plan->sched[1] = s1;
    plan->num_active = bad ? 0 : na;  // no work items on an inconsistent tally
  }
  __syncthreads();
}

// One token per warp, 8 per CTA. With SLICE and rows of up to 2048
// values, each warp first slices its token's h row (K = H values) into two
// int8 words per lane and step, held in registers; the CTA then derives the
// expert ranges from the tallies (CTA 0 also writes the plan). Then lane r < k
// of a token's warp claims the position of slot r (its expert's range start,
// plus the CTA's block of it, plus the pair's rank inside the CTA) and the
// warp writes the slices to the k claimed rows; the shared expert's row
// nk + t needs no position and is written before the scan. Longer rows are
// read twice after the scan. The row
// loop is not unrolled: this kernel runs once per block, mostly from a cold
// instruction cache, so its code is kept short.
template <typename XT, bool SLICE>
__global__ void __launch_bounds__(256) dispatch_kernel(const XT* __restrict__ h, const int32_t* __restrict__ idx,
                                                       const float* __restrict__ w, int n, int k, int E, int H, int I,
                                                       int Is, SchedSpec spec0, SchedSpec spec1, int shared,
                                                       Plan* __restrict__ plan, const uint64_t* __restrict__ records,
                                                       int32_t* __restrict__ perm_token,
                                                       float* __restrict__ perm_w, int32_t* __restrict__ pos_of,
                                                       int8_t* __restrict__ s0, int8_t* __restrict__ s1,
                                                       float* __restrict__ scale) {
  __shared__ int hist[kMaxExperts];
  __shared__ int offs[kMaxExperts];
  __shared__ int act[kMaxExperts + 1];
  __shared__ int bad;
  __shared__ int scan_tmp[16];
  __shared__ int ccount[kMaxExperts];  // this CTA's pairs per expert
  __shared__ int cbase[kMaxExperts];   // their first position in the expert's range
  for (int x = threadIdx.x; x < E; x += blockDim.x) ccount[x] = 0;  // ordered by plan_scan's barriers
  chain_wait();
  uint64_t rec0, rec1;
  plan_records(records, blockIdx.x == 0, E, rec0, rec1);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t = blockIdx.x * 8 + warp;
  constexpr int kRegVec = 16;  // float4 per lane held in registers: H <= 2048
  const bool in_regs = SLICE && H <= 128 * kRegVec;
  uint32_t q0[kRegVec], q1[kRegVec];
  float amax = 0.f;
  if (in_regs && t < n) {
    const XT* x = h + (size_t)t * H;
    float4 v[kRegVec];
#pragma unroll
    for (int i = 0; i < kRegVec; ++i) {
      const int c = lane * 4 + 128 * i;
      v[i] = c < H ? load4(x + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      amax = fmaxf(amax, abs_max4(v[i]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float inv = amax > 0.f ? 127.f / amax : 0.f;
#pragma unroll
    for (int i = 0; i < kRegVec; ++i) slice4(v[i], inv, q0[i], q1[i]);
    if (shared) {
      // the shared expert's row (nk + t) needs no position: written now, so
      // its stores overlap the scan and the position claims below
      const size_t row = (size_t)n * k + t;
#pragma unroll
      for (int i = 0; i < kRegVec; ++i) {
        const int c = lane * 4 + 128 * i;
        if (c < H) {
          *reinterpret_cast<uint32_t*>(s0 + row * H + c) = q0[i];
          *reinterpret_cast<uint32_t*>(s1 + row * H + c) = q1[i];
        }
      }
      if (lane == 31) scale[row] = amax / 127.f;
    }
  }
  plan_scan(plan, n, k, E, H, I, Is, spec0, spec1, shared, blockIdx.x == 0, hist, offs, act, &bad, scan_tmp, nullptr,
            rec0, rec1);
  // Positions: each (token, slot) pair takes a rank among this CTA's pairs
  // of the same expert (shared-memory atomics), then one thread per expert
  // claims the CTA's block of the expert's range with one global atomic (a
  // popular expert would otherwise serialise hundreds of atomics on one
  // address). Nothing downstream reads positions of an inconsistent tally.
  const bool live = t < n && !bad;
  int e = -1, li = 0;
  if (live && lane < k) {
    e = idx[(size_t)t * k + lane];
    if (e >= 0 && e < E)
      li = atomicAdd(&ccount[e], 1);
    else
      atomicOr(&plan->error, 1);
  }
  __syncthreads();
  for (int x = threadIdx.x; x < E; x += blockDim.x)
    if (ccount[x] > 0) cbase[x] = atomicAdd(&plan->cursor[x], ccount[x]);
  __syncthreads();
  if (!live) return;
  const int nk = n * k;
  int p = -1;
  if (lane < k) {
    if (e >= 0 && e < E) {
      const int c = cbase[e] + li;
      if (c >= hist[e]) {  // only an inconsistent tally gets here
        atomicOr(&plan->error, 2);
      } else {
        p = offs[e] + c;
        perm_token[p] = t;
        perm_w[p] = w[(size_t)t * k + lane];
      }
    }
    pos_of[(size_t)t * k + lane] = p;
  }
  if constexpr (SLICE) {
    const XT* x = h + (size_t)t * H;
    if (!in_regs) {
      for (int c = lane * 4; c < H; c += 128) amax = fmaxf(amax, abs_max4(load4(x + c)));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    }
    const float inv = amax > 0.f ? 127.f / amax : 0.f;
    // rows r < k: the claimed positions; row k: the shared expert's row
    // (already written when the slices are held in registers)
#pragma unroll 1
    for (int r = 0; r <= k; ++r) {
      const int pr = __shfl_sync(0xffffffffu, p, r < k ? r : 0);
      const int row = r < k ? pr : (shared && !in_regs ? nk + t : -1);
      if (row < 0) continue;
      int8_t* d0 = s0 + (size_t)row * H;
      int8_t* d1 = s1 + (size_t)row * H;
      if (in_regs) {
#pragma unroll
        for (int i = 0; i < kRegVec; ++i) {
          const int c = lane * 4 + 128 * i;
          if (c < H) {
            *reinterpret_cast<uint32_t*>(d0 + c) = q0[i];
            *reinterpret_cast<uint32_t*>(d1 + c) = q1[i];
          }
        }
      } else {
        for (int c = lane * 4; c < H; c += 128) {
          uint32_t w0, w1;
          slice4(load4(x + c), inv, w0, w1);
          *reinterpret_cast<uint32_t*>(d0 + c) = w0;
          *reinterpret_cast<uint32_t*>(d1 + c) = w1;
        }
      }
    }
    if (lane < k && p >= 0) scale[p] = amax / 127.f;
    if (lane == 31 && shared && !in_regs) scale[nk + t] = amax / 127.f;
  }
}

// Small batches (n <= kFusedTopkMaxTok), top-k fused: CTA c of n owns token
// c. Every CTA runs the softmax + top-k of all n tokens (a warp each) into
// shared memory and derives the plan from those tallies (an extra CTA n
// writes it, so the plan's writes and the row slicing run side by side; the
// top-k outputs of token c are written by CTA c), so the positions need no
// atomics: slot j of token t goes to its expert's range start plus the
// number of earlier (token, slot) pairs of the same expert. The whole CTA
// slices token c's h row into its k rows and the shared row, so the rows'
// stores spread over n SMs: the row is loaded right after the wait (thread i
// holds values 4i + 4 blockDim j, in registers for rows of up to
// 4 kSmallVec blockDim values), so its latency hides behind the top-k and
// the plan, and its max is reduced across the warps on the way.
constexpr int kSmallVec = 2;
template <typename XT, bool SLICE, int KPER>
__global__ void __launch_bounds__(512) dispatch_small_kernel(const XT* __restrict__ h, int n, int k, int E, int H,
                                                             int I, int Is, SchedSpec spec0, SchedSpec spec1,
                                                             int shared, Plan* __restrict__ plan,
                                                             const uint64_t* __restrict__ records,
                                                             int32_t* __restrict__ perm_token,
                                                             float* __restrict__ perm_w, int32_t* __restrict__ pos_of,
                                                             int8_t* __restrict__ s0, int8_t* __restrict__ s1,
                                                             float* __restrict__ scale, TopkArgs topk) {
  __shared__ int hist[kMaxExperts];
  __shared__ int offs[kMaxExperts];
  __shared__ int act[kMaxExperts + 1];
  __shared__ int tally_s[kMaxExperts];
  __shared__ int sel_s[kFusedTopkMaxTok * kMaxTopK];
  __shared__ float w_s[kFusedTopkMaxTok * kMaxTopK];
  __shared__ int bad;
  __shared__ int scan_tmp[16];
  __shared__ float amax_s[16];       // per warp: max |h| over its values of the token's row
  __shared__ int pos_s[kMaxTopK];    // the token's slots' expert-sorted positions
  chain_trigger();  // the gate/up GEMM's CTAs may start their prologue meanwhile
  chain_wait();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nthr = blockDim.x;
  const int me = blockIdx.x;  // this CTA's token; CTA n has none and writes the plan
  const XT* x = SLICE ? h + (size_t)(me < n ? me : 0) * H : h;
  const bool in_regs = H <= 4 * kSmallVec * nthr;
  float4 hv[kSmallVec];
  // issued now, used after the top-k: the row's latency overlaps it
  if (SLICE && me < n && in_regs) {
#pragma unroll
    for (int j = 0; j < kSmallVec; ++j) {
      const int c = 4 * (threadIdx.x + nthr * j);
      hv[j] = c < H ? load4(x + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  uint64_t rec0, rec1;
  plan_records(records, me == n, E, rec0, rec1);
  for (int e = threadIdx.x; e < E; e += nthr) tally_s[e] = 0;
  __syncthreads();
  if (warp < n) {
    TopkArgs a = topk;
    a.idx64 = nullptr;
    a.idx32 = sel_s;
    a.wout = w_s;
    a.tally = tally_s;
    if (warp != me) {  // the token's own CTA writes its gate and summed logits
      a.gate_sig = nullptr;
      a.logits_sum = nullptr;
    }
    topk_token<KPER>(a, n, E, k, warp, lane);
  }
  if (SLICE && me < n) {
    float amax = 0.f;
    if (in_regs) {
#pragma unroll
      for (int j = 0; j < kSmallVec; ++j) amax = fmaxf(amax, abs_max4(hv[j]));
    } else {
      for (int c = 4 * threadIdx.x; c < H; c += 4 * nthr) amax = fmaxf(amax, abs_max4(load4(x + c)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) amax_s[warp] = amax;
  }
  __syncthreads();
  plan_scan(plan, n, k, E, H, I, Is, spec0, spec1, shared, me == n, hist, offs, act, &bad, scan_tmp, tally_s, rec0,
            rec1);
  if (me >= n || bad) return;  // uniform over the CTA
  const int nk = n * k;
  if (warp == 0 && lane < k) {
    const int e = sel_s[me * k + lane];
    const float wt = w_s[me * k + lane];
    if (topk.idx32) topk.idx32[(size_t)me * k + lane] = e;
    if (topk.idx64) topk.idx64[(size_t)me * k + lane] = e;
    if (topk.wout) topk.wout[(size_t)me * k + lane] = wt;
    int before = 0;  // earlier (token, slot) pairs routed to e
    for (int i = 0; i < me * k + lane; ++i) before += sel_s[i] == e;
    const int p = offs[e] + before;
    perm_token[p] = me;
    perm_w[p] = wt;
    pos_of[(size_t)me * k + lane] = p;
    pos_s[lane] = p;
  }
  if constexpr (SLICE) {
    __syncthreads();
    float amax = 0.f;
    for (int w = 0; w < nthr / 32; ++w) amax = fmaxf(amax, amax_s[w]);
    const float inv = amax > 0.f ? 127.f / amax : 0.f;
#pragma unroll 1
    for (int r = 0; r <= k; ++r) {  // rows r < k: the slots' positions; row k: the shared expert's row
      const int row = r < k ? pos_s[r] : (shared ? nk + me : -1);
      if (row < 0) continue;
      int8_t* d0 = s0 + (size_t)row * H;
      int8_t* d1 = s1 + (size_t)row * H;
      if (in_regs) {
#pragma unroll
        for (int j = 0; j < kSmallVec; ++j) {
          const int c = 4 * (threadIdx.x + nthr * j);
          if (c < H) {
            uint32_t w0, w1;
            slice4(hv[j], inv, w0, w1);
            *reinterpret_cast<uint32_t*>(d0 + c) = w0;
            *reinterpret_cast<uint32_t*>(d1 + c) = w1;
          }
        }
      } else {
        for (int c = 4 * threadIdx.x; c < H; c += 4 * nthr) {
          uint32_t w0, w1;
          slice4(load4(x + c), inv, w0, w1);
          *reinterpret_cast<uint32_t*>(d0 + c) = w0;
          *reinterpret_cast<uint32_t*>(d1 + c) = w1;
        }
      }
    }
    if (threadIdx.x < k) scale[pos_s[threadIdx.x]] = amax / 127.f;
    if (threadIdx.x == 32 && shared) scale[nk + me] = amax / 127.f;
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
  return routed_rows_tiles * nt_r + shared_tiles * nt_s * (s.which == 1 && s.ks > 1 ? s.ks : 1);
}

__global__ void __launch_bounds__(256) tally_kernel(const int32_t* __restrict__ ids, int m, int E,
                                                    int* __restrict__ tally) {
  chain_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= m) return;
  const int e = ids[i];
  if (e >= 0 && e < E) atomicAdd(&tally[e], 1);
}

int launch_tally(const int32_t* ids, int m, int E, int* tally, int nclear, cudaStream_t st) {
  if (int rc = cuda_check(cudaMemsetAsync(tally, 0, (size_t)nclear * sizeof(int), st), "clear tally")) return rc;
  if (m <= 0) return ER_OK;
  return launch_chained(tally_kernel, dim3((m + 255) / 256), dim3(256), 0, st, "tally_kernel", ids, m, E, tally);
}

template <typename XT, bool SLICE>
static int launch_dispatch_t(const XT* h, const int32_t* idx, const float* w, int n, int k, int E, int H, int I, int Is,
                             const SchedSpec* specs, int shared, Plan* plan, const uint64_t* records,
                             int32_t* perm_token, float* perm_w, int32_t* pos_of, int8_t* s0, int8_t* s1,
                             float* scale, const TopkArgs* topk, cudaStream_t st) {
  if (topk) {  // a CTA per token and one more that writes the plan, a warp per token inside each
    const dim3 grid(n + 1), block(32 * (n > 8 ? 16 : 8));
    if (E <= 64)
      return launch_chained(dispatch_small_kernel<XT, SLICE, 2>, grid, block, 0, st, "dispatch_small_kernel", h, n,
                            k, E, H, I, Is, specs[0], specs[1], shared, plan, records, perm_token, perm_w, pos_of, s0,
                            s1, scale, *topk);
    return launch_chained(dispatch_small_kernel<XT, SLICE, kMaxExperts / 32>, grid, block, 0, st,
                          "dispatch_small_kernel", h, n, k, E, H, I, Is, specs[0], specs[1], shared, plan, records,
                          perm_token, perm_w, pos_of, s0, s1, scale, *topk);
  }
  const int blocks = n > 0 ? (n + 7) / 8 : 1;  // CTA 0 writes the plan even for no tokens
  return launch_chained(dispatch_kernel<XT, SLICE>, dim3(blocks), dim3(256), 0, st, "dispatch_kernel", h, idx, w, n,
                        k, E, H, I, Is, specs[0], specs[1], shared, plan, records, perm_token, perm_w, pos_of, s0, s1,
                        scale);
}

int launch_dispatch(const void* h, int h_dtype, const int32_t* idx, const float* w, int n, int k, int E, int H, int I,
                    int Is, const SchedSpec* specs, int shared, Plan* plan, const uint64_t* records,
                    int32_t* perm_token, float* perm_w, int32_t* pos_of, int8_t* s0, int8_t* s1, float* scale,
                    const TopkArgs* topk, cudaStream_t st) {
  if (topk && (n > kFusedTopkMaxTok || topk->idx32 != idx || topk->wout != w || topk->tally != plan->tally))
    return fail(ER_EINVAL, "dispatch: fused top-k needs n <= %d and its outputs as the dispatch inputs",
                kFusedTopkMaxTok);
  if (!s0)
    return launch_dispatch_t<float, false>(nullptr, idx, w, n, k, E, H, I, Is, specs, shared, plan, records, perm_token,
                                           perm_w, pos_of, nullptr, nullptr, nullptr, topk, st);
  if (h_dtype == ER_DTYPE_BF16)
    return launch_dispatch_t<__nv_bfloat16, true>((const __nv_bfloat16*)h, idx, w, n, k, E, H, I, Is, specs, shared,
                                                  plan, records, perm_token, perm_w, pos_of, s0, s1, scale, topk, st);
  return launch_dispatch_t<float, true>((const float*)h, idx, w, n, k, E, H, I, Is, specs, shared, plan, records,
                                        perm_token, perm_w, pos_of, s0, s1, scale, topk, st);
}

}  // namespace er
