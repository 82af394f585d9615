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
#include "er_internal.cuh"

namespace er {

// The plan from the per-expert tallies, by one warp: lane l owns entries
// 9l .. 9l+8 of the per-expert lists (enough for E + 2 <= 258) and the scans
// run over the lanes. Every caller gets the expert ranges' first positions in
// `offs` (shared memory) and whether the tallies are consistent; with
// write_plan it also writes the plan's groups, ranges and work-item schedules
// for the expert kernels.
__device__ void plan_scan(Plan* __restrict__ plan, int n, int k, int E, int H, int I, int Is, SchedSpec s0,
                          SchedSpec s1, int shared, bool write_plan, int* hist, int* offs, int* act, int* bad_out) {
  constexpr int kPer = 9;
  const int lane = threadIdx.x & 31;
  const int nk = n * k;
  auto warp_excl_scan = [&](int v) {  // exclusive prefix of v over the lanes
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    return incl - v;
  };
  for (int e = lane; e < E; e += 32) hist[e] = plan->tally[e];
  __syncwarp();
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
  const int total = __shfl_sync(0xffffffffu, off + sum, 31);
  const int na_routed = __shfl_sync(0xffffffffu, pos + nact, 31);
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = lane * kPer + j;
    if (e < E) {
      offs[e] = off;
      if (write_plan) {
        plan->counts[e] = hist[e];
        plan->offsets[e] = off;
      }
      off += hist[e];
      if (hist[e] > 0) act[pos++] = e;
    }
  }
  // every pair lands in some expert's range: the counts must add up to n * k
  const bool bad = total != nk;
  if (lane == 0) *bad_out = bad;
  if (!write_plan) {
    __syncwarp();
    return;
  }
  const int na = na_routed + (shared && n > 0 ? 1 : 0);
  if (lane == 0) {
    if (shared && n > 0) act[na_routed] = E;
    plan->counts[E] = n;
    plan->offsets[E] = 0;
  }
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
    plan->num_active = bad ? 0 : na;  // no work items on an inconsistent tally
  }
  __syncwarp();
}

// Eight tokens per CTA, one warp each. Warp 0 first derives the expert
// ranges from the tallies (CTA 0 also writes the plan). Then lane r < k of a
// token's warp claims the position of slot r (its expert's range start plus
// an atomic count, from 0); with SLICE the warp slices h[t] (K = H values)
// and writes the slices to the k claimed rows and, for the shared expert, to
// row nk + t. Rows of up to 2048 values stay in registers; longer rows are
// read twice.
template <typename XT, bool SLICE>
__global__ void __launch_bounds__(256) dispatch_kernel(const XT* __restrict__ h, const int32_t* __restrict__ idx,
                                                       const float* __restrict__ w, int n, int k, int E, int H, int I,
                                                       int Is, SchedSpec spec0, SchedSpec spec1, int shared,
                                                       Plan* __restrict__ plan, int32_t* __restrict__ perm_token,
                                                       float* __restrict__ perm_w, int32_t* __restrict__ pos_of,
                                                       int8_t* __restrict__ s0, int8_t* __restrict__ s1,
                                                       float* __restrict__ scale) {
  __shared__ int hist[kMaxExperts];
  __shared__ int offs[kMaxExperts];
  __shared__ int act[kMaxExperts + 1];
  __shared__ int bad;
  chain_wait();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (warp == 0) plan_scan(plan, n, k, E, H, I, Is, spec0, spec1, shared, blockIdx.x == 0, hist, offs, act, &bad);
  __syncthreads();
  const int t = blockIdx.x * 8 + warp;
  if (t >= n || bad) return;  // nothing downstream reads positions of an inconsistent tally
  const int nk = n * k;
  int p = -1;
  if (lane < k) {
    const int e = idx[(size_t)t * k + lane];
    if (e >= 0 && e < E) {
      const int c = atomicAdd(&plan->cursor[e], 1);
      if (c >= hist[e]) {  // only an inconsistent tally gets here
        atomicOr(&plan->error, 2);
      } else {
        p = offs[e] + c;
        perm_token[p] = t;
        perm_w[p] = w[(size_t)t * k + lane];
      }
    } else {
      atomicOr(&plan->error, 1);
    }
    pos_of[(size_t)t * k + lane] = p;
  }
  if constexpr (SLICE) {
    int prow[kMaxTopK + 1];
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r) prow[r] = __shfl_sync(0xffffffffu, p, r < k ? r : 31);
    prow[kMaxTopK] = shared ? nk + t : -1;  // the shared expert's row
    const XT* x = h + (size_t)t * H;
    auto put = [&](int c, float4 v, float inv) {
      uint32_t w0, w1;
      slice4(v, inv, w0, w1);
#pragma unroll
      for (int r = 0; r <= kMaxTopK; ++r) {
        const int row = r < kMaxTopK ? (r < k ? prow[r] : -1) : prow[kMaxTopK];
        if (row >= 0) {
          *reinterpret_cast<uint32_t*>(s0 + (size_t)row * H + c) = w0;
          *reinterpret_cast<uint32_t*>(s1 + (size_t)row * H + c) = w1;
        }
      }
    };
    float amax = 0.f;
    constexpr int kRegVec = 16;  // float4 per lane held in registers: H <= 2048
    if (H <= 128 * kRegVec) {
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
      for (int i = 0; i < kRegVec; ++i) {
        const int c = lane * 4 + 128 * i;
        if (c < H) put(c, v[i], inv);
      }
    } else {
      for (int c = lane * 4; c < H; c += 128) amax = fmaxf(amax, abs_max4(load4(x + c)));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float inv = amax > 0.f ? 127.f / amax : 0.f;
      for (int c = lane * 4; c < H; c += 128) put(c, load4(x + c), inv);
    }
    if (lane < k && p >= 0) scale[p] = amax / 127.f;
    if (lane == 31 && shared) scale[nk + t] = amax / 127.f;
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

int launch_dispatch(const void* h, int h_dtype, const int32_t* idx, const float* w, int n, int k, int E, int H, int I,
                    int Is, const SchedSpec* specs, int shared, Plan* plan, int32_t* perm_token, float* perm_w,
                    int32_t* pos_of, int8_t* s0, int8_t* s1, float* scale, cudaStream_t st) {
  const int blocks = n > 0 ? (n + 7) / 8 : 1;  // CTA 0 writes the plan even for no tokens
  if (!s0)
    return launch_chained(dispatch_kernel<float, false>, dim3(blocks), dim3(256), 0, st, "dispatch_kernel",
                          (const float*)nullptr, idx, w, n, k, E, H, I, Is, specs[0], specs[1], shared, plan,
                          perm_token, perm_w, pos_of, (int8_t*)nullptr, (int8_t*)nullptr, (float*)nullptr);
  if (h_dtype == ER_DTYPE_BF16)
    return launch_chained(dispatch_kernel<__nv_bfloat16, true>, dim3(blocks), dim3(256), 0, st, "dispatch_kernel",
                          (const __nv_bfloat16*)h, idx, w, n, k, E, H, I, Is, specs[0], specs[1], shared, plan,
                          perm_token, perm_w, pos_of, s0, s1, scale);
  return launch_chained(dispatch_kernel<float, true>, dim3(blocks), dim3(256), 0, st, "dispatch_kernel",
                        (const float*)h, idx, w, n, k, E, H, I, Is, specs[0], specs[1], shared, plan, perm_token,
                        perm_w, pos_of, s0, s1, scale);
}

}  // namespace er
