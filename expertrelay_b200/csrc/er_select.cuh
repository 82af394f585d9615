// er_select.cuh -- the router's softmax + top-k of one token, by one warp
// (used by the top-k kernel and, for small batches, by the dispatch kernel).
#pragma once
#include "er_internal.cuh"

namespace er {

// Softmax over the E logits of one token held by a warp (lane l holds
// experts l + 32 j in v[j]; max subtracted, expf, sum, divide) and top-k by
// logit value, largest first, exact ties to the lower expert id. Ranking by
// the logits equals ranking by the probabilities because every step of the
// softmax is monotone; NaN logits rank as -inf. Writes token t's ids and
// weights; tally (optional) counts the selected experts.
template <int kPer>
__device__ __forceinline__ void warp_select(const float (&v)[kPer], int E, int k, int norm, int t, int lane,
                                            int64_t* __restrict__ idx64, int32_t* __restrict__ idx32,
                                            float* __restrict__ wout, int* __restrict__ tally) {
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kPer; ++j) mx = fmaxf(mx, v[j]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float ex[kPer], s = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = lane + 32 * j;
    ex[j] = (e < E) ? expf(v[j] - mx) : 0.f;
    s += ex[j];
  }
  s = warp_sum(s);

  uint32_t taken = 0;  // bit j: entry lane + 32 j already selected
  // lane r < k keeps slot r's expert and probability; the rounds are not
  // unrolled (the dispatch kernel of decode batches runs this code cold)
  int my_sel = 0;
  float my_p = 0.f, wsum = 0.f;
#pragma unroll 1
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int e = lane + 32 * j;
      if (e < E && !(taken & (1u << j))) {
        const float c = (v[j] != v[j]) ? -INFINITY : v[j];
        if (c > bv || (c == bv && e < bi)) {
          bv = c;
          bi = e;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    // the owner lane marks the entry and broadcasts its probability
    const int owner = bi & 31, oj = bi >> 5;
    float p = 0.f;
    if (lane == owner) {
#pragma unroll
      for (int j = 0; j < kPer; ++j)
        if (j == oj) {
          taken |= 1u << j;
          p = ex[j] / s;
        }
    }
    p = __shfl_sync(0xffffffffu, p, owner);
    if (lane == r) {
      my_sel = bi;
      my_p = p;
    }
    wsum += p;
  }
  if (lane < k) {
    if (tally) atomicAdd(&tally[my_sel], 1);
    const float w = norm ? my_p / wsum : my_p;
    if (idx64) idx64[(size_t)t * k + lane] = my_sel;
    if (idx32) idx32[(size_t)t * k + lane] = my_sel;
    if (wout) wout[(size_t)t * k + lane] = w;
  }
}

// Token t's logits (the sum of `nparts` K-slice partials, added in slice
// order) through warp_select, and its shared-expert gate.
template <int kPer>
__device__ __forceinline__ void topk_token(const TopkArgs& a, int n, int E, int k, int t, int lane) {
  const float* l = a.logits + (size_t)t * E;
  // the shared gate's logit is loaded with the router's (added in part order)
  const bool gate = lane == 0 && a.gate_sig && a.gate_logit;
  float gl = 0.f;
  if (gate) {
    gl = a.gate_logit[t];
    for (int p = 1; p < a.gparts; ++p) gl += a.gate_logit[(size_t)p * n + t];
  }
  // every partial of every entry is loaded before any is added (one memory
  // latency, not one per partial), then added in partial order
  float part[kPer][kRouterKSplit];
#pragma unroll
  for (int j = 0; j < kPer; ++j)
#pragma unroll
    for (int p = 0; p < kRouterKSplit; ++p) {
      const int e = lane + 32 * j;
      part[j][p] = (e < E && p < a.nparts) ? l[(size_t)p * n * E + e] : 0.f;
    }
  float v[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = lane + 32 * j;
    v[j] = -INFINITY;
    if (e < E) {
      float s = part[j][0];
#pragma unroll
      for (int p = 1; p < kRouterKSplit; ++p)
        if (p < a.nparts) s += part[j][p];
      for (int p = kRouterKSplit; p < a.nparts; ++p) s += l[(size_t)p * n * E + e];  // more partials than kept
      v[j] = s;
      if (a.logits_sum) a.logits_sum[(size_t)t * E + e] = s;
    }
  }
  warp_select<kPer>(v, E, k, a.norm, t, lane, a.idx64, a.idx32, a.wout, a.tally);
  if (gate) a.gate_sig[t] = sigmoid_f(gl);
}

}  // namespace er
