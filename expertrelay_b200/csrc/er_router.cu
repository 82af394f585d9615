// er_router.cu -- K1: router logits, softmax and top-k.
//
// Reference: runtime/qwen_moe.py:303-308 (router = backend.linear(h, W_r),
// probs = softmax over all experts in fp32, selected = top-k largest first,
// weights = probs of the selected experts, no renormalisation when
// norm_topk_prob is False) and :358 (shared-expert gate logit h @ w_g^T).
#include "er_internal.cuh"

namespace er {

// logits[t, e] = h[t] . W_r[e] for e < E and gate_logit[t] = h[t] . w_g (row E),
// fp32 FMA. One CTA holds kTok tokens of h in shared memory; its warps walk
// a slice of the E + 1 weight rows (grid.y slices split the rows for small n).
template <typename XT>
__global__ void __launch_bounds__(256) router_logits_kernel(const XT* __restrict__ h, int n, int H,
                                                            const float* __restrict__ wr,
                                                            const float* __restrict__ wg, int E,
                                                            float* __restrict__ logits,
                                                            float* __restrict__ gate_logit,
                                                            int rows_per_cta) {
  constexpr int kTok = kRouterTok;
  extern __shared__ __align__(16) float hs[];  // [kTok][H]
  const int t0 = blockIdx.x * kTok;
  const int nt = min(kTok, n - t0);
  for (int i = threadIdx.x; i < kTok * H; i += blockDim.x) {
    const int t = i / H, k = i - t * H;
    hs[i] = (t < nt) ? to_f32(h[(size_t)(t0 + t) * H + k]) : 0.f;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int r_begin = blockIdx.y * rows_per_cta;
  const int r_end = min(E + 1, r_begin + rows_per_cta);
  for (int r = r_begin + warp; r < r_end; r += nw) {
    const float* w = (r < E) ? wr + (size_t)r * H : wg;
    float acc[kTok];
#pragma unroll
    for (int t = 0; t < kTok; ++t) acc[t] = 0.f;
    for (int k = lane * 4; k < H; k += 128) {
      const float4 wv = *reinterpret_cast<const float4*>(w + k);
#pragma unroll
      for (int t = 0; t < kTok; ++t) {
        const float4 xv = *reinterpret_cast<const float4*>(hs + t * H + k);
        acc[t] = fmaf(wv.x, xv.x, acc[t]);
        acc[t] = fmaf(wv.y, xv.y, acc[t]);
        acc[t] = fmaf(wv.z, xv.z, acc[t]);
        acc[t] = fmaf(wv.w, xv.w, acc[t]);
      }
    }
#pragma unroll
    for (int t = 0; t < kTok; ++t) acc[t] = warp_sum(acc[t]);
    if (lane == 0) {
      for (int t = 0; t < nt; ++t) {
        if (r < E)
          logits[(size_t)(t0 + t) * E + r] = acc[t];
        else if (gate_logit)
          gate_logit[t0 + t] = acc[t];
      }
    }
  }
}

// One warp per token: softmax over the E logits (max subtracted, expf, sum,
// divide) and top-k by logit value, largest first, exact ties to the lower
// expert id. Ranking by the logits equals ranking by the probabilities
// because every step of the softmax is monotone; NaN logits rank as -inf.
__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ logits, int n, int E,
                                                          int k, int norm, int64_t* __restrict__ idx64,
                                                          int32_t* __restrict__ idx32,
                                                          float* __restrict__ wout,
                                                          const float* __restrict__ gate_logit,
                                                          float* __restrict__ gate_sig) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= n) return;
  const float* l = logits + (size_t)t * E;
  constexpr int kPer = kMaxExperts / 32;
  float v[kPer], ex[kPer];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = lane + 32 * j;
    v[j] = (e < E) ? l[e] : -INFINITY;
    mx = fmaxf(mx, v[j]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = lane + 32 * j;
    ex[j] = (e < E) ? expf(v[j] - mx) : 0.f;
    s += ex[j];
  }
  s = warp_sum(s);

  uint32_t taken = 0;  // bit j: entry lane + 32 j already selected
  int sel[kMaxTopK];
  float pw[kMaxTopK];
  float wsum = 0.f;
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
    sel[r] = bi;
    pw[r] = p;
    wsum += p;
  }
  if (lane == 0) {
    for (int r = 0; r < k; ++r) {
      const float w = norm ? pw[r] / wsum : pw[r];
      if (idx64) idx64[(size_t)t * k + r] = sel[r];
      if (idx32) idx32[(size_t)t * k + r] = sel[r];
      if (wout) wout[(size_t)t * k + r] = w;
    }
    if (gate_sig && gate_logit) gate_sig[t] = sigmoid_f(gate_logit[t]);
  }
}

int launch_router_logits(const void* h, int h_dtype, int n, int H, const float* wr, const float* wg, int E,
                         float* logits, float* gate_logit, cudaStream_t st) {
  if (n <= 0) return ER_OK;
  const size_t smem = (size_t)kRouterTok * H * sizeof(float);
  static thread_local int configured_dev[2] = {-1, -1};
  int dev = 0;
  if (int rc = cuda_check(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  const int tiles = (n + kRouterTok - 1) / kRouterTok;
  // few token tiles: split the E + 1 rows over CTAs so the launch fills the GPU
  const int splits = tiles >= 64 ? 1 : 8;
  const int rows_per_cta = (E + 1 + splits - 1) / splits;
  dim3 grid(tiles, splits);
  if (h_dtype == ER_DTYPE_F32) {
    if (configured_dev[0] != dev) {
      if (int rc = cuda_check(cudaFuncSetAttribute(router_logits_kernel<float>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024),
                              "router smem attribute"))
        return rc;
      configured_dev[0] = dev;
    }
    router_logits_kernel<float><<<grid, 256, smem, st>>>((const float*)h, n, H, wr, wg, E, logits, gate_logit,
                                                         rows_per_cta);
  } else {
    if (configured_dev[1] != dev) {
      if (int rc = cuda_check(cudaFuncSetAttribute(router_logits_kernel<__nv_bfloat16>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024),
                              "router smem attribute"))
        return rc;
      configured_dev[1] = dev;
    }
    router_logits_kernel<__nv_bfloat16><<<grid, 256, smem, st>>>((const __nv_bfloat16*)h, n, H, wr, wg, E,
                                                                 logits, gate_logit, rows_per_cta);
  }
  return launch_check("router_logits_kernel");
}

int launch_router_topk(const float* logits, int n, int E, int k, int norm, int64_t* idx64, int32_t* idx32,
                       float* wout, const float* gate_logit, float* gate_sig, cudaStream_t st) {
  if (n <= 0) return ER_OK;
  const int warps_per_block = 8;
  const int blocks = (n + warps_per_block - 1) / warps_per_block;
  router_topk_kernel<<<blocks, warps_per_block * 32, 0, st>>>(logits, n, E, k, norm, idx64, idx32, wout,
                                                               gate_logit, gate_sig);
  return launch_check("router_topk_kernel");
}

}  // namespace er

extern "C" int er_router_topk(const float* logits, int n, int num_experts, int k, int64_t* idx64, int32_t* idx32,
                              float* probs_out, void* stream) {
  using namespace er;
  if (!logits || n < 0) return fail(ER_EINVAL, "er_router_topk: null logits or negative n");
  if (num_experts < 1 || num_experts > kMaxExperts)
    return fail(ER_EINVAL, "er_router_topk: num_experts %d outside 1..%d", num_experts, kMaxExperts);
  if (k < 1 || k > kMaxTopK || k > num_experts)
    return fail(ER_EINVAL, "er_router_topk: k %d outside 1..min(%d, num_experts)", k, kMaxTopK);
  return launch_router_topk(logits, n, num_experts, k, 0, idx64, idx32, probs_out, nullptr, nullptr,
                            (cudaStream_t)stream);
}
