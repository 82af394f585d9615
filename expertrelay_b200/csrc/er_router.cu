// er_router.cu -- K1: router logits, softmax and top-k.
//
// Reference: runtime/qwen_moe.py:303-308 (router = backend.linear(h, W_r),
// probs = softmax over all experts in fp32, selected = top-k largest first,
// weights = probs of the selected experts, no renormalisation when
// norm_topk_prob is False) and :358 (shared-expert gate logit h @ w_g^T).
#include "er_select.cuh"

namespace er {

// Decode-sized batches: one CTA per weight row r of [W_r; w_g] (E + 1 rows).
// Thread i owns columns {4i + 1024j}; the row stays in registers while the
// CTA walks the tokens kRouterTok at a time; fp32 FMA, then a block reduction.
template <typename XT>
__global__ void __launch_bounds__(256) router_rows_kernel(const XT* __restrict__ h, int n, int H,
                                                          const float* __restrict__ wr, const float* __restrict__ wg,
                                                          int E, float* __restrict__ logits,
                                                          float* __restrict__ gate_logit, int* __restrict__ tally,
                                                          int ntally) {
  chain_wait();
  constexpr int kTok = kRouterTok;
  if (blockIdx.x == 0 && tally)  // cleared for the top-k kernel's per-expert counts
    for (int i = threadIdx.x; i < ntally; i += blockDim.x) tally[i] = 0;
  __shared__ float red[8][kTok];
  const int r = blockIdx.x;
  const float* w = (r < E) ? wr + (size_t)r * H : wg;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int t0 = 0; t0 < n; t0 += kTok) {
    const int nt = min(kTok, n - t0);
    float acc[kTok];
#pragma unroll
    for (int t = 0; t < kTok; ++t) acc[t] = 0.f;
    for (int k = threadIdx.x * 4; k < H; k += 1024) {
      const float4 wv = *reinterpret_cast<const float4*>(w + k);
#pragma unroll
      for (int t = 0; t < kTok; ++t) {
        if (t < nt) {
          const float4 xv = load4(h + (size_t)(t0 + t) * H + k);
          acc[t] = fmaf(wv.x, xv.x, acc[t]);
          acc[t] = fmaf(wv.y, xv.y, acc[t]);
          acc[t] = fmaf(wv.z, xv.z, acc[t]);
          acc[t] = fmaf(wv.w, xv.w, acc[t]);
        }
      }
    }
#pragma unroll
    for (int t = 0; t < kTok; ++t) {
      const float v = warp_sum(acc[t]);
      if (lane == 0) red[warp][t] = v;
    }
    __syncthreads();
    if (threadIdx.x < nt) {
      float v = 0.f;
      for (int w8 = 0; w8 < 8; ++w8) v += red[w8][threadIdx.x];
      if (r < E)
        logits[(size_t)(t0 + threadIdx.x) * E + r] = v;
      else if (gate_logit)
        gate_logit[t0 + threadIdx.x] = v;
    }
    __syncthreads();
  }
}

// Large batches: a tiled fp32 GEMM, 32 tokens x 64 rows of [W_r; w_g] per
// CTA (rows past E + 1 are zero). blockIdx.y picks one of gridDim.y slices of
// K and the CTA writes that slice's partial logits (the top-k kernel adds the
// slices in a fixed order). Inside, the 256 threads form four K-groups of 64
// that each walk a quarter of the slice through shared memory, fetching the
// next tile into registers while computing; a thread owns 4 tokens x 8 rows.
// The four group sums are added in a fixed order.
template <typename XT>
__global__ void __launch_bounds__(256) router_gemm_kernel(const XT* __restrict__ h, int n, int H,
                                                          const float* __restrict__ wr,
                                                          const float* __restrict__ wg, int E,
                                                          float* __restrict__ logits,
                                                          float* __restrict__ gate_logit, int* __restrict__ tally,
                                                          int ntally) {
  chain_wait();
  constexpr int BM = 32, BN = 64, BK = 16, KG = 4;
  if (blockIdx.x == 0 && blockIdx.y == 0 && tally)  // cleared for the top-k kernel's per-expert counts
    for (int i = threadIdx.x; i < ntally; i += blockDim.x) tally[i] = 0;
  struct Tiles {
    float A[KG][BK][BM + 4];
    float B[KG][BK][BN + 4];
  };
  __shared__ __align__(16) union {
    Tiles t;
    float red[KG - 1][BM][BN];
  } sm;
  const int kg = threadIdx.x >> 6, tid = threadIdx.x & 63;
  const int tx = tid & 7, ty = tid >> 3;  // rows 8tx..8tx+7, tokens 4ty..4ty+3
  const int m0 = blockIdx.x * BM;
  const int rows = E + 1;
  const int slice = (H + gridDim.y - 1) / gridDim.y;
  const int s_beg = blockIdx.y * slice, s_end = min(H, s_beg + slice);
  const int kspan = (slice + KG - 1) / KG;
  const int kbeg = s_beg + kg * kspan, kend = min(s_end, kbeg + kspan);
  const int iters = (kspan + BK - 1) / BK;  // the same for every K-group (barriers inside)
  logits += (size_t)blockIdx.y * n * E;
  if (gate_logit) gate_logit += (size_t)blockIdx.y * n;
  float acc[4][8] = {};
  // the next step's tiles are fetched into registers while this step computes
  float4 ra[2], rb[4];
  auto fetch = [&](int k0) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {  // A: 32 tokens x 16 k = 128 float4
      const int v4 = tid + 64 * q;
      const int r = v4 >> 2, kk = (v4 & 3) * 4;
      ra[q] = (m0 + r < n && k0 + kk < kend) ? load4(h + (size_t)(m0 + r) * H + k0 + kk)
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // B: 64 rows x 16 k = 256 float4
      const int v4 = tid + 64 * q;
      const int r = v4 >> 2, kk = (v4 & 3) * 4;
      rb[q] = (r < rows && k0 + kk < kend)
                  ? *reinterpret_cast<const float4*>((r < E ? wr + (size_t)r * H : wg) + k0 + kk)
                  : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  fetch(kbeg);
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int v4 = tid + 64 * q;
      const int r = v4 >> 2, kk = (v4 & 3) * 4;
      sm.t.A[kg][kk + 0][r] = ra[q].x;
      sm.t.A[kg][kk + 1][r] = ra[q].y;
      sm.t.A[kg][kk + 2][r] = ra[q].z;
      sm.t.A[kg][kk + 3][r] = ra[q].w;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int v4 = tid + 64 * q;
      const int r = v4 >> 2, kk = (v4 & 3) * 4;
      sm.t.B[kg][kk + 0][r] = rb[q].x;
      sm.t.B[kg][kk + 1][r] = rb[q].y;
      sm.t.B[kg][kk + 2][r] = rb[q].z;
      sm.t.B[kg][kk + 3][r] = rb[q].w;
    }
    __syncthreads();
    if (it + 1 < iters) fetch(kbeg + (it + 1) * BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&sm.t.A[kg][kk][ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&sm.t.B[kg][kk][tx * 8]);
      const float4 b1 = *reinterpret_cast<const float4*>(&sm.t.B[kg][kk][tx * 8 + 4]);
      const float av[4] = {a.x, a.y, a.z, a.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
  if (kg > 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) sm.red[kg - 1][ty * 4 + i][tx * 8 + j] = acc[i][j];
  }
  __syncthreads();
  if (kg != 0) return;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = m0 + ty * 4 + i;
    if (t >= n) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int r = tx * 8 + j;
      float v = acc[i][j];
#pragma unroll
      for (int g = 0; g < KG - 1; ++g) v += sm.red[g][ty * 4 + i][r];
      if (r < E)
        logits[(size_t)t * E + r] = v;
      else if (r == E && gate_logit)
        gate_logit[t] = v;
    }
  }
}

// One warp per token over logits summed from `nparts` K-slice partials.
template <int kPer>
__global__ void __launch_bounds__(256) router_topk_kernel(TopkArgs a, int n, int E, int k) {
  chain_wait();
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (t >= n) return;
  topk_token<kPer>(a, n, E, k, t, threadIdx.x & 31);
}

__global__ void __launch_bounds__(256) gate_sigmoid_kernel(const float* __restrict__ gate_logit, int nparts, int n,
                                                           float* __restrict__ gate_sig) {
  chain_wait();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n) return;
  float gl = gate_logit[t];
  for (int p = 1; p < nparts; ++p) gl += gate_logit[(size_t)p * n + t];  // slices in order, as the top-k kernel
  gate_sig[t] = sigmoid_f(gl);
}

int launch_gate_sigmoid(const float* gate_logit, int nparts, int n, float* gate_sig, cudaStream_t st) {
  if (n <= 0) return ER_OK;
  return launch_chained(gate_sigmoid_kernel, dim3((n + 255) / 256), dim3(256), 0, st, "gate_sigmoid_kernel",
                        gate_logit, nparts, n, gate_sig);
}

int launch_router_logits(const void* h, int h_dtype, int n, int H, const float* wr, const float* wg, int E,
                         float* logits, float* gate_logit, int* nparts, int* tally, int ntally, cudaStream_t st) {
  *nparts = 1;
  if (n <= 0) return ER_OK;
  // E == 0: only the shared-gate row (the caller supplies router logits)
  if (n <= 64 || E + 1 > 64) {
    if (h_dtype == ER_DTYPE_BF16)
      return launch_chained(router_rows_kernel<__nv_bfloat16>, dim3(E + 1), dim3(256), 0, st, "router_rows_kernel",
                            (const __nv_bfloat16*)h, n, H, wr, wg, E, logits, gate_logit, tally, ntally);
    return launch_chained(router_rows_kernel<float>, dim3(E + 1), dim3(256), 0, st, "router_rows_kernel",
                          (const float*)h, n, H, wr, wg, E, logits, gate_logit, tally, ntally);
  }
  *nparts = kRouterKSplit;
  const dim3 grid((n + 31) / 32, kRouterKSplit);
  if (h_dtype == ER_DTYPE_BF16)
    return launch_chained(router_gemm_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, "router_gemm_kernel",
                          (const __nv_bfloat16*)h, n, H, wr, wg, E, logits, gate_logit, tally, ntally);
  return launch_chained(router_gemm_kernel<float>, grid, dim3(256), 0, st, "router_gemm_kernel", (const float*)h, n, H,
                        wr, wg, E, logits, gate_logit, tally, ntally);
}

int launch_router_topk(const TopkArgs& a, int n, int E, int k, cudaStream_t st) {
  if (n <= 0) return ER_OK;
  const int warps_per_block = 8;
  const int blocks = (n + warps_per_block - 1) / warps_per_block;
  if (E <= 64)
    return launch_chained(router_topk_kernel<2>, dim3(blocks), dim3(warps_per_block * 32), 0, st,
                          "router_topk_kernel", a, n, E, k);
  return launch_chained(router_topk_kernel<kMaxExperts / 32>, dim3(blocks), dim3(warps_per_block * 32), 0, st,
                        "router_topk_kernel", a, n, E, k);
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
  TopkArgs a{};
  a.logits = logits;
  a.nparts = 1;
  a.gparts = 1;
  a.idx64 = idx64;
  a.idx32 = idx32;
  a.wout = probs_out;
  return launch_router_topk(a, n, num_experts, k, (cudaStream_t)stream);
}
