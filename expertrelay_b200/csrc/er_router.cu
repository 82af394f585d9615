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
  chain_trigger();  // the dispatch kernel, and through it the gate/up GEMM, may start meanwhile
  chain_wait();
  constexpr int kTok = kRouterTok;
  if (blockIdx.x == 0 && tally)  // cleared for the top-k kernel's per-expert counts
    for (int i = threadIdx.x; i < ntally; i += blockDim.x) tally[i] = 0;
  __shared__ float red[8][kTok];
  const int r = blockIdx.x;  // grid: E rows, plus the shared-gate row when wg is given
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

// Large batches: a tiled fp32 GEMM over [W_r; w_g] (E + 1 <= 64 rows; the
// shared-gate row only when wg is given). A CTA of 128 threads computes 128
// tokens x 64 rows over one of gridDim.y K slices and writes that slice's
// partial logits (the top-k kernel adds the slices in a fixed order). Each
// thread holds an 8-token x 8-row register tile, so a 32-deep K step costs it
// 4 shared-memory vector loads per 64 FMAs; the next step's tiles are fetched
// into registers while this one computes.
constexpr int kRgThreads = 128, kRgBM = 128, kRgBN = 64, kRgBK = 32;

template <typename XT>
__global__ void __launch_bounds__(kRgThreads) router_gemm_kernel(const XT* __restrict__ h, int n, int H,
                                                                 const float* __restrict__ wr,
                                                                 const float* __restrict__ wg, int E,
                                                                 float* __restrict__ logits,
                                                                 float* __restrict__ gate_logit,
                                                                 int* __restrict__ tally, int ntally) {
  chain_wait();
  if (blockIdx.x == 0 && blockIdx.y == 0 && tally)  // cleared for the top-k kernel's per-expert counts
    for (int i = threadIdx.x; i < ntally; i += blockDim.x) tally[i] = 0;
  __shared__ __align__(16) float As[kRgBK][kRgBM];  // [k][token]
  __shared__ __align__(16) float Bs[kRgBK][kRgBN];  // [k][row]
  const int tid = threadIdx.x;
  const int tx = tid & 7, ty = tid >> 3;  // rows 8 tx .. +7, tokens 8 ty .. +7
  const int m0 = blockIdx.x * kRgBM;
  const int rows = E + (wg ? 1 : 0);
  // K slices in whole 32-wide steps (so every float4 stays inside a row)
  const int slice = ((H + gridDim.y - 1) / gridDim.y + kRgBK - 1) / kRgBK * kRgBK;
  const int kbeg = blockIdx.y * slice, kend = min(H, kbeg + slice);
  logits += (size_t)blockIdx.y * n * E;
  if (gate_logit) gate_logit += (size_t)blockIdx.y * n;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  // A: 128 tokens x 32 k = 1024 float4, thread t holds token t's k 4q .. 4q + 3 (q < 8);
  // B: 64 rows x 32 k = 512 float4, thread t holds row t % 64's k 4 (2q + t / 64) .. (q < 4).
  // Consecutive lanes store consecutive tokens / rows: no bank conflicts.
  float4 ra[8], rb[4];
  const int brow = tid & 63, bk = (tid >> 6) * 4;
  const bool a_ok = m0 + tid < n, b_ok = brow < rows;
  const XT* arow = h + (size_t)(a_ok ? m0 + tid : 0) * H;
  const float* brow_p = b_ok ? (brow < E ? wr + (size_t)brow * H : wg) : wr;
  auto fetch = [&](int k0) {
#pragma unroll
    for (int q = 0; q < 8; ++q)
      ra[q] = (a_ok && k0 + 4 * q < kend) ? load4(arow + k0 + 4 * q) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int kk = 8 * q + bk;
      rb[q] = (b_ok && k0 + kk < kend) ? *reinterpret_cast<const float4*>(brow_p + k0 + kk)
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  fetch(kbeg);
  for (int k0 = kbeg; k0 < kend; k0 += kRgBK) {
    __syncthreads();  // the previous step's tiles are no longer read
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      As[4 * q + 0][tid] = ra[q].x;
      As[4 * q + 1][tid] = ra[q].y;
      As[4 * q + 2][tid] = ra[q].z;
      As[4 * q + 3][tid] = ra[q].w;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int kk = 8 * q + bk;
      Bs[kk + 0][brow] = rb[q].x;
      Bs[kk + 1][brow] = rb[q].y;
      Bs[kk + 2][brow] = rb[q].z;
      Bs[kk + 3][brow] = rb[q].w;
    }
    __syncthreads();
    if (k0 + kRgBK < kend) fetch(k0 + kRgBK);
#pragma unroll
    for (int kk = 0; kk < kRgBK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[kk][ty * 8]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[kk][ty * 8 + 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[kk][tx * 8]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[kk][tx * 8 + 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int t = m0 + ty * 8 + i;
    if (t >= n) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int r = tx * 8 + j;
      if (r < E)
        logits[(size_t)t * E + r] = acc[i][j];
      else if (r == E && gate_logit)
        gate_logit[t] = acc[i][j];
    }
  }
}

// One warp per token over logits summed from `nparts` K-slice partials. The
// per-expert tallies are counted in shared memory and added to the plan's
// once per CTA and expert: a popular expert (hundreds of tokens under Zipf
// routing) would otherwise take one global atomic per token, serialised on
// one address.
template <int kPer>
__global__ void __launch_bounds__(512) router_topk_kernel(TopkArgs a, int n, int E, int k) {
  __shared__ int stally[kMaxExperts];
  int* const gtally = a.tally;  // the same for the whole CTA
  if (gtally) {
    for (int e = threadIdx.x; e < E; e += blockDim.x) stally[e] = 0;
    __syncthreads();
    a.tally = stally;
  }
  chain_wait();
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (t < n) topk_token<kPer>(a, n, E, k, t, threadIdx.x & 31);
  if (gtally) {
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x)
      if (stally[e]) atomicAdd(&gtally[e], stally[e]);
  }
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
                         float* logits, float* gate_logit, int* nparts, int* tally, int ntally, cudaStream_t st,
                         int* error) {
  *nparts = 1;
  if (n <= 0) return ER_OK;
  // E == 0: only the shared-gate row (the caller supplies router logits); wg
  // NULL: only the router rows
  const int rows = E + (wg ? 1 : 0);
  if (rows <= 0) return ER_OK;
  if (H % 4) return fail(ER_EINVAL, "router: hidden %d must be a multiple of 4", H);
  static_assert(kRgBN == 64, "router_parts() assumes 64-row tiles");
  if (router_parts(n, rows) == 1) {
    if (h_dtype == ER_DTYPE_BF16)
      return launch_chained(router_rows_kernel<__nv_bfloat16>, dim3(rows), dim3(256), 0, st, "router_rows_kernel",
                            (const __nv_bfloat16*)h, n, H, wr, wg, E, logits, gate_logit, tally, ntally);
    return launch_chained(router_rows_kernel<float>, dim3(rows), dim3(256), 0, st, "router_rows_kernel",
                          (const float*)h, n, H, wr, wg, E, logits, gate_logit, tally, ntally);
  }
  *nparts = kRouterKSplit;
  if (router_tc_ok(n, H, E, wr, wg))
    return launch_router_tc(h, h_dtype, n, H, wr, wg, E, logits, gate_logit, tally, ntally, error, st);
  const dim3 grid((n + kRgBM - 1) / kRgBM, kRouterKSplit);
  if (h_dtype == ER_DTYPE_BF16)
    return launch_chained(router_gemm_kernel<__nv_bfloat16>, grid, dim3(kRgThreads), 0, st, "router_gemm_kernel",
                          (const __nv_bfloat16*)h, n, H, wr, wg, E, logits, gate_logit, tally, ntally);
  return launch_chained(router_gemm_kernel<float>, grid, dim3(kRgThreads), 0, st, "router_gemm_kernel",
                        (const float*)h, n, H, wr, wg, E, logits, gate_logit, tally, ntally);
}

int launch_router_topk(const TopkArgs& a, int n, int E, int k, cudaStream_t st) {
  if (n <= 0) return ER_OK;
  const int warps_per_block = 16;
  const int blocks = (n + warps_per_block - 1) / warps_per_block;
  if (E <= 64)
    return launch_chained(router_topk_kernel<2>, dim3(blocks), dim3(warps_per_block * 32), 0, st,
                          "router_topk_kernel", a, n, E, k);
  return launch_chained(router_topk_kernel<kMaxExperts / 32>, dim3(blocks), dim3(warps_per_block * 32), 0, st,
                        "router_topk_kernel", a, n, E, k);
}


}  // namespace er

extern "C" size_t er_route_scratch_bytes(int n, int num_experts) {
  return n < 0 || num_experts < 1 ? 0 : (size_t)er::router_parts(n, num_experts) * n * num_experts * sizeof(float);
}

extern "C" int er_route(const void* h, int h_dtype, int n, int hidden, const float* router_w, int num_experts, int k,
                        int norm_topk_prob, float* scratch, size_t scratch_bytes, float* logits_out, int32_t* idx32,
                        float* w_out, void* stream) {
  using namespace er;
  if (n < 0 || hidden <= 0 || hidden % 4 || num_experts < 1 || num_experts > kMaxExperts || k < 1 || k > kMaxTopK ||
      k > num_experts)
    return fail(ER_EINVAL, "er_route: n %d, hidden %d (a multiple of 4), experts %d, k %d", n, hidden, num_experts, k);
  if (h_dtype != ER_DTYPE_F32 && h_dtype != ER_DTYPE_BF16) return fail(ER_EINVAL, "er_route: dtype %d", h_dtype);
  if (n == 0) return ER_OK;
  if (!h || !router_w || !scratch || !idx32 || !w_out) return fail(ER_EINVAL, "er_route: null argument");
  if (((uintptr_t)h | (uintptr_t)router_w) & 15) return fail(ER_EINVAL, "er_route: h and the router must be aligned");
  if (scratch_bytes < er_route_scratch_bytes(n, num_experts))
    return fail(ER_ENOSPACE, "er_route: scratch %zu bytes, need %zu", scratch_bytes, er_route_scratch_bytes(n, num_experts));
  cudaStream_t st = (cudaStream_t)stream;
  int nparts = 1;
  if (int rc = launch_router_logits(h, h_dtype, n, hidden, router_w, nullptr, num_experts, scratch, nullptr, &nparts,
                                    nullptr, 0, st))
    return rc;
  TopkArgs a{};
  a.logits = scratch;
  a.nparts = nparts;
  a.gparts = 0;
  a.norm = norm_topk_prob;
  a.idx32 = idx32;
  a.wout = w_out;
  a.logits_sum = logits_out;
  return launch_router_topk(a, n, num_experts, k, st);
}

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
