// er_ep.cu -- send buffers of the expert-parallel exchange.
//
// With experts spread over ranks, each routed (token, slot) pair of a rank's
// tokens is computed by the rank holding its expert: the pairs are grouped by
// destination rank, their token rows copied into one contiguous send buffer
// (each destination's rows one range of it) for an all-to-all, and pos_of
// remembers where pair (t, j) went, so the combine can find its result in the
// buffer that comes back. One warp per token claims positions with an atomic
// cursor per destination, like the block's dispatch.
#include "er_internal.cuh"

namespace er {

__global__ void __launch_bounds__(256) ep_count_kernel(const int32_t* __restrict__ idx, int nk,
                                                       const int32_t* __restrict__ owner, int E, int ranks,
                                                       int32_t* __restrict__ counts) {
  chain_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nk) return;
  const int e = idx[i];
  if (e < 0 || e >= E) return;
  const int r = owner[e];
  if (r >= 0 && r < ranks) atomicAdd(&counts[r], 1);
}

// One warp per token t: lane j < k claims slot j's position, then the warp
// copies h[t] (H elements of XT, 16 bytes per lane and step) to each claimed row.
template <typename XT>
__global__ void __launch_bounds__(256) ep_pack_kernel(const XT* __restrict__ h, int H, const int32_t* __restrict__ idx,
                                                      const float* __restrict__ w, int n, int k,
                                                      const int32_t* __restrict__ owner,
                                                      const int32_t* __restrict__ local, int E, int ranks,
                                                      const int32_t* __restrict__ offsets,
                                                      int32_t* __restrict__ cursor, XT* __restrict__ x_send,
                                                      int32_t* __restrict__ expert_send,
                                                      float* __restrict__ weight_send, int meta_stride,
                                                      int32_t* __restrict__ pos_of) {
  chain_wait();
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= n) return;
  int p = -1;
  if (lane < k) {
    const int e = idx[(size_t)t * k + lane];
    const int r = (e >= 0 && e < E) ? owner[e] : -1;
    if (r >= 0 && r < ranks) {
      p = offsets[r] + atomicAdd(&cursor[r], 1);
      expert_send[(size_t)p * meta_stride] = local[e];
      weight_send[(size_t)p * meta_stride] = w[(size_t)t * k + lane];
    }
    pos_of[(size_t)t * k + lane] = p;
  }
  constexpr int kVec = 16 / sizeof(XT);  // elements per 16-byte chunk
  const uint4* src = reinterpret_cast<const uint4*>(h + (size_t)t * H);
  const int chunks = H / kVec;
  for (int j = 0; j < k; ++j) {
    const int pj = __shfl_sync(0xffffffffu, p, j);
    if (pj < 0) continue;
    uint4* dst = reinterpret_cast<uint4*>(x_send + (size_t)pj * H);
    for (int c = lane; c < chunks; c += 32) dst[c] = src[c];
  }
}

}  // namespace er

using namespace er;

extern "C" int er_ep_count(const int32_t* idx, int n, int k, const int32_t* owner, int num_experts, int ranks,
                           int32_t* counts, void* stream) {
  if (n < 0 || k < 1 || k > kMaxTopK || num_experts < 1 || ranks < 1 || !counts || (n > 0 && (!idx || !owner)))
    return fail(ER_EINVAL, "er_ep_count: bad arguments (n %d, k %d, experts %d, ranks %d)", n, k, num_experts, ranks);
  cudaStream_t st = (cudaStream_t)stream;
  if (int rc = cuda_check(cudaMemsetAsync(counts, 0, (size_t)ranks * sizeof(int32_t), st), "er_ep_count: clear"))
    return rc;
  const int nk = n * k;
  if (nk == 0) return ER_OK;
  return launch_chained(ep_count_kernel, dim3((nk + 255) / 256), dim3(256), 0, st, "ep_count_kernel", idx, nk, owner,
                        num_experts, ranks, counts);
}

extern "C" int er_ep_pack(const void* h, int h_dtype, int hidden, const int32_t* idx, const float* w, int n, int k,
                          const int32_t* owner, const int32_t* local, int num_experts, int ranks,
                          const int32_t* offsets, int32_t* cursor, void* x_send, int32_t* expert_send,
                          float* weight_send, int meta_stride, int32_t* pos_of, void* stream) {
  if (n < 0 || k < 1 || k > kMaxTopK || num_experts < 1 || ranks < 1 || hidden <= 0)
    return fail(ER_EINVAL, "er_ep_pack: bad sizes (n %d, k %d, experts %d, ranks %d, hidden %d)", n, k, num_experts,
                ranks, hidden);
  if (h_dtype != ER_DTYPE_F32 && h_dtype != ER_DTYPE_BF16) return fail(ER_EINVAL, "er_ep_pack: dtype %d", h_dtype);
  if (meta_stride < 1) return fail(ER_EINVAL, "er_ep_pack: meta stride %d", meta_stride);
  const int vec = h_dtype == ER_DTYPE_F32 ? 4 : 8;
  if (hidden % vec || ((uintptr_t)h | (uintptr_t)x_send) & 15)
    return fail(ER_EINVAL, "er_ep_pack: rows must be 16-byte aligned and a multiple of 16 bytes");
  if (n == 0) return ER_OK;
  if (!h || !idx || !w || !owner || !local || !offsets || !cursor || !x_send || !expert_send || !weight_send || !pos_of)
    return fail(ER_EINVAL, "er_ep_pack: null argument");
  cudaStream_t st = (cudaStream_t)stream;
  if (int rc = cuda_check(cudaMemsetAsync(cursor, 0, (size_t)ranks * sizeof(int32_t), st), "er_ep_pack: clear"))
    return rc;
  const int blocks = (n + 7) / 8;
  if (h_dtype == ER_DTYPE_BF16)
    return launch_chained(ep_pack_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, st, "ep_pack_kernel",
                          (const __nv_bfloat16*)h, hidden, idx, w, n, k, owner, local, num_experts, ranks, offsets,
                          cursor, (__nv_bfloat16*)x_send, expert_send, weight_send, meta_stride, pos_of);
  return launch_chained(ep_pack_kernel<float>, dim3(blocks), dim3(256), 0, st, "ep_pack_kernel", (const float*)h,
                        hidden, idx, w, n, k, owner, local, num_experts, ranks, offsets, cursor, (float*)x_send,
                        expert_send, weight_send, meta_stride, pos_of);
}
