// er_gemm_simt.cu -- grouped expert GEMM on the fp32 FMA pipes (exact-fp32 path).
//
// Reference: runtime/qwen_moe.py:341-348 and 353-357 with the "blocked"
// kernels runtime/int8_linear.py:129-138 (int8 -> fp32 block, matmul, then
// out *= scales) and runtime/int4_linear.py:110-119 (nibbles -> (code - 8) *
// fp16 group scale in fp32, then matmul). Same operand values as the
// reference: int8 codes multiply fp32 activations and the row scale is
// applied to the accumulated output; int4 weights are dequantized exactly to
// fp32 before the product.
//
// Work item = one BM x BN output tile of one group (see the plan in er_plan.cu).
// mode 0: A = h rows gathered through the expert-sorted token list,
//         B = gate and up rows; epilogue act = silu(g * s_g) * (u * s_u).
// mode 1: A = act rows, B = down rows; epilogue y = acc * s_d * routing weight.
#include "er_internal.cuh"

namespace er {

template <int FMT, int MODE, typename XT>
__global__ void __launch_bounds__(256) gemm_simt_kernel(GroupArgs a, int sched, const XT* __restrict__ x,
                                                        float* act_r,
                                                        float* act_s, float* __restrict__ out_r,
                                                        float* __restrict__ out_s) {
  constexpr int BM = kSimtBM, BN = kSimtBN, BK = 16;
  constexpr int NB = MODE == 0 ? 2 : 1;
  constexpr bool kInt8 = (FMT == ER_FMT_INT8);
  __shared__ __align__(16) float As[BK][BM + 4];
  __shared__ __align__(16) float Bs[NB][BK][BN + 4];
  chain_wait();
  const Plan* P = a.plan;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int lrow = tid >> 2, lk = (tid & 3) * 4;  // load mapping: row 0..63, k 0,4,8,12
  const int total = P->item_start[sched][P->num_active];
  for (int item = blockIdx.x; item < total; item += gridDim.x) {
    int local = 0;
    const int g = find_item(P, sched, item, &local);
    if (g < 0) break;
    const GroupView v = group_view(a, g);
    if (v.fmt != FMT) continue;
    const RecordGeom geo{v.fmt, a.H, v.inter, a.group};
    const int K = MODE == 0 ? a.H : v.inter;
    const int units = MODE == 0 ? v.inter : a.H;
    const int ntiles = (units + BN - 1) / BN;
    const int m0 = (local / ntiles) * BM, n0 = (local % ntiles) * BN;
    const int ngroups = kInt8 ? 1 : K / a.group;

    // A source row for this thread's load slot
    const bool a_ok = m0 + lrow < v.rows;
    const XT* asrc_x = nullptr;
    const float* asrc_f = nullptr;
    if (a_ok) {
      if (MODE == 0) {
        const int tok = v.shared ? m0 + lrow : a.perm_token[v.row0 + m0 + lrow];
        asrc_x = x + (size_t)tok * a.H;
      } else {
        asrc_f = v.shared ? act_s + (size_t)(m0 + lrow) * v.inter : act_r + (size_t)(v.row0 + m0 + lrow) * a.I;
      }
    }
    const int brow = n0 + lrow;
    const bool b_ok = brow < units;

    float acc[NB][4][4];
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[b][i][j] = 0.f;

    for (int k0 = 0; k0 < K; k0 += BK) {
      float4 av = make_float4(0.f, 0.f, 0.f, 0.f);
      if (a_ok) av = MODE == 0 ? load4(asrc_x + k0 + lk) : *reinterpret_cast<const float4*>(asrc_f + k0 + lk);
      As[lk + 0][lrow] = av.x;
      As[lk + 1][lrow] = av.y;
      As[lk + 2][lrow] = av.z;
      As[lk + 3][lrow] = av.w;
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const int which = MODE == 0 ? b : 2;
        float f[4] = {0.f, 0.f, 0.f, 0.f};
        if (b_ok) {
          if (kInt8) {
            const uint32_t w4 =
                *reinterpret_cast<const uint32_t*>(v.rec + geo.weight_offset(which) + (size_t)brow * K + k0 + lk);
            i8x4_to_f32(w4, f);
          } else {
            const uint16_t w2 = *reinterpret_cast<const uint16_t*>(v.rec + geo.weight_offset(which) +
                                                                   (size_t)brow * (K / 2) + (k0 + lk) / 2);
            const size_t gidx = (size_t)brow * ngroups + (k0 + lk) / a.group;
            const float s = half_bits_to_f32(reinterpret_cast<const uint16_t*>(v.rec + geo.scale_offset(which))[gidx]);
            const float z = FMT == ER_FMT_INT4_ZP ? (float)(v.rec + geo.zero_offset(which))[gidx] : 8.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) f[j] = ((float)((w2 >> (4 * j)) & 0xf) - z) * s;
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) Bs[b][lk + j][lrow] = f[j];
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < BK; ++kk) {
        const float4 a4 = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
        const float ar[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const float4 b4 = *reinterpret_cast<const float4*>(&Bs[b][kk][tx * 4]);
          const float br[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[b][i][j] = fmaf(ar[i], br[j], acc[b][i][j]);
        }
      }
      __syncthreads();
    }

    // epilogue
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = m0 + ty * 4 + i;
      if (r >= v.rows) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = n0 + tx * 4 + j;
        if (c >= units) continue;
        if (MODE == 0) {
          float gv = acc[0][i][j], uv = acc[1][i][j];
          if (kInt8) {
            gv *= reinterpret_cast<const float*>(v.rec + geo.scale_offset(0))[c];
            uv *= reinterpret_cast<const float*>(v.rec + geo.scale_offset(1))[c];
          }
          float* dst = v.shared ? act_s + (size_t)r * v.inter : act_r + (size_t)(v.row0 + r) * a.I;
          dst[c] = silu_f(gv) * uv;
        } else {
          float yv = acc[0][i][j];
          if (kInt8) yv *= reinterpret_cast<const float*>(v.rec + geo.scale_offset(2))[c];
          if (v.shared)
            out_s[(size_t)r * a.H + c] = yv * a.gate_sig[r];
          else
            out_r[(size_t)(v.row0 + r) * a.H + c] = yv * a.perm_w[v.row0 + r];
        }
      }
    }
  }
}

template <int MODE, typename XT>
static int launch_simt_fmt(const GroupArgs& a, int sched, const XT* x, float* act_r, float* act_s,
                           float* out_r, float* out_s, int grid, cudaStream_t st) {
  if (int rc = launch_chained(gemm_simt_kernel<ER_FMT_INT8, MODE, XT>, dim3(grid), dim3(256), 0, st,
                              "gemm_simt_kernel<int8>", a, sched, x, act_r, act_s, out_r, out_s))
    return rc;
  if (a.fmt == ER_FMT_INT4)
    return launch_chained(gemm_simt_kernel<ER_FMT_INT4, MODE, XT>, dim3(grid), dim3(256), 0, st,
                          "gemm_simt_kernel<int4>", a, sched, x, act_r, act_s, out_r, out_s);
  if (a.fmt == ER_FMT_INT4_ZP)
    return launch_chained(gemm_simt_kernel<ER_FMT_INT4_ZP, MODE, XT>, dim3(grid), dim3(256), 0, st,
                          "gemm_simt_kernel<int4zp>", a, sched, x, act_r, act_s, out_r, out_s);
  return ER_OK;
}

int launch_gemm_simt_grouped(const GroupArgs& a, int sched, int mode, const void* x, int x_dtype,
                             float* act_r, float* act_s, float* out_r, float* out_s,
                             long long items_bound, cudaStream_t st) {
  if (items_bound <= 0) return ER_OK;
  const int grid = (int)(items_bound < 1048576 ? items_bound : 1048576);
  if (mode == 0) {
    if (x_dtype == ER_DTYPE_BF16)
      return launch_simt_fmt<0, __nv_bfloat16>(a, sched, (const __nv_bfloat16*)x, act_r, act_s, out_r, out_s,
                                               grid, st);
    return launch_simt_fmt<0, float>(a, sched, (const float*)x, act_r, act_s, out_r, out_s, grid, st);
  }
  return launch_simt_fmt<1, float>(a, sched, nullptr, act_r, act_s, out_r, out_s, grid, st);
}

// out[t] = sum over the token's k routed outputs in ascending expert id (the
// reference accumulates experts in that order, runtime/qwen_moe.py:341-349)
// + the gated shared-expert output (:359), itself the sum of `parts` partial
// rows in order. y_s may be NULL (no shared term); error (optional): nonzero
// turns the rows into NaN, and so does a slot without a position.
// CTA (t, y): 128 threads of token t, one float4 column each per step over
// columns y*512 + j*gridDim.y*512. The slots' order is ranked once per CTA;
// every thread issues all of a column's loads before adding them, so a step
// costs one round of memory latency. KMAX / PMAX bound k and parts.
constexpr int kCombineThreads = 128;
constexpr int kCombineMaxParts = 8;

// RT / OT: the row results' and the output's element type (float or bf16; the
// sums are fp32 either way).
__device__ __forceinline__ float4 load_f4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 load_f4(const __nv_bfloat16* p) { return load4(p); }
__device__ __forceinline__ void store_f4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void store_f4(__nv_bfloat16* p, float4 v) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t*>(&a);
  u.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

template <int KMAX, int PMAX, typename RT, typename OT>
__global__ void __launch_bounds__(kCombineThreads) combine_kernel(const RT* __restrict__ y_r,
                                                                  const float* __restrict__ y_s, int parts,
                                                                  const int32_t* __restrict__ pos_of,
                                                                  const int32_t* __restrict__ idx, int n, int k,
                                                                  int H, const int* __restrict__ error,
                                                                  OT* __restrict__ out) {
  __shared__ int pos_sorted[KMAX];
  chain_wait();
  const int t = blockIdx.x;
  if (threadIdx.x < k) {
    // rank of slot s: slots with a smaller expert id, or the same id and a smaller slot, come first
    const int s = threadIdx.x;
    const int e = idx[(size_t)t * k + s];
    int rank = 0;
    for (int j = 0; j < k; ++j) {
      const int ej = idx[(size_t)t * k + j];
      rank += (ej < e) || (ej == e && j < s);
    }
    pos_sorted[rank] = pos_of[(size_t)t * k + s];
  }
  __syncthreads();
  const float nan = __int_as_float(0x7fc00000);
  const bool failed = error && *error;
  int pos[KMAX];
  bool missing = false;
#pragma unroll
  for (int s = 0; s < KMAX; ++s) {
    pos[s] = s < k ? pos_sorted[s] : 0;
    missing |= s < k && pos[s] < 0;
  }
  const int step = gridDim.y * kCombineThreads * 4;
  for (int c = (blockIdx.y * kCombineThreads + threadIdx.x) * 4; c < H; c += step) {
    OT* dst = out + (size_t)t * H + c;
    if (failed || missing) {
      store_f4(dst, make_float4(nan, nan, nan, nan));
      continue;
    }
    float4 v[KMAX], sv[PMAX];
#pragma unroll
    for (int s = 0; s < KMAX; ++s)
      if (s < k) v[s] = load_f4(y_r + (size_t)pos[s] * H + c);
    if (y_s) {
#pragma unroll
      for (int q = 0; q < PMAX; ++q)
        if (q < parts) sv[q] = *reinterpret_cast<const float4*>(y_s + ((size_t)q * n + t) * H + c);
    }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int s = 0; s < KMAX; ++s) {
      if (s < k) {
        acc.x += v[s].x;
        acc.y += v[s].y;
        acc.z += v[s].z;
        acc.w += v[s].w;
      }
    }
    if (y_s) {
      float4 sh = sv[0];
#pragma unroll
      for (int q = 1; q < PMAX; ++q) {
        if (q < parts) {
          sh.x += sv[q].x;
          sh.y += sv[q].y;
          sh.z += sv[q].z;
          sh.w += sv[q].w;
        }
      }
      acc.x += sh.x;
      acc.y += sh.y;
      acc.z += sh.z;
      acc.w += sh.w;
    }
    store_f4(dst, acc);
  }
}

template <int KMAX, typename RT, typename OT>
static int launch_combine_k(const RT* y_r, const float* y_s, int parts, const int32_t* pos_of, const int32_t* idx,
                            int n, int k, int H, const int* error, OT* out, dim3 grid, cudaStream_t st) {
  if (parts <= 1)
    return launch_chained(combine_kernel<KMAX, 1, RT, OT>, grid, dim3(kCombineThreads), 0, st, "combine_kernel", y_r,
                          y_s, parts, pos_of, idx, n, k, H, error, out);
  if (parts <= 4)
    return launch_chained(combine_kernel<KMAX, 4, RT, OT>, grid, dim3(kCombineThreads), 0, st, "combine_kernel", y_r,
                          y_s, parts, pos_of, idx, n, k, H, error, out);
  return launch_chained(combine_kernel<KMAX, kCombineMaxParts, RT, OT>, grid, dim3(kCombineThreads), 0, st,
                        "combine_kernel", y_r, y_s, parts, pos_of, idx, n, k, H, error, out);
}

template <typename RT, typename OT>
static int launch_combine_t(const RT* y_r, const float* y_s, int parts, const int32_t* pos_of, const int32_t* idx,
                            int n, int k, int H, const int* error, OT* out, cudaStream_t st) {
  if (n <= 0) return ER_OK;
  if (parts < 1 || parts > kCombineMaxParts) return fail(ER_EINVAL, "combine: %d shared parts", parts);
  // a few tokens: their columns spread over CTAs; many: one CTA per token row
  const int col_blocks = (H / 4 + kCombineThreads - 1) / kCombineThreads;
  const dim3 grid(n, n >= 2 * 148 ? 1 : col_blocks);
  if (k <= 4) return launch_combine_k<4>(y_r, y_s, parts, pos_of, idx, n, k, H, error, out, grid, st);
  return launch_combine_k<kMaxTopK>(y_r, y_s, parts, pos_of, idx, n, k, H, error, out, grid, st);
}

int launch_combine(const float* y_r, const float* y_s, int parts, const int32_t* pos_of, const int32_t* idx, int n,
                   int k, int H, const int* error, float* out, cudaStream_t st) {
  return launch_combine_t(y_r, y_s, parts, pos_of, idx, n, k, H, error, out, st);
}

int launch_combine_dt(const void* y_r, int r_dtype, const float* y_s, int parts, const int32_t* pos_of,
                      const int32_t* idx, int n, int k, int H, const int* error, void* out, int o_dtype,
                      cudaStream_t st) {
  const bool rb = r_dtype == ER_DTYPE_BF16, ob = o_dtype == ER_DTYPE_BF16;
  if (!rb && !ob)
    return launch_combine_t((const float*)y_r, y_s, parts, pos_of, idx, n, k, H, error, (float*)out, st);
  if (rb && !ob)
    return launch_combine_t((const __nv_bfloat16*)y_r, y_s, parts, pos_of, idx, n, k, H, error, (float*)out, st);
  if (!rb && ob)
    return launch_combine_t((const float*)y_r, y_s, parts, pos_of, idx, n, k, H, error, (__nv_bfloat16*)out, st);
  return fail(ER_EINVAL, "combine: bf16 rows into a bf16 output is not provided");
}

}  // namespace er
