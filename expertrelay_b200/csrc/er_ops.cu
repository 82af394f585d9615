// er_ops.cu -- the Backend-protocol ops (runtime/backends.py:44-67) as
// standalone C entry points, the weight reconstruction kernels, error
// plumbing and record-layout queries.
#include <stdarg.h>
#include <stdio.h>

#include "er_internal.cuh"

namespace er {

static thread_local char g_err[1024] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return ER_OK;
  return fail(ER_ECUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

// ---------------------------------------------------------------------------
// generic tiled linear: y[m, out] = x[m, in] @ W^T (+ bias)
// WT 0: W fp32; 1: W int8 with the row scale applied to the output
// (runtime/int8_linear.py:129-138); 2: W int4 dequantized exactly to fp32 as
// (code - zero) * fp16 scale (runtime/int4_linear.py:110-119). Any shape and
// input row stride; scalar loads with full bounds checks.
// ---------------------------------------------------------------------------
template <int WT>
__global__ void __launch_bounds__(256) linear_tiled_kernel(const float* __restrict__ x, long long ldx,
                                                           const void* __restrict__ w, const float* __restrict__ s8,
                                                           const uint16_t* __restrict__ s4,
                                                           const uint8_t* __restrict__ z4, int group,
                                                           const float* __restrict__ bias, float* __restrict__ y,
                                                           int m, int out, int in) {
  constexpr int BM = 64, BN = 64, BK = 16;
  __shared__ float As[BK][BM + 1];
  __shared__ float Bs[BK][BN + 1];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int ngroups = WT == 2 ? in / group : 1;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < in; k0 += BK) {
    for (int i = tid; i < BM * BK; i += 256) {
      const int r = i / BK, kk = i % BK;
      const int gr = m0 + r, gk = k0 + kk;
      As[kk][r] = (gr < m && gk < in) ? x[(size_t)gr * ldx + gk] : 0.f;
      const int gc = n0 + r;
      float bv = 0.f;
      if (gc < out && gk < in) {
        if (WT == 0) {
          bv = reinterpret_cast<const float*>(w)[(size_t)gc * in + gk];
        } else if (WT == 1) {
          bv = (float)reinterpret_cast<const int8_t*>(w)[(size_t)gc * in + gk];
        } else {
          const uint8_t byte = reinterpret_cast<const uint8_t*>(w)[(size_t)gc * (in / 2) + gk / 2];
          const int code = (gk & 1) ? (byte >> 4) : (byte & 0xf);
          const size_t gi = (size_t)gc * ngroups + gk / group;
          const float z = z4 ? (float)z4[gi] : 8.f;
          bv = ((float)code - z) * half_bits_to_f32(s4[gi]);
        }
      }
      Bs[kk][r] = bv;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float ar[4], br[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) ar[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) br[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = m0 + ty * 4 + i;
    if (r >= m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = n0 + tx * 4 + j;
      if (c >= out) continue;
      float v = acc[i][j];
      if (WT == 1) v *= s8[c];
      if (bias) v += bias[c];
      y[(size_t)r * out + c] = v;
    }
  }
}

template <int WT>
static int launch_linear(const float* x, long long ldx, const void* w, const float* s8, const uint16_t* s4,
                         const uint8_t* z4, int group, const float* bias, float* y, int m, int out, int in,
                         cudaStream_t st) {
  if (m == 0 || out == 0) return ER_OK;
  dim3 grid((out + 63) / 64, (m + 63) / 64);
  if (grid.y > 65535) return fail(ER_EINVAL, "linear: m %d too large", m);
  linear_tiled_kernel<WT><<<grid, 256, 0, st>>>(x, ldx, w, s8, s4, z4, group, bias, y, m, out, in);
  return launch_check("linear_tiled_kernel");
}

// ---------------------------------------------------------------------------
// int8 weight streaming for a few rows (decode): y[m, out] = (x @ Q^T) * s (+ b)
// Each warp owns R output rows (R = 4 for tall matrices such as the lm_head,
// 1 when that would leave SMs idle); each lane reads 16 codes of every one of
// them per step (16-byte loads, not kept in L1, all issued before the math),
// every row of x (m <= MT) from L1, and the warp sums its lanes at the end.
// The weights cross HBM once; x stays cached.
// ---------------------------------------------------------------------------
template <int MT, int kGemvRows>
__global__ void __launch_bounds__(256) int8_gemv_kernel(const float* __restrict__ x, long long ldx,
                                                        const int8_t* __restrict__ q, const float* __restrict__ s,
                                                        const float* __restrict__ bias, float* __restrict__ y,
                                                        int m, int out, int in) {
  const int row0 = (blockIdx.x * 8 + (threadIdx.x >> 5)) * kGemvRows;
  const int lane = threadIdx.x & 31;
  if (row0 >= out) return;
  float acc[kGemvRows][MT];
#pragma unroll
  for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
    for (int i = 0; i < MT; ++i) acc[r][i] = 0.f;
  for (int c = lane * 16; c < in; c += 32 * 16) {
    uint4 raw[kGemvRows];
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r)
      raw[r] = row0 + r < out ? ld_stream_u4(q + (size_t)(row0 + r) * in + c) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int i = 0; i < MT; ++i) {
      if (i < m) {
        const float4* xr = reinterpret_cast<const float4*>(x + (size_t)i * ldx + c);
        float xv[16];
#pragma unroll
        for (int j4 = 0; j4 < 4; ++j4) {
          const float4 v = __ldg(xr + j4);
          xv[4 * j4] = v.x;
          xv[4 * j4 + 1] = v.y;
          xv[4 * j4 + 2] = v.z;
          xv[4 * j4 + 3] = v.w;
        }
#pragma unroll
        for (int r = 0; r < kGemvRows; ++r) {
          const int8_t* b = reinterpret_cast<const int8_t*>(&raw[r]);
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[r][i] = fmaf((float)b[j], xv[j], acc[r][i]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kGemvRows; ++r) {
#pragma unroll
    for (int i = 0; i < MT; ++i) acc[r][i] = warp_sum(acc[r][i]);
    const int row = row0 + r;
    if (lane == 0 && row < out) {
      const float sc = s[row], bv = bias ? bias[row] : 0.f;
#pragma unroll
      for (int i = 0; i < MT; ++i)
        if (i < m) y[(size_t)i * out + row] = bias ? acc[r][i] * sc + bv : acc[r][i] * sc;
    }
  }
}

template <int R>
static void launch_int8_gemv_r(const float* x, long long ldx, const int8_t* q, const float* s, const float* bias,
                               float* y, int m, int out, int in, cudaStream_t st) {
  const dim3 grid((out + 8 * R - 1) / (8 * R)), block(256);
  if (m <= 1) int8_gemv_kernel<1, R><<<grid, block, 0, st>>>(x, ldx, q, s, bias, y, m, out, in);
  else if (m <= 2) int8_gemv_kernel<2, R><<<grid, block, 0, st>>>(x, ldx, q, s, bias, y, m, out, in);
  else if (m <= 4) int8_gemv_kernel<4, R><<<grid, block, 0, st>>>(x, ldx, q, s, bias, y, m, out, in);
  else int8_gemv_kernel<8, R><<<grid, block, 0, st>>>(x, ldx, q, s, bias, y, m, out, in);
}

static int launch_int8_gemv(const float* x, long long ldx, const int8_t* q, const float* s, const float* bias,
                            float* y, int m, int out, int in, cudaStream_t st) {
  // four rows per warp only while that still gives every SM several CTAs
  if (out >= 4 * 8 * 148 * 4)
    launch_int8_gemv_r<4>(x, ldx, q, s, bias, y, m, out, in, st);
  else
    launch_int8_gemv_r<1>(x, ldx, q, s, bias, y, m, out, in, st);
  return launch_check("int8_gemv_kernel");
}

// fp32 weights, a few rows: one warp per output row, x rows (m <= MT) from L1
template <int MT>
__global__ void __launch_bounds__(256) f32_gemv_kernel(const float* __restrict__ x, long long ldx,
                                                       const float* __restrict__ w, const float* __restrict__ bias,
                                                       float* __restrict__ y, int m, int out, int in) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= out) return;
  const float* wr = w + (size_t)row * in;
  float acc[MT];
#pragma unroll
  for (int i = 0; i < MT; ++i) acc[i] = 0.f;
  for (int c = lane * 4; c < in; c += 32 * 4) {
    const float4 wv = __ldg(reinterpret_cast<const float4*>(wr + c));
#pragma unroll
    for (int i = 0; i < MT; ++i) {
      if (i < m) {
        const float4 xv = __ldg(reinterpret_cast<const float4*>(x + (size_t)i * ldx + c));
        acc[i] = fmaf(wv.x, xv.x, fmaf(wv.y, xv.y, fmaf(wv.z, xv.z, fmaf(wv.w, xv.w, acc[i]))));
      }
    }
  }
#pragma unroll
  for (int i = 0; i < MT; ++i) acc[i] = warp_sum(acc[i]);
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < MT; ++i)
      if (i < m) y[(size_t)i * out + row] = bias ? acc[i] + bias[row] : acc[i];
  }
}

// fp32 weights, few output rows (a router: 60 x 2048), many input rows: CTA
// (o, chunk) holds weight row o in shared memory and gives each warp one
// input row at a time of its 64-row chunk.
__global__ void __launch_bounds__(256) f32_rows_kernel(const float* __restrict__ x, long long ldx,
                                                       const float* __restrict__ w, const float* __restrict__ bias,
                                                       float* __restrict__ y, int m, int out, int in) {
  extern __shared__ float wrow[];
  const int o = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int c = threadIdx.x * 4; c < in; c += blockDim.x * 4)
    *reinterpret_cast<float4*>(wrow + c) = __ldg(reinterpret_cast<const float4*>(w + (size_t)o * in + c));
  __syncthreads();
  const float b = bias ? bias[o] : 0.f;
  const int r_end = min(m, (int)(blockIdx.y + 1) * 64);
  for (int r = blockIdx.y * 64 + warp; r < r_end; r += 8) {
    const float* xr = x + (size_t)r * ldx;
    float acc = 0.f;
    for (int c = lane * 4; c < in; c += 32 * 4) {
      const float4 xv = __ldg(reinterpret_cast<const float4*>(xr + c));
      const float4 wv = *reinterpret_cast<const float4*>(wrow + c);
      acc = fmaf(wv.x, xv.x, fmaf(wv.y, xv.y, fmaf(wv.z, xv.z, fmaf(wv.w, xv.w, acc))));
    }
    acc = warp_sum(acc);
    if (lane == 0) y[(size_t)r * out + o] = acc + b;
  }
}

static int launch_f32_small(const float* x, long long ldx, const float* w, const float* bias, float* y, int m, int out,
                            int in, cudaStream_t st) {
  if (m <= 8) {
    const dim3 grid((out + 7) / 8), block(256);
    if (m <= 1) f32_gemv_kernel<1><<<grid, block, 0, st>>>(x, ldx, w, bias, y, m, out, in);
    else if (m <= 2) f32_gemv_kernel<2><<<grid, block, 0, st>>>(x, ldx, w, bias, y, m, out, in);
    else if (m <= 4) f32_gemv_kernel<4><<<grid, block, 0, st>>>(x, ldx, w, bias, y, m, out, in);
    else f32_gemv_kernel<8><<<grid, block, 0, st>>>(x, ldx, w, bias, y, m, out, in);
    return launch_check("f32_gemv_kernel");
  }
  const size_t smem = (size_t)in * sizeof(float);
  if (smem > 48 * 1024) {
    if (int rc = cuda_check(cudaFuncSetAttribute(f32_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem),
                            "f32 rows smem attribute"))
      return rc;
  }
  f32_rows_kernel<<<dim3(out, (m + 63) / 64), 256, smem, st>>>(x, ldx, w, bias, y, m, out, in);
  return launch_check("f32_rows_kernel");
}


static int check_linear_args(const char* name, const float* x, long long ldx, const void* w, float* y, int m, int out,
                             int in) {
  if (m < 0 || out < 0 || in < 0) return fail(ER_EINVAL, "%s: negative size", name);
  if ((m > 0 && in > 0 && !x) || (out > 0 && in > 0 && !w) || (m > 0 && out > 0 && !y))
    return fail(ER_EINVAL, "%s: null pointer", name);
  if (ldx < in) return fail(ER_EINVAL, "%s: row stride %lld < in %d", name, ldx, in);
  return ER_OK;
}

// ---------------------------------------------------------------------------
// attention (runtime/backends.py:90-95): scores = q.k * d^-0.5 (fp32), masked
// to -inf where not allowed, softmax (max-subtracted exp / sum), then p @ v.
// One CTA per (query, head).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) attention_kernel(const float* __restrict__ q, const float* __restrict__ keys,
                                                        const float* __restrict__ values,
                                                        const uint8_t* __restrict__ allowed,
                                                        float* __restrict__ out, int n, int kv, int heads, int d,
                                                        float scale) {
  extern __shared__ float sc[];  // [kv]
  __shared__ float red[32];
  const int i = blockIdx.x / heads, hh = blockIdx.x % heads;
  const float* qv = q + ((size_t)i * heads + hh) * d;
  for (int j = threadIdx.x; j < kv; j += blockDim.x) {
    const float* kp = keys + ((size_t)j * heads + hh) * d;
    float s = 0.f;
    for (int c = 0; c < d; ++c) s = fmaf(qv[c], kp[c], s);
    s *= scale;
    sc[j] = allowed[(size_t)i * kv + j] ? s : -INFINITY;
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int j = threadIdx.x; j < kv; j += blockDim.x) mx = fmaxf(mx, sc[j]);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = red[0];
  for (int w2 = 1; w2 < (int)(blockDim.x >> 5); ++w2) mx = fmaxf(mx, red[w2]);
  __syncthreads();
  float sum = 0.f;
  for (int j = threadIdx.x; j < kv; j += blockDim.x) {
    const float e = expf(sc[j] - mx);
    sc[j] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
  __syncthreads();
  sum = 0.f;
  for (int w2 = 0; w2 < (int)(blockDim.x >> 5); ++w2) sum += red[w2];
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    float acc = 0.f;
    for (int j = 0; j < kv; ++j) acc = fmaf(sc[j] / sum, values[((size_t)j * heads + hh) * d + c], acc);
    out[((size_t)i * heads + hh) * d + c] = acc;
  }
}

// The same with vector loads (d a multiple of 4, rows 16-byte aligned): a
// warp per key for the scores (one coalesced pass over the key row, lanes
// splitting d), then for p @ v each thread owns output columns and walks
// half of the keys, four loads in flight, halves added through shared memory.
// One CTA per (query, head), 256 threads.
__global__ void __launch_bounds__(256) attention_vec_kernel(const float* __restrict__ q,
                                                            const float* __restrict__ keys,
                                                            const float* __restrict__ values,
                                                            const uint8_t* __restrict__ allowed,
                                                            float* __restrict__ out, int n, int kv, int heads, int d,
                                                            float scale) {
  extern __shared__ float sm[];  // [kv] scores, then [2][d] partial outputs (the two halves of the keys)
  float* sc = sm;
  float* part = sm + kv;  // [2][d] (two halves of the keys)
  __shared__ float red[8];
  const int i = blockIdx.x / heads, hh = blockIdx.x % heads;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* qv = q + ((size_t)i * heads + hh) * d;
  for (int j = warp; j < kv; j += 8) {
    const float* kp = keys + ((size_t)j * heads + hh) * d;
    float s = 0.f;
    for (int c = lane * 4; c < d; c += 128) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(qv + c));
      const float4 b = __ldg(reinterpret_cast<const float4*>(kp + c));
      s = fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, fmaf(a.w, b.w, s))));
    }
    s = warp_sum(s) * scale;
    if (lane == 0) sc[j] = allowed[(size_t)i * kv + j] ? s : -INFINITY;
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int j = threadIdx.x; j < kv; j += blockDim.x) mx = fmaxf(mx, sc[j]);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = red[0];
  for (int w2 = 1; w2 < 8; ++w2) mx = fmaxf(mx, red[w2]);
  __syncthreads();
  float sum = 0.f;
  for (int j = threadIdx.x; j < kv; j += blockDim.x) {
    const float e = expf(sc[j] - mx);
    sc[j] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  if (lane == 0) red[warp] = sum;
  __syncthreads();
  sum = 0.f;
  for (int w2 = 0; w2 < 8; ++w2) sum += red[w2];
  const float inv = 1.0f / sum;
  // p @ v: thread t takes column c = t mod 128 (+128 per pass) and half t / 128 of the keys
  const int half = threadIdx.x >> 7, col = threadIdx.x & 127;
  const int j_mid = (kv + 1) / 2, j0 = half ? j_mid : 0, j1 = half ? kv : j_mid;
  for (int c = col; c < d; c += 128) {
    const float* vp = values + (size_t)hh * d + c;
    const size_t stride = (size_t)heads * d;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    int j = j0;
    for (; j + 3 < j1; j += 4) {
      a0 = fmaf(sc[j] * inv, vp[(size_t)j * stride], a0);
      a1 = fmaf(sc[j + 1] * inv, vp[(size_t)(j + 1) * stride], a1);
      a2 = fmaf(sc[j + 2] * inv, vp[(size_t)(j + 2) * stride], a2);
      a3 = fmaf(sc[j + 3] * inv, vp[(size_t)(j + 3) * stride], a3);
    }
    for (; j < j1; ++j) a0 = fmaf(sc[j] * inv, vp[(size_t)j * stride], a0);
    part[half * d + c] = (a0 + a1) + (a2 + a3);
  }
  __syncthreads();
  for (int c = threadIdx.x; c < d; c += blockDim.x)
    out[((size_t)i * heads + hh) * d + c] = part[c] + part[d + c];
}

// ---------------------------------------------------------------------------
// weight reconstruction: bit-exact fp32 (store/quantize.py:45-46,
// store/int4.py:142-144, bench/gptq_conversion_check.py:42-55)
// ---------------------------------------------------------------------------
__global__ void dequant_int8_kernel(const int8_t* __restrict__ q, const float* __restrict__ s, float* __restrict__ w,
                                    int rows, int cols) {
  const size_t total = (size_t)rows * cols;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x)
    w[i] = (float)q[i] * s[i / cols];
}

__global__ void dequant_int4_kernel(const uint8_t* __restrict__ p, const uint16_t* __restrict__ s,
                                    const uint8_t* __restrict__ z, int group, float* __restrict__ w, int rows,
                                    int cols) {
  const size_t total = (size_t)rows * cols;
  const int ng = cols / group;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / cols, c = i % cols;
    const uint8_t byte = p[r * (cols / 2) + c / 2];
    const int code = (c & 1) ? (byte >> 4) : (byte & 0xf);
    const size_t gi = r * ng + c / group;
    const float zero = z ? (float)z[gi] : 8.f;
    w[i] = ((float)code - zero) * half_bits_to_f32(s[gi]);
  }
}

}  // namespace er

using namespace er;

extern "C" {

int er_version(void) { return 100; }

const char* er_last_error(void) { return g_err; }

int er_device_sm_count(int* sms) {
  if (!sms) return fail(ER_EINVAL, "er_device_sm_count: null pointer");
  int dev = 0;
  if (int rc = cuda_check(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  return cuda_check(cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev), "cudaDeviceGetAttribute");
}

size_t er_record_bytes(int fmt, int hidden, int inter, int group) {
  if (fmt != ER_FMT_INT8 && (group <= 0 || hidden % group || inter % group)) return 0;
  RecordGeom g{fmt, hidden, inter, fmt == ER_FMT_INT8 ? 1 : group};
  return g.record_bytes();
}

size_t er_record_offset(int fmt, int hidden, int inter, int group, int which, int part) {
  if (which < 0 || which > 2 || part < 0 || part > 2) return (size_t)-1;
  if (fmt != ER_FMT_INT8 && (group <= 0 || hidden % group || inter % group)) return (size_t)-1;
  RecordGeom g{fmt, hidden, inter, fmt == ER_FMT_INT8 ? 1 : group};
  if (part == 0) return g.weight_offset(which);
  if (part == 1) return g.scale_offset(which);
  if (fmt != ER_FMT_INT4_ZP) return (size_t)-1;
  return g.zero_offset(which);
}

int er_linear_f32(const float* x, long long ldx, const float* w, const float* bias, float* y, int m, int out, int in,
                  void* stream) {
  if (int rc = check_linear_args("er_linear_f32", x, ldx, w, y, m, out, in)) return rc;
  // a few rows, or few output rows (a router) over many: vector kernels
  // with a dot product per warp; the tiled kernel for the rest
  const bool vec_ok = in % 4 == 0 && ldx % 4 == 0 && !(((uintptr_t)x | (uintptr_t)w) & 15) && in <= 16384;
  if (m > 0 && out > 0 && vec_ok && (m <= 8 || out <= 256))
    return launch_f32_small(x, ldx, w, bias, y, m, out, in, (cudaStream_t)stream);
  return launch_linear<0>(x, ldx, w, nullptr, nullptr, nullptr, 1, bias, y, m, out, in, (cudaStream_t)stream);
}

int er_int8_linear(const float* x, long long ldx, const int8_t* q, const float* scales, const float* bias, float* y,
                   int m, int out, int in, void* stream) {
  if (int rc = check_linear_args("er_int8_linear", x, ldx, q, y, m, out, in)) return rc;
  if (out > 0 && !scales) return fail(ER_EINVAL, "er_int8_linear: null scales");
  // a few rows, aligned rows of 16-byte multiples: stream the weights once
  if (m > 0 && m <= 8 && out > 0 && in % 16 == 0 && ldx % 4 == 0 && !(((uintptr_t)x | (uintptr_t)q) & 15))
    return launch_int8_gemv(x, ldx, q, scales, bias, y, m, out, in, (cudaStream_t)stream);
  return launch_linear<1>(x, ldx, q, scales, nullptr, nullptr, 1, bias, y, m, out, in, (cudaStream_t)stream);
}

int er_int4_linear(const float* x, long long ldx, const uint8_t* packed, const uint16_t* scales_f16,
                   const uint8_t* zeros, int group, const float* bias, float* y, int m, int out, int in,
                   void* stream) {
  if (int rc = check_linear_args("er_int4_linear", x, ldx, packed, y, m, out, in)) return rc;
  if (group <= 0 || group % 2 || in % group)
    return fail(ER_EINVAL, "er_int4_linear: %d input columns don't split into even groups of %d", in, group);
  if (out > 0 && in > 0 && !scales_f16) return fail(ER_EINVAL, "er_int4_linear: null scales");
  return launch_linear<2>(x, ldx, packed, nullptr, scales_f16, zeros, group, bias, y, m, out, in,
                          (cudaStream_t)stream);
}

int er_attention(const float* q, const float* keys, const float* values, const uint8_t* allowed, float* out, int n,
                 int kv, int heads, int d, void* stream) {
  if (n < 0 || kv < 0 || heads <= 0 || d <= 0) return fail(ER_EINVAL, "er_attention: bad sizes");
  if (n == 0) return ER_OK;
  if (!q || !keys || !values || !allowed || !out) return fail(ER_EINVAL, "er_attention: null pointer");
  const bool vec = d % 4 == 0 && !(((uintptr_t)q | (uintptr_t)keys | (uintptr_t)values) & 15);
  if (vec) {
    const size_t smem_v = ((size_t)kv + 2 * (size_t)d) * sizeof(float);
    if (smem_v > 200 * 1024) return fail(ER_EINVAL, "er_attention: kv %d too long for one CTA", kv);
    if (smem_v > 48 * 1024) {
      if (int rc = cuda_check(cudaFuncSetAttribute(attention_vec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   200 * 1024),
                              "attention smem attribute"))
        return rc;
    }
    attention_vec_kernel<<<n * heads, 256, smem_v, (cudaStream_t)stream>>>(q, keys, values, allowed, out, n, kv, heads,
                                                                           d, 1.0f / sqrtf((float)d));
    return launch_check("attention_vec_kernel");
  }
  const size_t smem = (size_t)kv * sizeof(float);
  if (smem > 200 * 1024) return fail(ER_EINVAL, "er_attention: kv %d too long for one CTA", kv);
  if (smem > 48 * 1024) {
    if (int rc = cuda_check(
            cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024),
            "attention smem attribute"))
      return rc;
  }
  attention_kernel<<<n * heads, 128, smem, (cudaStream_t)stream>>>(q, keys, values, allowed, out, n, kv, heads, d,
                                                                   1.0f / sqrtf((float)d));
  return launch_check("attention_kernel");
}

int er_dequant_int8(const int8_t* q, const float* scales, float* w, int rows, int cols, void* stream) {
  if (rows < 0 || cols < 0) return fail(ER_EINVAL, "er_dequant_int8: negative size");
  if ((size_t)rows * cols == 0) return ER_OK;
  if (!q || !scales || !w) return fail(ER_EINVAL, "er_dequant_int8: null pointer");
  dequant_int8_kernel<<<1184, 256, 0, (cudaStream_t)stream>>>(q, scales, w, rows, cols);
  return launch_check("dequant_int8_kernel");
}

int er_dequant_int4(const uint8_t* packed, const uint16_t* scales_f16, const uint8_t* zeros, int group, float* w,
                    int rows, int cols, void* stream) {
  if (rows < 0 || cols < 0) return fail(ER_EINVAL, "er_dequant_int4: negative size");
  if (group <= 0 || group % 2 || cols % group)
    return fail(ER_EINVAL, "er_dequant_int4: %d columns don't split into even groups of %d", cols, group);
  if ((size_t)rows * cols == 0) return ER_OK;
  if (!packed || !scales_f16 || !w) return fail(ER_EINVAL, "er_dequant_int4: null pointer");
  dequant_int4_kernel<<<1184, 256, 0, (cudaStream_t)stream>>>(packed, scales_f16, zeros, group, w, rows, cols);
  return launch_check("dequant_int4_kernel");
}

}  // extern "C"
