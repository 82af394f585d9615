// er_model.cu -- the non-MoE parts of the Qwen1.5-MoE decoder layer.
//
// Reference: runtime/qwen_moe.py. rms_norm (:121-123): w * x / sqrt(mean(x^2)
// + eps) in fp32; RoPE (:126-138, 255-262): cos/sin of position * inv_freq,
// inv_freq = 1 / theta^(2i/d) in fp32, rotate_half convention, applied to q
// and k, then k and v appended to the layer's KV cache (:264-270); the
// embedding lookup Int8Matrix.dequantized_rows (runtime/weights.py:62-64):
// q[id] * scale[id]. The residual add before each norm is fused into the norm
// (x <- x + delta, h <- rms_norm(x)), so the hidden state makes one pass per
// sub-layer.
#include "er_internal.cuh"

namespace er {

// One CTA per row: x_out = x (+ add), h = w * x_out / sqrt(mean(x_out^2) + eps).
__global__ void __launch_bounds__(256) rms_norm_kernel(const float* x, const float* __restrict__ add,
                                                       const float* __restrict__ w, float eps, int H, float* x_out,
                                                       float* __restrict__ h) {
  __shared__ float red[8];
  chain_wait();
  const size_t row = blockIdx.x;
  const float* xr = x + row * H;
  const float* ar = add ? add + row * H : nullptr;
  float ss = 0.f;
  for (int c = threadIdx.x * 4; c < H; c += blockDim.x * 4) {
    float4 v = *reinterpret_cast<const float4*>(xr + c);
    if (ar) {
      const float4 a = *reinterpret_cast<const float4*>(ar + c);
      v.x += a.x;
      v.y += a.y;
      v.z += a.z;
      v.w += a.w;
      *reinterpret_cast<float4*>(x_out + row * H + c) = v;
    }
    ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
  const float inv = 1.0f / sqrtf(tot / (float)H + eps);
  // with the add, the sum was stored to x_out (which may be x itself) by this
  // same thread above: read it back from there
  const float* src = ar ? x_out + row * H : xr;
  for (int c = threadIdx.x * 4; c < H; c += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(src + c);
    const float4 g = *reinterpret_cast<const float4*>(w + c);
    float4 o;
    o.x = g.x * (v.x * inv);
    o.y = g.y * (v.y * inv);
    o.z = g.z * (v.z * inv);
    o.w = g.w * (v.w * inv);
    *reinterpret_cast<float4*>(h + row * H + c) = o;
  }
}

// One CTA per token: the token's row of the fused q|k|v projection (row
// stride ld); rotate its q heads into q_out and its k heads (position
// pos0 + t) into the cache rows pos0 + t, and copy v there. The d/2
// angles' cos and sin are computed once per token into shared memory; then
// thread j < d/2 of a head handles the pair (j, j + d/2): out_j = x_j cos_j -
// x_{j+d/2} sin_j, out_{j+d/2} = x_{j+d/2} cos_j + x_j sin_j (cos/sin of
// both halves equal).
__global__ void __launch_bounds__(256) rope_kv_kernel(const float* __restrict__ qkv, long long ld,
                                                      float* __restrict__ q_out, int heads, int kv_heads, int d,
                                                      int pos0, float theta, float* __restrict__ k_cache,
                                                      float* __restrict__ v_cache) {
  extern __shared__ float cs[];  // [d/2] cos, then [d/2] sin
  chain_wait();
  const int t = blockIdx.x;
  const int half = d / 2;
  const float pos = (float)(pos0 + t);
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    // inv_freq_j = 1 / theta^(2j / d), in fp32 like the reference's table
    const float inv_freq = 1.0f / powf(theta, (float)(2 * j) / (float)d);
    const float ang = pos * inv_freq;
    cs[j] = cosf(ang);
    cs[half + j] = sinf(ang);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < (heads + kv_heads) * half; i += blockDim.x) {
    const int head = i / half, j = i % half;
    const float c = cs[j], s = cs[half + j];
    const float* row = qkv + (size_t)t * ld;
    if (head < heads) {
      const float* qh = row + (size_t)head * d;
      float* qo = q_out + ((size_t)t * heads + head) * d;
      const float a = qh[j], b = qh[j + half];
      qo[j] = a * c - b * s;
      qo[j + half] = b * c + a * s;
    } else {
      const int kh = head - heads;
      const float* kr = row + (size_t)(heads + kh) * d;
      float* kc = k_cache + ((size_t)(pos0 + t) * kv_heads + kh) * d;
      const float a = kr[j], b = kr[j + half];
      kc[j] = a * c - b * s;
      kc[j + half] = b * c + a * s;
      const float* vr = row + (size_t)(heads + kv_heads + kh) * d;
      float* vc = v_cache + ((size_t)(pos0 + t) * kv_heads + kh) * d;
      vc[j] = vr[j];
      vc[j + half] = vr[j + half];
    }
  }
}

// out[t] = q[ids[t]] * scale[ids[t]]; one CTA per token, 16 bytes of codes per thread and step
__global__ void __launch_bounds__(256) embed_int8_kernel(const int8_t* __restrict__ q, const float* __restrict__ s,
                                                         const int64_t* __restrict__ ids, long long vocab, int H,
                                                         float* __restrict__ out, int* __restrict__ bad) {
  chain_wait();
  const int t = blockIdx.x;
  const long long id = ids[t];
  float* o = out + (size_t)t * H;
  if (id < 0 || id >= vocab) {  // reported; the row reads as NaN
    if (threadIdx.x == 0) atomicOr(bad, 1);
    for (int c = threadIdx.x; c < H; c += blockDim.x) o[c] = __int_as_float(0x7fc00000);
    return;
  }
  const int8_t* row = q + (size_t)id * H;
  const float sc = s[id];
  for (int c = threadIdx.x * 16; c < H; c += blockDim.x * 16) {
    const int4 raw = *reinterpret_cast<const int4*>(row + c);
    const int8_t* b = reinterpret_cast<const int8_t*>(&raw);
#pragma unroll
    for (int j = 0; j < 16; ++j) o[c + j] = (float)b[j] * sc;
  }
}

}  // namespace er

using namespace er;

extern "C" int er_rms_norm(const float* x, const float* add, const float* weight, float eps, int n, int hidden,
                           float* x_out, float* h, void* stream) {
  if (n < 0 || hidden <= 0 || hidden % 4) return fail(ER_EINVAL, "er_rms_norm: n %d, hidden %d (multiple of 4)", n, hidden);
  if (n == 0) return ER_OK;
  if (!x || !weight || !h || (add && !x_out)) return fail(ER_EINVAL, "er_rms_norm: null argument");
  if (((uintptr_t)x | (uintptr_t)add | (uintptr_t)weight | (uintptr_t)x_out | (uintptr_t)h) & 15)
    return fail(ER_EINVAL, "er_rms_norm: rows must be 16-byte aligned");
  return launch_chained(rms_norm_kernel, dim3(n), dim3(256), 0, (cudaStream_t)stream, "rms_norm_kernel", x, add,
                        weight, eps, hidden, x_out, h);
}

extern "C" int er_rope_kv(const float* qkv, long long ld, float* q_out, int n, int heads, int kv_heads, int head_dim,
                          int pos0, float theta, float* k_cache, float* v_cache, int max_seq, void* stream) {
  if (n < 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads || head_dim <= 0 || head_dim % 2 || pos0 < 0)
    return fail(ER_EINVAL, "er_rope_kv: n %d, heads %d / %d, head_dim %d, pos0 %d", n, heads, kv_heads, head_dim,
                pos0);
  if (pos0 + n > max_seq)
    return fail(ER_EINVAL, "sequence length %d exceeds the KV cache (%d)", pos0 + n, max_seq);
  if (n == 0) return ER_OK;
  if (!qkv || !q_out || !k_cache || !v_cache) return fail(ER_EINVAL, "er_rope_kv: null argument");
  if (ld < (long long)(heads + 2 * kv_heads) * head_dim)
    return fail(ER_EINVAL, "er_rope_kv: row stride %lld shorter than q|k|v (%d)", ld, (heads + 2 * kv_heads) * head_dim);
  if (head_dim > 8192) return fail(ER_EINVAL, "er_rope_kv: head_dim %d above 8192", head_dim);
  return launch_chained(rope_kv_kernel, dim3(n), dim3(256), (size_t)head_dim * sizeof(float), (cudaStream_t)stream,
                        "rope_kv_kernel", qkv, ld, q_out, heads, kv_heads, head_dim, pos0, theta, k_cache, v_cache);
}

extern "C" int er_embed_int8(const int8_t* q, const float* scales, long long vocab, int hidden, const int64_t* ids,
                             int n, float* out, int* bad, void* stream) {
  if (n < 0 || vocab <= 0 || hidden <= 0 || hidden % 16)
    return fail(ER_EINVAL, "er_embed_int8: n %d, vocab %lld, hidden %d (multiple of 16)", n, vocab, hidden);
  if (n == 0) return ER_OK;
  if (!q || !scales || !ids || !out || !bad) return fail(ER_EINVAL, "er_embed_int8: null argument");
  if ((uintptr_t)q & 15) return fail(ER_EINVAL, "er_embed_int8: codes must be 16-byte aligned");
  return launch_chained(embed_int8_kernel, dim3(n), dim3(128), 0, (cudaStream_t)stream, "embed_int8_kernel", q, scales,
                        ids, vocab, hidden, out, bad);
}
