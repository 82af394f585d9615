// er_trace.cu -- expert-usage trace records packed on the device.
//
// Reference: runtime/expert_trace.py. A trace file holds one packed
// little-endian record per (token, layer) (record_dtype, :34-65):
//   position u32 | token u32 | layer u8 | phase u8 | experts u8[k] |
//   weights f32[k] | logits f16[E] | fate_experts u8[k] | fate_logits f16[E] |
//   prev_token_experts u8[k]
// (10 + 7k + 4E bytes, no padding), a forward call's records ordered token
// major, layer minor. ExpertTraceWriter.layer (:114-135) fills one layer's
// records from the router's logits, choices and weights, the Fate logits
// passed at the previous layer (their top-k, largest first; NO_EXPERT and
// zeros at a call's first layer) and each token's previous-token experts at
// this layer (the previous call's last token for the first token).
//
// Here the values never leave the device until the call ends: one warp per
// token builds its record in shared memory and stores it into the call's
// record buffer, which the host copies out once per call. Expert ids are
// stored modulo 256 and logits rounded to float16 to nearest even, as
// numpy's casts do.
#include "er_internal.cuh"

namespace er {

constexpr int kTraceNoExpert = 255;
constexpr int kTraceMaxRecord = 10 + 7 * kMaxTopK + 4 * 254;  // E <= 254: u8 ids below NO_EXPERT

__host__ __device__ inline int trace_record_bytes(int E, int k) { return 10 + 7 * k + 4 * E; }

__device__ __forceinline__ void put_u32(uint8_t* p, uint32_t v) {
  p[0] = v & 0xff;
  p[1] = (v >> 8) & 0xff;
  p[2] = (v >> 16) & 0xff;
  p[3] = v >> 24;
}
// float16 bits of v (rounded to nearest even), stored low byte first. The
// bytes are picked with a byte permute: a plain cast of the low byte of the
// half's bits was compiled into an integer conversion of v itself.
__device__ __forceinline__ void put_f16(uint8_t* p, float v) {
  const uint32_t h = __half_as_ushort(__float2half_rn(v));
  p[0] = (uint8_t)__byte_perm(h, 0u, 0x4440);
  p[1] = (uint8_t)__byte_perm(h, 0u, 0x4441);
}

template <int kPer>
__global__ void __launch_bounds__(256) trace_pack_kernel(uint8_t* __restrict__ records, int n, int L, int layer,
                                                         const uint32_t* __restrict__ positions,
                                                         const uint32_t* __restrict__ tokens, int phase,
                                                         const float* __restrict__ logits,
                                                         const int64_t* __restrict__ ids64,
                                                         const int32_t* __restrict__ ids32,
                                                         const float* __restrict__ weights,
                                                         const float* __restrict__ fate,
                                                         const uint8_t* __restrict__ prev_in,
                                                         uint8_t* __restrict__ prev_out, int E, int k) {
  __shared__ uint8_t rec_s[8][(kTraceMaxRecord + 15) & ~15];
  chain_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= n) return;
  uint8_t* r = rec_s[warp];
  const int rb = trace_record_bytes(E, k);
  const int o_exp = 10, o_w = 10 + k, o_lg = 10 + 5 * k, o_fe = 10 + 5 * k + 2 * E, o_fl = 10 + 6 * k + 2 * E,
            o_prev = 10 + 6 * k + 4 * E;
  auto id_of = [&](int token, int j) -> int {
    return ids64 ? (int)(ids64[(size_t)token * k + j] & 0xff) : (ids32[(size_t)token * k + j] & 0xff);
  };
  if (lane == 0) {
    put_u32(r, positions[t]);
    put_u32(r + 4, tokens[t]);
    r[8] = (uint8_t)layer;
    r[9] = (uint8_t)phase;
  }
  if (lane < k) {
    r[o_exp + lane] = (uint8_t)id_of(t, lane);
    put_u32(r + o_w + 4 * lane, __float_as_uint(weights[(size_t)t * k + lane]));
    r[o_prev + lane] = t > 0 ? (uint8_t)id_of(t - 1, lane) : prev_in[(size_t)layer * k + lane];
    if (t == n - 1) prev_out[(size_t)layer * k + lane] = (uint8_t)id_of(t, lane);
  }
  for (int e = lane; e < E; e += 32) {
    put_f16(r + o_lg + 2 * e, logits[(size_t)t * E + e]);
    put_f16(r + o_fl + 2 * e, fate ? fate[(size_t)t * E + e] : 0.f);
  }
  // the Fate top-k: largest first, exact ties to the lower id, NaN as -inf
  float v[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = lane + 32 * j;
    const float x = (fate && e < E) ? fate[(size_t)t * E + e] : -INFINITY;
    v[j] = x != x ? -INFINITY : x;
  }
  uint32_t taken = 0;
  for (int s = 0; s < k; ++s) {
    int best = kTraceNoExpert;
    if (fate) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int e = lane + 32 * j;
        if (e < E && !(taken & (1u << j)) && (v[j] > bv || (v[j] == bv && e < bi))) {
          bv = v[j];
          bi = e;
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
      if (lane == (bi & 31)) taken |= 1u << (bi >> 5);
      best = bi;
    }
    if (lane == 0) r[o_fe + s] = (uint8_t)best;
  }
  __syncwarp();
  uint8_t* dst = records + ((size_t)t * L + layer) * rb;
  for (int b = lane; b < rb; b += 32) dst[b] = r[b];
}

}  // namespace er

using namespace er;

extern "C" size_t er_trace_record_bytes(int num_experts, int top_k) {
  if (num_experts < 1 || num_experts >= kTraceNoExpert || top_k < 1 || top_k > kMaxTopK) return 0;
  return (size_t)trace_record_bytes(num_experts, top_k);
}

extern "C" int er_trace_pack_layer(void* records, int n, int num_layers, int layer, const uint32_t* positions,
                                   const uint32_t* tokens, int phase, const float* logits, const void* experts,
                                   int experts_are_i64, const float* weights, const float* fate_logits,
                                   const uint8_t* prev_in, uint8_t* prev_out, int num_experts, int top_k,
                                   void* stream) {
  if (er_trace_record_bytes(num_experts, top_k) == 0)
    return fail(ER_EINVAL, "er_trace_pack_layer: %d experts (u8 ids: at most %d), top_k %d (1..%d)", num_experts,
                kTraceNoExpert - 1, top_k, kMaxTopK);
  if (n < 0 || num_layers < 1 || num_layers > 255 || layer < 0 || layer >= num_layers || phase < 0 || phase > 255)
    return fail(ER_EINVAL, "er_trace_pack_layer: n %d, layer %d of %d, phase %d", n, layer, num_layers, phase);
  if (n == 0) return ER_OK;
  if (!records || !positions || !tokens || !logits || !experts || !weights || !prev_in || !prev_out)
    return fail(ER_EINVAL, "er_trace_pack_layer: null argument");
  if (prev_in == prev_out && n > 1)
    return fail(ER_EINVAL, "er_trace_pack_layer: prev_in and prev_out must differ (the first token reads the old "
                           "state while the last writes the new)");
  const int64_t* i64 = experts_are_i64 ? static_cast<const int64_t*>(experts) : nullptr;
  const int32_t* i32 = experts_are_i64 ? nullptr : static_cast<const int32_t*>(experts);
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 grid((n + 7) / 8), block(256);
  uint8_t* rec = static_cast<uint8_t*>(records);
  if (num_experts <= 64)
    return launch_chained(trace_pack_kernel<2>, grid, block, 0, st, "trace_pack_kernel", rec, n, num_layers, layer,
                          positions, tokens, phase, logits, i64, i32, weights, fate_logits, prev_in, prev_out,
                          num_experts, top_k);
  return launch_chained(trace_pack_kernel<8>, grid, block, 0, st, "trace_pack_kernel", rec, n, num_layers, layer,
                        positions, tokens, phase, logits, i64, i32, weights, fate_logits, prev_in, prev_out,
                        num_experts, top_k);
}
