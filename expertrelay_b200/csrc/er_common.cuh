// er_common.cuh -- shared helpers for libexpertrelay_b200 (sm_100a).
#pragma once

#include <utility>

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/expertrelay_b200.h"

namespace er {

// ---- error reporting (er_capi.cu) ---------------------------------------
int fail(int code, const char* fmt, ...);                 // records the message, returns code
int cuda_check(cudaError_t e, const char* what);          // ER_OK or ER_ECUDA with the CUDA message
inline int launch_check(const char* what) { return cuda_check(cudaGetLastError(), what); }

// The block's kernels run as one chain on a stream. Each is launched with
// programmatic stream serialization, so its launch (and any prologue that
// touches only its own shared memory, TMEM and registers) overlaps the tail
// of the kernel before it; chain_wait() returns once that kernel has
// completed and its writes are visible. Every chained kernel calls
// chain_wait() before it reads or writes global memory another kernel of
// the stream uses. In a kernel launched without the attribute it returns at
// once.
__device__ __forceinline__ void chain_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel of the chain launch (its CTAs start as resources
// allow and run their prologue up to chain_wait) before this one completes;
// it changes nothing about what the next kernel's chain_wait waits for.
// Called first thing by the short kernels ahead of a tensor-core GEMM, so
// the GEMM's barrier set-up and tensor-map prefetch overlap them.
__device__ __forceinline__ void chain_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline int launch_chained(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                          const char* what, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_check(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...), what);
}

constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 8;
constexpr size_t kRecordAlign = 4096;  // store/unbuffered_io.py ALIGNMENT

__host__ __device__ inline size_t align_up(size_t n, size_t a) { return (n + a - 1) / a * a; }

// ---- expert record layout (store/layout.py:53-115, store/int4.py:165-244) ----
// Matrices in on-disk order: gate [inter, hidden], up [inter, hidden],
// down [hidden, inter]. Weights of all three first, then their scales, then
// (ER_FMT_INT4_ZP only) their zero points, then zero padding to 4096 bytes.
struct RecordGeom {
  int fmt, hidden, inter, group;

  __host__ __device__ int rows(int which) const { return which == 2 ? hidden : inter; }
  __host__ __device__ int cols(int which) const { return which == 2 ? inter : hidden; }
  __host__ __device__ size_t weight_bytes(int which) const {
    size_t e = (size_t)rows(which) * cols(which);
    return fmt == ER_FMT_INT8 ? e : e / 2;
  }
  __host__ __device__ size_t scale_bytes(int which) const {
    return fmt == ER_FMT_INT8 ? (size_t)rows(which) * 4 : (size_t)rows(which) * (cols(which) / group) * 2;
  }
  __host__ __device__ size_t zero_bytes(int which) const {
    return fmt == ER_FMT_INT4_ZP ? (size_t)rows(which) * (cols(which) / group) : 0;
  }
  __host__ __device__ size_t weight_offset(int which) const {
    size_t off = 0;
    for (int i = 0; i < which; ++i) off += weight_bytes(i);
    return off;
  }
  __host__ __device__ size_t scale_offset(int which) const {
    size_t off = weight_offset(3);
    for (int i = 0; i < which; ++i) off += scale_bytes(i);
    return off;
  }
  __host__ __device__ size_t zero_offset(int which) const {
    size_t off = scale_offset(3);
    for (int i = 0; i < which; ++i) off += zero_bytes(i);
    return off;
  }
  __host__ __device__ size_t payload_bytes() const { return zero_offset(3); }
  __host__ __device__ size_t record_bytes() const { return align_up(payload_bytes(), kRecordAlign); }
};

// ---- small device helpers -----------------------------------------------
__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

// SiLU and sigmoid exactly as the reference writes them
// (runtime/qwen_moe.py:149-154): x / (1 + e^-x), 1 / (1 + e^-x).
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float half_bits_to_f32(uint16_t b) {
  return __half2float(__ushort_as_half(b));
}

// Signed int8 lanes of a 32-bit word -> float.
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float* f) {
  f[0] = (float)(int8_t)(w & 0xff);
  f[1] = (float)(int8_t)((w >> 8) & 0xff);
  f[2] = (float)(int8_t)((w >> 16) & 0xff);
  f[3] = (float)(int8_t)(w >> 24);
}

// 8 nibbles of a 32-bit word (lowest first = lower input column) -> float codes 0..15.
__device__ __forceinline__ void u4x8_to_f32(uint32_t w, float* f) {
#pragma unroll
  for (int j = 0; j < 8; ++j) f[j] = (float)((w >> (4 * j)) & 0xf);
}

// Four consecutive activations as fp32 (16-byte fp32 or 8-byte bf16 load).
__device__ __forceinline__ float4 load4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 load4(const __nv_bfloat16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                     __uint_as_float(u.y & 0xffff0000u));
}

// Read-only, L1-bypassing 16-byte global load for weights read once.
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint2 ld_stream_u2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p));
  return r;
}

}  // namespace er
