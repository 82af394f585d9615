// er_router_tc.cu -- router logits of large fp32 batches on the tensor cores.
//
// Reference: runtime/qwen_moe.py:303 (router = h @ W_r^T in fp32) and :358
// (the shared-expert gate logit h @ w_g^T). The top-k that follows ranks
// these logits, so they must keep fp32 accuracy; tcgen05 has no fp32 MMA,
// but its tf32 MMA (10-bit mantissa, fp32 accumulation) does, three times:
// each operand is split exactly into x = hi + lo with hi = x with its low
// 13 mantissa bits cleared (a tf32 value) and lo = x - hi (|lo| < 2^-10 |hi|),
// and the logit is accumulated as hi_h*hi_w + hi_h*lo_w + lo_h*hi_w. The
// dropped lo_h*lo_w term and lo's own tf32 rounding are below 2^-20 of each
// product, the order of fp32 rounding itself.
//
// One CTA per 128-token tile and K slice (the same K slices, and the same
// partial-logit layout, as the SIMT router_gemm_kernel, so the top-k kernel
// adds them unchanged):
//  * warp 8 (lane 0) TMA-loads per 32-input k-block the token tile (128 rows
//    x 128 bytes), the router rows (64-row box: rows past E read as zeros)
//    and the gate row (16-row box: rows past 1 read as zeros), 128-byte
//    swizzled, into a stage of a 4-deep ring;
//  * warps 0-7 split every staged row into hi (in place) and lo (beside it):
//    the split is elementwise, so the swizzled layout is kept as it is; the
//    gate row is split into row E of the router tile (E < 64), so one MMA
//    covers both;
//  * warp 9 issues per 8-input step A_hi x [W_hi; W_lo] (M = 128 tokens,
//    N = 128) and A_lo x W_hi (N = 64) into a fresh TMEM accumulator per
//    k-block, and frees the stage;
//  * warps 0-7 add each k-block's accumulators into fp32 registers (lane =
//    token; two warps per TMEM lane quadrant, 32 router columns each) and
//    finally write the partial logits.
// Every mbarrier wait is bounded: a CTA that gives up raises bit 8 of the
// plan's error word (the combine then writes NaN rows), drains its copies
// and frees its TMEM.
#include "er_tc.cuh"

namespace er {

namespace {

constexpr int kRtTokens = 128;    // tokens per CTA (MMA M)
constexpr int kRtRows = 64;       // router rows of the B tile: E router rows, then the gate row (E < 64)
constexpr int kRtGateRows = 16;   // the gate's staging box (row 0 is the gate, rows 1.. read as zeros)
constexpr int kRtKBlock = 32;     // fp32 inputs per stage (128 bytes per row)
constexpr int kRtStages = 4;
constexpr int kRtSplitWarps = 8;  // warps 0-7 split / add / epilogue, 8 TMA, 9 MMA
constexpr int kRtSplitThreads = kRtSplitWarps * 32;
constexpr int kRtThreads = kRtSplitThreads + 64;
constexpr int kRtTmaWarp = kRtSplitWarps;
constexpr int kRtMmaWarp = kRtSplitWarps + 1;
// Per MMA step two MMAs: A_hi x [W_hi; W_lo] (N = 128: the hi and the lo
// products side by side) and A_lo x W_hi (N = 64; not for bf16 tokens). Small
// MMAs cost about the same as these regardless of N, so fewer and wider ones
// (the gate row rides in the router tile) keep the tensor pipe fed. Two
// accumulator buffers of 256 columns ([0, 128) the wide MMA, [128, 192) the
// other): each k-block's MMAs start a fresh accumulator, which warps 0-7 add
// into fp32 registers while the next block accumulates. The tensor core's fp32
// accumulation rounds less accurately than an fp32 add, and a running
// accumulator over a whole K slice drifted to ~6e-6 of a unit logit; a sum of
// 16 blocks rounded in registers stays at fp32 level.
constexpr int kRtAccCols = 256;
constexpr int kRtTmemCols = 2 * kRtAccCols;

// Stage layout (each tile 1024-byte aligned, as the 128-byte swizzle needs):
constexpr int kRtAHi = 0;                           // tokens, hi (TMA writes x, the split clears lo bits)
constexpr int kRtALo = kRtAHi + kRtTokens * 128;    // tokens, lo
constexpr int kRtBHi = kRtALo + kRtTokens * 128;    // router rows, hi
constexpr int kRtBLo = kRtBHi + kRtRows * 128;      // router rows, lo
constexpr int kRtGHi = kRtBLo + kRtRows * 128;      // the gate row as TMA stages it (moved into row E)
constexpr int kRtStageBytes = kRtGHi + kRtGateRows * 128;
constexpr int kRtTxBytes = (kRtTokens + kRtRows + kRtGateRows) * 128;  // bytes TMA writes per stage
constexpr size_t kRtSmem = 1024 + (size_t)kRtStages * kRtStageBytes + 256;
static_assert(kRtStageBytes % 1024 == 0 && kRtGHi % 1024 == 0, "tile alignment");
static_assert(kRtSmem <= 232448, "shared memory per CTA");

struct RtMaps {
  CUtensorMap h;     // [n, H] fp32, box 32 x 128
  CUtensorMap w;     // [E, H] fp32, box 32 x 64
  CUtensorMap gate;  // [1, H] fp32, box 32 x 16 (unused when has_gate is 0)
};

struct RtArgs {
  int n, H, E, has_gate;
  float* logits;      // [gridDim.y][n][E] partial logits
  float* gate_logit;  // [gridDim.y][n]
  int* tally;         // cleared (ntally ints) by CTA (0, 0) for the top-k kernel
  int ntally;
  int* error;         // bit 8 on a wait that gave up (may be null)
  unsigned long long wait_ns;
};

// tcgen05 instruction descriptor, kind::tf32: D f32, A and B tf32, both K-major.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// hi = x with the low 13 mantissa bits cleared (exactly a tf32 value), lo = x - hi (exact)
__device__ __forceinline__ void split_tf32(uint32_t x, uint32_t& hi, uint32_t& lo) {
  hi = x & 0xffffe000u;
  lo = __float_as_uint(__uint_as_float(x) - __uint_as_float(hi));
}

// Splits `rows` staged rows of 128 bytes (hi tile at `hi_addr`, lo tile at
// `lo_addr`, shared-memory addresses) by the calling thread's share: thread
// `tid` of `nthreads` takes 16-byte chunks tid, tid + nthreads, ...; row
// `skip` (if any) is left to the caller.
__device__ __forceinline__ void split_tile(uint32_t hi_addr, uint32_t lo_addr, int rows, int tid, int nthreads,
                                           int skip = -1) {
#pragma unroll 4
  for (int c = tid; c < rows * 8; c += nthreads) {
    if ((c >> 3) == skip) continue;
    const uint4 v = lds128(hi_addr + c * 16);
    uint4 h, l;
    split_tf32(v.x, h.x, l.x);
    split_tf32(v.y, h.y, l.y);
    split_tf32(v.z, h.z, l.z);
    split_tf32(v.w, h.w, l.w);
    sts128(hi_addr + c * 16, h.x, h.y, h.z, h.w);
    sts128(lo_addr + c * 16, l.x, l.y, l.z, l.w);
  }
}

}  // namespace

// bf16 tokens: bf16 values are exact tf32 values, so a token tile needs no
// lo part; TMA stages the 32 inputs of a k-block unswizzled (64 bytes per
// row, in the lo tile's space) and warps 0-7 widen them into the hi tile's
// swizzled fp32 layout. Two products per MMA step instead of three.
template <bool BF>
__global__ void __launch_bounds__(kRtThreads, 1) router_tc_kernel(const __grid_constant__ RtMaps maps, RtArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)kRtStages * kRtStageBytes);
  uint64_t* ready = full + kRtStages;
  uint64_t* empty = ready + kRtStages;
  uint64_t* acc_full = empty + kRtStages;   // [2]: a k-block's accumulators are complete
  uint64_t* acc_empty = acc_full + 2;       // [2]: warps 0-7 have read them
  uint64_t* drain_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kRtTokens;
  // this CTA's K slice, in whole 32-input blocks (blocks past H read as zeros)
  const int slice = ((a.H + gridDim.y - 1) / gridDim.y + kRtKBlock - 1) / kRtKBlock * kRtKBlock;
  const int kbeg = blockIdx.y * slice;
  const int klen = max(0, min(slice, a.H - kbeg));
  const int nkb = (klen + kRtKBlock - 1) / kRtKBlock;
  const uint32_t tx = kRtTxBytes - (a.has_gate ? 0 : kRtGateRows * 128) - (BF ? kRtTokens * 64 : 0);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kRtStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], kRtSplitWarps);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kRtSplitWarps);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kRtTmaWarp && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.h)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.w)) : "memory");
    if (a.has_gate) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.gate)) : "memory");
  }
  chain_wait();
  if (blockIdx.x == 0 && blockIdx.y == 0 && a.tally)  // cleared for the top-k kernel's per-expert counts
    for (int i = threadIdx.x; i < a.ntally; i += blockDim.x) a.tally[i] = 0;
  if (warp == kRtMmaWarp) tmem_alloc<1>(tmem_slot, kRtTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == kRtTmaWarp) {
    // ---------------- TMA producer ----------------
    int kb = 0;
    for (; kb < nkb; ++kb) {
      const int s = kb % kRtStages;
      const uint32_t ph = (kb / kRtStages) & 1;
      if (!warp_wait(&empty[s], ph ^ 1, abort_flag, lane, a.wait_ns)) break;
      if (lane == 0) {
        uint8_t* st = smem + (size_t)s * kRtStageBytes;
        const int x = kbeg + kb * kRtKBlock;
        mbar_expect_tx(&full[s], tx);
        tma_load_2d(st + (BF ? kRtALo : kRtAHi), &maps.h, &full[s], x, m0);
        tma_load_2d(st + kRtBHi, &maps.w, &full[s], x, 0);
        if (a.has_gate) tma_load_2d(st + kRtGHi, &maps.gate, &full[s], x, 0);
      }
      __syncwarp();
    }
    if (kb < nkb && lane == 0) {
      // aborted: every stage issued so far lands before the CTA exits
      for (int s = 0; s < kRtStages && s < kb; ++s) {
        const int last = kb - 1 - ((kb - 1 - s) % kRtStages);
        mbar_drain(&full[s], (last / kRtStages) & 1, 100000000ull);
      }
    }
    __syncwarp();
  } else if (warp == kRtMmaWarp) {
    // ---------------- MMA issuer ----------------
    const uint32_t id_w = idesc_tf32(kRtTokens, 2 * kRtRows), id_r = idesc_tf32(kRtTokens, kRtRows);
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % kRtStages, b = kb & 1;
      const uint32_t ph = (kb / kRtStages) & 1, bph = (kb >> 1) & 1;
      if (!warp_wait(&ready[s], ph, abort_flag, lane, a.wait_ns)) break;
      if (!warp_wait(&acc_empty[b], bph ^ 1, abort_flag, lane, a.wait_ns)) break;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t st = smem_u32(smem + (size_t)s * kRtStageBytes);
        const uint32_t d_w = tmem_base + b * kRtAccCols, d_l = d_w + 2 * kRtRows;
#pragma unroll 1
        for (int ks = 0; ks < kRtKBlock / 8; ++ks) {  // 8 fp32 inputs (32 bytes) per MMA
          const uint32_t o = ks * 32;
          const uint32_t acc = ks > 0 ? 1u : 0u;
          // B = [W_hi; W_lo]: the lo tile follows the hi tile, 128 rows in 16 swizzle atoms
          mma_tf32(d_w, umma_desc_sw128(st + kRtAHi + o), umma_desc_sw128(st + kRtBHi + o), id_w, acc);
          if (!BF) mma_tf32(d_l, umma_desc_sw128(st + kRtALo + o), umma_desc_sw128(st + kRtBHi + o), id_r, acc);
        }
        umma_commit<1>(&empty[s]);     // the stage is free once these MMAs have read it
        umma_commit<1>(&acc_full[b]);  // and the block's accumulators are complete
      }
      __syncwarp();
    }
    if (lane == 0) {
      // every MMA issued by this thread has finished before TMEM is released
      umma_commit<1>(drain_bar);
      mbar_drain(drain_bar, 0, 100000000ull);
    }
    __syncwarp();
  } else {
    // ---------------- split (warps 0-7), block sums, epilogue ----------------
    // Split k-block kb, then add k-block kb - 1's accumulators, so the MMAs
    // of block kb overlap the add of block kb - 1. Lane l of warp w holds
    // token m0 + 32 (w % 4) + l (TMEM lanes of quadrant w % 4) and router
    // columns 32 (w / 4) .. + 31.
    constexpr int kCols = kRtRows / 2;
    const int tid = threadIdx.x;  // 0..255
    const int quad = warp & 3, col0 = (warp >> 2) * kCols;
    // the gate logit is column E (held by the warp whose columns include it)
    const bool gate_warp = a.has_gate && a.E >= col0 && a.E < col0 + kCols;
    const uint32_t lanes = (uint32_t)(quad * 32) << 16;
    float acc[kCols];
#pragma unroll
    for (int j = 0; j < kCols; ++j) acc[j] = 0.f;
    auto add_block = [&](int kb) -> bool {
      const int b = kb & 1;
      if (!warp_wait(&acc_full[b], (kb >> 1) & 1, abort_flag, lane, a.wait_ns)) return false;
      tc_fence_after();
      const uint32_t tb = tmem_base + b * kRtAccCols + lanes;
      // this warp's 32 columns of the three products: hi x hi at c, hi x lo
      // at 64 + c, lo x hi at 128 + c (the block's partials, added in order)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t v0[16], v1[16], v2[16];
        tmem_ld16(tb + col0 + 16 * h, v0);
        tmem_ld16(tb + kRtRows + col0 + 16 * h, v1);
        if (!BF) tmem_ld16(tb + 2 * kRtRows + col0 + 16 * h, v2);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float p = __uint_as_float(v0[j]) + __uint_as_float(v1[j]);
          if (!BF) p += __uint_as_float(v2[j]);
          acc[16 * h + j] += p;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      return true;
    };
    bool ok = true;
    for (int kb = 0; ok && kb < nkb; ++kb) {
      const int s = kb % kRtStages;
      const uint32_t ph = (kb / kRtStages) & 1;
      if (!warp_wait(&full[s], ph, abort_flag, lane, a.wait_ns)) {
        ok = false;
        break;
      }
      const uint32_t st = smem_u32(smem + (size_t)s * kRtStageBytes);
      if (BF) {
        // widen: 16-byte fp32 chunk j of row r (inputs 4j .. 4j + 3) from 8
        // staged bytes, stored at chunk j ^ (r % 8) of the 128-byte-swizzled row
#pragma unroll 4
        for (int c = tid; c < kRtTokens * 8; c += kRtSplitThreads) {
          const int r = c >> 3, j = c & 7;
          uint32_t u0, u1;
          asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(u0), "=r"(u1) : "r"(st + kRtALo + r * 64 + j * 8));
          sts128(st + kRtAHi + r * 128 + ((j ^ (r & 7)) << 4), u0 << 16, u0 & 0xffff0000u, u1 << 16,
                 u1 & 0xffff0000u);
        }
      } else {
        split_tile(st + kRtAHi, st + kRtALo, kRtTokens, tid, kRtSplitThreads);
      }
      // router rows (rows past E are zeros) and, in row E, the gate row from
      // its staging tile: logical chunk j sits at chunk j ^ (row % 8)
      split_tile(st + kRtBHi, st + kRtBLo, kRtRows, tid, kRtSplitThreads, a.has_gate ? a.E : -1);
      if (a.has_gate && tid < 8) {
        const uint4 v = lds128(st + kRtGHi + tid * 16);  // gate row 0: chunk j at j
        uint4 h, l;
        split_tf32(v.x, h.x, l.x);
        split_tf32(v.y, h.y, l.y);
        split_tf32(v.z, h.z, l.z);
        split_tf32(v.w, h.w, l.w);
        const uint32_t off = a.E * 128 + ((tid ^ (a.E & 7)) << 4);
        sts128(st + kRtBHi + off, h.x, h.y, h.z, h.w);
        sts128(st + kRtBLo + off, l.x, l.y, l.z, l.w);
      }
      fence_async_smem();  // the split tiles are read by tcgen05.mma (async proxy)
      __syncwarp();
      if (lane == 0) mbar_arrive(&ready[s]);
      if (kb > 0) ok = add_block(kb - 1);
    }
    if (ok && nkb > 0) ok = add_block(nkb - 1);
    if (ok) {  // an empty K slice (a hidden size smaller than the slices) writes zeros
      const int t = m0 + quad * 32 + lane;
      if (t < a.n) {
        float* lrow = a.logits + ((size_t)blockIdx.y * a.n + t) * a.E;
#pragma unroll
        for (int j = 0; j < kCols; ++j)
          if (col0 + j < a.E) lrow[col0 + j] = acc[j];
        if (gate_warp) {
          float g = acc[0];  // register select of column E, no local-memory indexing
#pragma unroll
          for (int j = 1; j < kCols; ++j)
            if (col0 + j == a.E) g = acc[j];
          a.gate_logit[(size_t)blockIdx.y * a.n + t] = g;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (*abort_flag && threadIdx.x == 0 && a.error) atomicOr(a.error, 8);
  if (warp == kRtMmaWarp) tmem_dealloc<1>(tmem_base, kRtTmemCols);
}

// fp32 [rows, k] matrix, box 32 x box_rows, 128-byte swizzle (rows and
// inputs past the matrix read as zeros)
static int make_map_f32(CUtensorMap* m, const float* base, uint64_t k, uint64_t rows, uint32_t box_rows,
                        const char* what) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(ER_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (((uintptr_t)base & 15) || ((k * 4) & 15))
    return fail(ER_EINVAL, "tensor map %s: base and row stride must be 16-byte aligned", what);
  const cuuint64_t dims[2] = {k, rows};
  const cuuint64_t strides[1] = {k * 4};
  const cuuint32_t box[2] = {(cuuint32_t)kRtKBlock, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ER_ECUDA, "cuTensorMapEncodeTiled(%s) failed (%d)", what, (int)r);
  return ER_OK;
}

bool router_tc_ok(int n, int H, int E, const void* wr, const void* wg) {
  return wr && E >= 1 && E + (wg ? 1 : 0) <= kRtRows && n > 64 && H % 8 == 0;
}

int launch_router_tc(const void* h, int h_dtype, int n, int H, const float* wr, const float* wg, int E, float* logits,
                     float* gate_logit, int* tally, int ntally, int* error, cudaStream_t st) {
  if (!router_tc_ok(n, H, E, wr, wg)) return fail(ER_EINVAL, "tensor-core router: n %d, hidden %d, experts %d", n, H, E);
  const bool bf = h_dtype == ER_DTYPE_BF16;
  static int done_dev = -1;
  int dev = 0;
  if (int rc = cuda_check(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (done_dev != dev) {
    for (auto* k : {router_tc_kernel<false>, router_tc_kernel<true>})
      if (int rc = cuda_check(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRtSmem),
                              "router_tc smem attribute"))
        return rc;
    done_dev = dev;
  }
  RtMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (bf) {
    // bf16 tokens: 32 inputs (64 bytes) per row and k-block, unswizzled
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(ER_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
    if (((uintptr_t)h & 15) || ((H * 2) & 15)) return fail(ER_EINVAL, "tensor map router tokens: alignment");
    const cuuint64_t dims[2] = {(cuuint64_t)H, (cuuint64_t)n};
    const cuuint64_t strides[1] = {(cuuint64_t)H * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kRtKBlock, (cuuint32_t)kRtTokens};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(&maps.h, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(h), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(ER_ECUDA, "cuTensorMapEncodeTiled(router tokens) failed (%d)", (int)r);
  } else if (int rc = make_map_f32(&maps.h, static_cast<const float*>(h), H, n, kRtTokens, "router tokens")) {
    return rc;
  }
  if (int rc = make_map_f32(&maps.w, wr, H, E, kRtRows, "router rows")) return rc;
  if (wg)
    if (int rc = make_map_f32(&maps.gate, wg, H, 1, kRtGateRows, "shared gate row")) return rc;
  RtArgs a;
  a.n = n;
  a.H = H;
  a.E = E;
  a.has_gate = wg != nullptr;
  a.logits = logits;
  a.gate_logit = gate_logit;
  a.tally = tally;
  a.ntally = ntally;
  a.error = error;
  a.wait_ns = kDefaultWaitNs;
  const dim3 grid((n + kRtTokens - 1) / kRtTokens, kRouterKSplit);
  if (int rc = launch_chained(bf ? router_tc_kernel<true> : router_tc_kernel<false>, grid, dim3(kRtThreads), kRtSmem,
                              st, "router_tc_kernel", maps, a))
    return rc;
  return launch_check("router_tc_kernel");
}

}  // namespace er
