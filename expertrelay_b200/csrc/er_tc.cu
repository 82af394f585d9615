// er_tc.cu -- tensor-core (tcgen05) grouped expert GEMM for sm_100a.
//
// Reference arithmetic: runtime/qwen_moe.py:341-357 (per expert
// down(silu(gate x) * up x), shared expert) over runtime/int8_linear.py:129-138
// (int8 codes times activations, row scale applied to the output).
//
// Design:
//  * Operand A = int8 weight rows, loaded by TMA straight from the store
//    records (3-D tensor maps over the record arena: K x rows x slot), so the
//    weights reach the tensor core with no dequantisation pass.
//  * Operand B = activations as two int8 slices with one fp32 scale per row:
//    x ~= s * (x0 + x1 / 256), x0 = rint(x / s), x1 = rint((x / s - x0) * 256),
//    s = max|x| / 127 (slice_rows_kernel). Each slice gets its own TMEM
//    accumulator; tcgen05.mma kind::i8 accumulates exactly in int32, and the
//    epilogue recombines (D0 + D1 / 256) * s_token * s_row in fp32. The
//    activation error is below 2^-16 of the row's max, so the product is as
//    accurate as the fp32 reference path.
//  * D = weights x tokens: M = 128 weight rows per item, N = the group's
//    tokens (rounded up to 16, at most kTokTile), so decode (a few tokens per
//    expert) and prefill use the same kernel.
//  * One persistent CTA per SM, warp-specialised: warp 0 issues TMA, warp 1
//    allocates TMEM and issues MMAs, warps 2-5 run the epilogue out of TMEM.
//    A 4-stage shared-memory ring and double-buffered accumulators overlap
//    loads, MMAs and epilogue. Every mbarrier wait is bounded: after
//    kWaitNs the kernel sets an abort flag and an error bit in the plan,
//    drains what it has in flight and frees its TMEM.
//  mode 0: A = gate rows and up rows of 128 intermediate columns; four
//          accumulators (gate/up x slice); epilogue writes act = silu(g)*u.
//  mode 1: A = 128 rows of down; two accumulators; epilogue writes
//          y = acc * s_down * routing weight (sigmoid gate for the shared expert).
#include <cuda.h>
#include <string.h>

#include "er_internal.cuh"

namespace er {

constexpr int kTcStages = 4;
constexpr int kTcStageBytes = 48 * 1024;
constexpr int kTcEpiWarps = 4;
constexpr int kTcThreads = (2 + kTcEpiWarps) * 32;
constexpr int kTcAccCols = 256;  // TMEM columns per accumulator set (x2 buffers = 512)
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s
constexpr size_t kTcSmem = (size_t)kTcStages * kTcStageBytes + 2048;

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with `parity` to complete. Returns false (and
// raises the CTA's abort flag) after kWaitNs, or at once if another role
// already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_test(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_test(bar, parity)) return true;
    if ((i & 63) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > kWaitNs) {
        *abort_flag = 1;
        return false;
      }
    }
  }
}
// Bounded wait used while draining after an abort (no abort check).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity, unsigned long long ns) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_test(bar, parity) && globaltimer() - t0 < ns) {
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), LBO unused (1), descriptor version 1.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::i8: D s32, A and B signed int8, both K-major.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------
// activation slicing
// ---------------------------------------------------------------------------

// One warp per output row: s = max|x| / 127, x0 = rint(x/s), x1 = rint((x/s - x0) * 256)
// clamped to +-127. src_mode 0: row p < nk is h[perm_token[p]], row nk + t is
// h[t]; src_mode 1: row p is src[p] (contiguous rows of width K).
template <typename XT>
__global__ void __launch_bounds__(256) slice_rows_kernel(const XT* __restrict__ src, const int32_t* __restrict__ perm_token,
                                                         int nk, int rows, int K, int src_mode,
                                                         int8_t* __restrict__ s0, int8_t* __restrict__ s1,
                                                         float* __restrict__ scale) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const XT* x;
  if (src_mode == 0)
    x = src + (size_t)(row < nk ? perm_token[row] : row - nk) * K;
  else
    x = src + (size_t)row * K;
  float amax = 0.f;
  for (int k = lane * 4; k < K; k += 128) {
    const float4 v = load4(x + k);
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float s = amax / 127.f;
  const float inv = amax > 0.f ? 127.f / amax : 0.f;
  int8_t* d0 = s0 + (size_t)row * K;
  int8_t* d1 = s1 + (size_t)row * K;
  for (int k = lane * 4; k < K; k += 128) {
    const float4 v = load4(x + k);
    const float f[4] = {v.x, v.y, v.z, v.w};
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float y = f[j] * inv;
      const float q0 = rintf(y);
      const float q1 = fminf(fmaxf(rintf((y - q0) * 256.f), -127.f), 127.f);
      w0 |= (uint32_t)((int)q0 & 0xff) << (8 * j);
      w1 |= (uint32_t)((int)q1 & 0xff) << (8 * j);
    }
    *reinterpret_cast<uint32_t*>(d0 + k) = w0;
    *reinterpret_cast<uint32_t*>(d1 + k) = w1;
  }
  if (lane == 0) scale[row] = s;
}

// ---------------------------------------------------------------------------
// the GEMM
// ---------------------------------------------------------------------------

struct TcMaps {
  CUtensorMap a_routed[2];  // mode 0: gate, up over the arena; mode 1: down in [0]
  CUtensorMap a_shared[2];  // the same for the shared-expert record (2-D)
  CUtensorMap b_routed[2];  // activation slices of the routed rows
  CUtensorMap b_shared[2];  // activation slices of the shared rows (mode 1; mode 0 uses b_routed)
};

struct TcArgs {
  GroupArgs g;
  const uint8_t* arena;      // base of the routed-record arena
  int arena_slots;
  size_t record_bytes;
  int sched;
  const float* xscale_r;     // per-row slice scale of the B rows (routed / all rows in mode 0)
  const float* xscale_s;     // mode 1: shared rows
  float* out_r;              // mode 0: act routed [nk, I]; mode 1: y routed [nk, H]
  float* out_s;              // mode 0: act shared [n, Is]; mode 1: y shared [n, H]
  Plan* plan_rw;             // error bits
};

template <int MODE>
struct TcGeom {
  static constexpr int kTokTile = MODE == 0 ? kTcTokTileGU : kTcTokTileDN;  // B rows (tokens) per item
  static constexpr int kNumAcc = MODE == 0 ? 4 : 2;      // accumulators per item
  static constexpr int kABytes = MODE == 0 ? 32768 : 16384;
  static constexpr int kBSliceBytes = kTokTile * 128;
  static constexpr int kTxBytes = kABytes + 2 * kBSliceBytes;
};

struct TcItem {
  int g, shared, valid;
  int unit0;   // first weight row of the tile (mode 0: intermediate column; mode 1: hidden row)
  int tok0;    // first token of the tile within the group
  int nvalid;  // tokens in the tile
  int npad;    // MMA N (multiple of 16)
  int brow0;   // first B row in the operand matrix
  int slot;    // arena slot of the routed record
  int units, K, nkb;
};

template <int MODE>
__device__ __forceinline__ bool tc_item(const TcArgs& t, int item, TcItem& it) {
  using Geo = TcGeom<MODE>;
  int local = 0;
  const int g = find_item(t.g.plan, t.sched, item, &local);
  if (g < 0) return false;
  const Plan* P = t.g.plan;
  it.g = g;
  it.shared = (g == t.g.E);
  const int inter = it.shared ? t.g.Is : t.g.I;
  it.units = MODE == 0 ? inter : t.g.H;
  it.K = MODE == 0 ? t.g.H : inter;
  it.nkb = (it.K + 127) / 128;
  const int ntiles = (it.units + kTcUnits - 1) / kTcUnits;
  const int rows = P->counts[g];
  it.tok0 = (local / ntiles) * Geo::kTokTile;
  it.unit0 = (local % ntiles) * kTcUnits;
  it.nvalid = min(Geo::kTokTile, rows - it.tok0);
  it.npad = (it.nvalid + 15) & ~15;
  if (MODE == 0)
    it.brow0 = (it.shared ? P->nk : P->offsets[g]) + it.tok0;
  else
    it.brow0 = (it.shared ? 0 : P->offsets[g]) + it.tok0;
  it.valid = 1;
  it.slot = 0;
  if (!it.shared) {
    const uint64_t addr = t.g.expert_records[g];
    const uint64_t base = (uint64_t)t.arena;
    if (addr < base || (addr - base) % t.record_bytes != 0 || (addr - base) / t.record_bytes >= (uint64_t)t.arena_slots) {
      it.valid = 0;  // record outside the arena: reported, never loaded
    } else {
      it.slot = (int)((addr - base) / t.record_bytes);
    }
  }
  return true;
}

template <int MODE>
__global__ void __launch_bounds__(kTcThreads, 1) tc_expert_gemm_kernel(const __grid_constant__ TcMaps maps, TcArgs t) {
  using Geo = TcGeom<MODE>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kTcStages * kTcStageBytes);
  uint64_t* empty = full + kTcStages;
  uint64_t* acc_full = empty + kTcStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kTcEpiWarps * 32);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * kTcAccCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const Plan* P = t.g.plan;
  const int total = P->item_start[t.sched][P->num_active];

  if (warp == 0) {
    // ---------------- TMA producer (lane 0 issues; the warp moves in step) ----------------
    uint32_t kc = 0;  // k-blocks issued so far
    bool ok = true;
    for (int item = blockIdx.x; ok && item < total; item += gridDim.x) {
      TcItem it;
      if (!tc_item<MODE>(t, item, it)) break;
      if (!it.valid) continue;
      for (int kb = 0; kb < it.nkb; ++kb, ++kc) {
        const int s = kc % kTcStages;
        const uint32_t ph = (kc / kTcStages) & 1;
        bool w = true;
        if (lane == 0) w = mbar_wait(&empty[s], ph ^ 1, abort_flag);
        if (!__shfl_sync(0xffffffffu, (int)w, 0)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t* st = smem + s * kTcStageBytes;
          mbar_expect_tx(&full[s], Geo::kTxBytes);
          const int x = kb * 128;
          if (MODE == 0) {
            if (it.shared) {
              tma_load_2d(st, &maps.a_shared[0], &full[s], x, it.unit0);
              tma_load_2d(st + 16384, &maps.a_shared[1], &full[s], x, it.unit0);
            } else {
              tma_load_3d(st, &maps.a_routed[0], &full[s], x, it.unit0, it.slot);
              tma_load_3d(st + 16384, &maps.a_routed[1], &full[s], x, it.unit0, it.slot);
            }
            tma_load_2d(st + Geo::kABytes, &maps.b_routed[0], &full[s], x, it.brow0);
            tma_load_2d(st + Geo::kABytes + Geo::kBSliceBytes, &maps.b_routed[1], &full[s], x, it.brow0);
          } else {
            if (it.shared) {
              tma_load_2d(st, &maps.a_shared[0], &full[s], x, it.unit0);
              tma_load_2d(st + Geo::kABytes, &maps.b_shared[0], &full[s], x, it.brow0);
              tma_load_2d(st + Geo::kABytes + Geo::kBSliceBytes, &maps.b_shared[1], &full[s], x, it.brow0);
            } else {
              tma_load_3d(st, &maps.a_routed[0], &full[s], x, it.unit0, it.slot);
              tma_load_2d(st + Geo::kABytes, &maps.b_routed[0], &full[s], x, it.brow0);
              tma_load_2d(st + Geo::kABytes + Geo::kBSliceBytes, &maps.b_routed[1], &full[s], x, it.brow0);
            }
          }
        }
        __syncwarp();
      }
    }
    if (!ok && lane == 0) {
      // aborted: let every stage this thread filled land before the CTA exits
      for (int s = 0; s < kTcStages; ++s) {
        if (kc > (uint32_t)s) {
          const uint32_t last = kc - 1 - ((kc - 1 - s) % kTcStages);
          mbar_drain(&full[s], (last / kTcStages) & 1, 100000000ull);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer (lane 0 issues; the warp moves in step) ----------------
    uint32_t kc = 0, ic = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < total; item += gridDim.x) {
      TcItem it;
      if (!tc_item<MODE>(t, item, it)) break;
      if (!it.valid) continue;
      const int ab = ic & 1;
      const uint32_t aph = (ic >> 1) & 1;
      bool w = true;
      if (lane == 0) w = mbar_wait(&acc_empty[ab], aph ^ 1, abort_flag);
      if (!__shfl_sync(0xffffffffu, (int)w, 0)) break;
      tc_fence_after();
      const uint32_t d0 = tmem_base + ab * kTcAccCols;
      const uint32_t idesc = idesc_i8(128, it.npad);
      for (int kb = 0; kb < it.nkb; ++kb, ++kc) {
        const int s = kc % kTcStages;
        const uint32_t ph = (kc / kTcStages) & 1;
        if (lane == 0) w = mbar_wait(&full[s], ph, abort_flag);
        if (!__shfl_sync(0xffffffffu, (int)w, 0)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t st = smem_u32(smem + s * kTcStageBytes);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint32_t acc = (kb > 0 || ks > 0) ? 1u : 0u;
            const uint64_t b0 = umma_desc_sw128(st + Geo::kABytes + ks * 32);
            const uint64_t b1 = umma_desc_sw128(st + Geo::kABytes + Geo::kBSliceBytes + ks * 32);
            const uint64_t a0 = umma_desc_sw128(st + ks * 32);
            mma_i8(d0 + 0 * Geo::kTokTile, a0, b0, idesc, acc);
            mma_i8(d0 + 1 * Geo::kTokTile, a0, b1, idesc, acc);
            if (MODE == 0) {
              const uint64_t a1 = umma_desc_sw128(st + 16384 + ks * 32);
              mma_i8(d0 + 2 * Geo::kTokTile, a1, b0, idesc, acc);
              mma_i8(d0 + 3 * Geo::kTokTile, a1, b1, idesc, acc);
            }
          }
          umma_commit(&empty[s]);  // frees the stage once these MMAs have read it
        }
        __syncwarp();
      }
      if (!ok) break;
      if (lane == 0) umma_commit(&acc_full[ab]);  // accumulators ready for the epilogue
      __syncwarp();
      ++ic;
    }
    if (lane == 0) {
      // every MMA issued by this thread has finished before TMEM is released
      umma_commit(drain_bar);
      mbar_drain(drain_bar, 0, 100000000ull);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2..5, 128 threads = 128 TMEM lanes) ----------------
    const int quad = warp & 3;              // TMEM lanes quad*32 .. +31 of this warp
    const int r_local = quad * 32 + lane;   // weight row within the tile
    uint32_t ic = 0;
    for (int item = blockIdx.x; item < total; item += gridDim.x) {
      TcItem it;
      if (!tc_item<MODE>(t, item, it)) break;
      if (!it.valid) {
        if (threadIdx.x == 64) atomicOr(&t.plan_rw->error, 4);
        continue;
      }
      const int ab = ic & 1;
      const uint32_t aph = (ic >> 1) & 1;
      const bool w = mbar_wait(&acc_full[ab], aph, abort_flag);
      if (!__all_sync(0xffffffffu, w)) break;
      tc_fence_after();
      const int row = it.unit0 + r_local;
      const bool row_ok = row < it.units;
      const uint8_t* rec = it.shared ? t.g.shared_record : reinterpret_cast<const uint8_t*>(t.g.expert_records[it.g]);
      const RecordGeom geo{ER_FMT_INT8, t.g.H, it.shared ? t.g.Is : t.g.I, 1};
      float sw0 = 0.f, sw1 = 0.f;
      if (row_ok) {
        if (MODE == 0) {
          sw0 = reinterpret_cast<const float*>(rec + geo.scale_offset(0))[row];
          sw1 = reinterpret_cast<const float*>(rec + geo.scale_offset(1))[row];
        } else {
          sw0 = reinterpret_cast<const float*>(rec + geo.scale_offset(2))[row];
        }
      }
      const uint32_t tbase = tmem_base + ab * kTcAccCols + ((uint32_t)(quad * 32) << 16);
      const int inter = it.shared ? t.g.Is : t.g.I;
      for (int c0 = 0; c0 < it.npad; c0 += 16) {
        uint32_t v0[16], v1[16], v2[16], v3[16];
        tmem_ld16(tbase + 0 * Geo::kTokTile + c0, v0);
        tmem_ld16(tbase + 1 * Geo::kTokTile + c0, v1);
        if (MODE == 0) {
          tmem_ld16(tbase + 2 * Geo::kTokTile + c0, v2);
          tmem_ld16(tbase + 3 * Geo::kTokTile + c0, v3);
        }
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int tk = c0 + j;
            if (tk < it.nvalid) {
              const int brow = it.brow0 + tk;
              if (MODE == 0) {
                const float xs = t.xscale_r[brow];
                const float gv = ((float)(int)v0[j] + (float)(int)v1[j] * (1.f / 256.f)) * xs * sw0;
                const float uv = ((float)(int)v2[j] + (float)(int)v3[j] * (1.f / 256.f)) * xs * sw1;
                float* dst = it.shared ? t.out_s + (size_t)(it.tok0 + tk) * inter
                                       : t.out_r + (size_t)brow * t.g.I;
                dst[row] = silu_f(gv) * uv;
              } else {
                const float xs = it.shared ? t.xscale_s[brow] : t.xscale_r[brow];
                const float yv = ((float)(int)v0[j] + (float)(int)v1[j] * (1.f / 256.f)) * xs * sw0;
                if (it.shared)
                  t.out_s[(size_t)brow * t.g.H + row] = yv * t.g.gate_sig[brow];
                else
                  t.out_r[(size_t)brow * t.g.H + row] = yv * t.g.perm_w[brow];
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[ab]);
      ++ic;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (*abort_flag && threadIdx.x == 0) atomicOr(&t.plan_rw->error, 8);
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(2 * kTcAccCols));
  }
}

// ---------------------------------------------------------------------------
// host side: tensor maps and launches
// ---------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// int8 tensor map, K innermost (contiguous), 128-byte swizzle, box 128 x box_rows [x 1].
static int make_map(CUtensorMap* m, const void* base, int rank, uint64_t k, uint64_t rows, uint64_t slots,
                    uint64_t row_stride, uint64_t slot_stride, uint32_t box_rows, const char* what) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(ER_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (((uintptr_t)base & 15) || (row_stride & 15) || (rank == 3 && (slot_stride & 15)))
    return fail(ER_EINVAL, "tensor map %s: base and strides must be 16-byte aligned", what);
  const cuuint64_t dims[3] = {k, rows, slots};
  const cuuint64_t strides[2] = {row_stride, slot_stride};
  const cuuint32_t box[3] = {128, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, (cuuint32_t)rank, const_cast<void*>(base), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ER_ECUDA, "cuTensorMapEncodeTiled(%s) failed (%d)", what, (int)r);
  return ER_OK;
}

template <int MODE>
static int configure_tc() {
  static int done_dev = -1;
  int dev = 0;
  if (int rc = cuda_check(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (done_dev == dev) return ER_OK;
  if (int rc = cuda_check(cudaFuncSetAttribute(tc_expert_gemm_kernel<MODE>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem),
                          "tc smem attribute"))
    return rc;
  done_dev = dev;
  return ER_OK;
}

int launch_slice_rows(const void* src, int dtype, const int32_t* perm_token, int nk, int rows, int K, int src_mode,
                      int8_t* s0, int8_t* s1, float* scale, cudaStream_t st) {
  if (rows <= 0) return ER_OK;
  const int blocks = (rows + 7) / 8;
  if (dtype == ER_DTYPE_BF16)
    slice_rows_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>((const __nv_bfloat16*)src, perm_token, nk, rows, K,
                                                             src_mode, s0, s1, scale);
  else
    slice_rows_kernel<float><<<blocks, 256, 0, st>>>((const float*)src, perm_token, nk, rows, K, src_mode, s0, s1,
                                                     scale);
  return launch_check("slice_rows_kernel");
}

int launch_tc_grouped(const TcLaunch& L, cudaStream_t st) {
  const GroupArgs& a = L.g;
  TcMaps maps;
  memset(&maps, 0, sizeof(maps));
  const RecordGeom rg{ER_FMT_INT8, a.H, a.I, 1};
  const RecordGeom sg{ER_FMT_INT8, a.H, a.Is, 1};
  const uint8_t* arena = static_cast<const uint8_t*>(L.arena);
  const uint8_t* shr = a.shared_record;
  const int rows_b0 = L.nk + L.n;
  if (L.mode == 0) {
    if (int rc = make_map(&maps.a_routed[0], arena + rg.weight_offset(0), 3, a.H, a.I, L.arena_slots, a.H,
                          L.record_bytes, 128, "gate"))
      return rc;
    if (int rc = make_map(&maps.a_routed[1], arena + rg.weight_offset(1), 3, a.H, a.I, L.arena_slots, a.H,
                          L.record_bytes, 128, "up"))
      return rc;
    if (int rc = make_map(&maps.a_shared[0], shr + sg.weight_offset(0), 2, a.H, a.Is, 1, a.H, 0, 128, "shared gate"))
      return rc;
    if (int rc = make_map(&maps.a_shared[1], shr + sg.weight_offset(1), 2, a.H, a.Is, 1, a.H, 0, 128, "shared up"))
      return rc;
    if (int rc = make_map(&maps.b_routed[0], L.b0_r, 2, a.H, rows_b0, 1, a.H, 0, TcGeom<0>::kTokTile, "x slice 0"))
      return rc;
    if (int rc = make_map(&maps.b_routed[1], L.b1_r, 2, a.H, rows_b0, 1, a.H, 0, TcGeom<0>::kTokTile, "x slice 1"))
      return rc;
  } else {
    if (int rc = make_map(&maps.a_routed[0], arena + rg.weight_offset(2), 3, a.I, a.H, L.arena_slots, a.I,
                          L.record_bytes, 128, "down"))
      return rc;
    if (int rc = make_map(&maps.a_shared[0], shr + sg.weight_offset(2), 2, a.Is, a.H, 1, a.Is, 0, 128, "shared down"))
      return rc;
    const int tt = TcGeom<1>::kTokTile;
    if (L.nk > 0) {
      if (int rc = make_map(&maps.b_routed[0], L.b0_r, 2, a.I, L.nk, 1, a.I, 0, tt, "act slice 0")) return rc;
      if (int rc = make_map(&maps.b_routed[1], L.b1_r, 2, a.I, L.nk, 1, a.I, 0, tt, "act slice 1")) return rc;
    }
    if (int rc = make_map(&maps.b_shared[0], L.b0_s, 2, a.Is, L.n, 1, a.Is, 0, tt, "shared act slice 0")) return rc;
    if (int rc = make_map(&maps.b_shared[1], L.b1_s, 2, a.Is, L.n, 1, a.Is, 0, tt, "shared act slice 1")) return rc;
  }
  TcArgs t;
  t.g = a;
  t.arena = arena;
  t.arena_slots = L.arena_slots;
  t.record_bytes = L.record_bytes;
  t.sched = L.sched;
  t.xscale_r = L.xscale_r;
  t.xscale_s = L.xscale_s;
  t.out_r = L.out_r;
  t.out_s = L.out_s;
  t.plan_rw = const_cast<Plan*>(a.plan);
  int sms = 148;
  if (int rc = er_device_sm_count(&sms)) return rc;
  const int grid = (int)(L.items_bound < sms ? (L.items_bound > 0 ? L.items_bound : 1) : sms);
  if (L.mode == 0) {
    if (int rc = configure_tc<0>()) return rc;
    tc_expert_gemm_kernel<0><<<grid, kTcThreads, kTcSmem, st>>>(maps, t);
  } else {
    if (int rc = configure_tc<1>()) return rc;
    tc_expert_gemm_kernel<1><<<grid, kTcThreads, kTcSmem, st>>>(maps, t);
  }
  return launch_check("tc_expert_gemm_kernel");
}

}  // namespace er
