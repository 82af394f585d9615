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
//  * One persistent CTA per SM, warp-specialised: one warp issues TMA, one
//    allocates TMEM and issues MMAs, eight run the epilogue out of TMEM.
//    A shared-memory ring and a ring of TMEM accumulators overlap loads,
//    MMAs and epilogue. Every mbarrier wait is bounded: after the launch's
//    wait bound (2 s unless a test shortens it) the
//    kernel sets an abort flag and an error bit in the plan, drains what it
//    has in flight and frees its TMEM.
//  * 128-token tiles run on SM pairs (a cluster of 2, tcgen05 cta_group::2):
//    one MMA is M = 256 weight rows (128 from each CTA's shared memory) by
//    N = 256 (slice 0 of the 128 tokens from CTA 0, slice 1 from CTA 1), so
//    each SM loads 32 KB per 128-deep K block instead of 48 KB for the same
//    MMA work. CTA 0 issues the MMAs and commits to both CTAs' barriers;
//    CTA 1's loads complete on CTA 0's full barriers and its epilogue frees
//    the accumulator on CTA 0's barrier. No load uses cluster multicast.
//    16-token tiles (decode) run on single SMs: there the weight bytes, not
//    the activations, bound the kernel.
//  mode 0: A = gate rows and up rows of 128 intermediate columns; four
//          accumulators (gate/up x slice); epilogue writes act = silu(g)*u.
//  mode 1: A = 128 rows of down; two accumulators; epilogue writes
//          y = acc * s_down * routing weight (sigmoid gate for the shared expert).
#include "er_tc.cuh"

namespace er {

// Warp roles. A warp runs on SM sub-partition (warp % 4) and may read TMEM
// lanes 32 * (warp % 4) .. +31 only. The 8 epilogue warps are 4..11 (two per
// lane quadrant); quadrants 2 and 3 hold the up rows, whose warps only hand
// values over, so the MMA issuer (warp 2) and the TMA producer (warp 3) share
// those two sub-partitions and are not held up by the gate warps' math.
// Warps 0 and 1 have no role.
constexpr int kTcEpiWarps = 8;
constexpr int kTcEpiWarp0 = 4;
constexpr int kTcMmaWarp = 2;
constexpr int kTcTmaWarp = 3;
constexpr int kTcThreads = (kTcEpiWarp0 + kTcEpiWarps) * 32;
static_assert(kTcThreads >= kMaxExperts + 2, "tc_cache_plan reads one plan entry per thread");
constexpr int kTcTmemCols = 512;  // TMEM columns allocated: a ring of accumulators

// ---------------------------------------------------------------------------
// activation slicing
// ---------------------------------------------------------------------------

// One warp per row of a [rows, K] matrix: s = max|x| / 127 and the two int8
// slices (slice4). Rows of up to 2048 values are held in registers and read
// once; longer rows are read twice (max, then slices).
template <typename XT>
__device__ __forceinline__ void slice_row_warp(const XT* __restrict__ src, int row, int K, int8_t* __restrict__ s0,
                                               int8_t* __restrict__ s1, float* __restrict__ scale, int lane) {
  constexpr int kRegVec = 16;  // float4 per lane held in registers: K <= 2048
  const XT* x = src + (size_t)row * K;
  int8_t* d0 = s0 + (size_t)row * K;
  int8_t* d1 = s1 + (size_t)row * K;
  auto emit = [&](int k, float4 v, float inv) {
    uint32_t w0, w1;
    slice4(v, inv, w0, w1);
    *reinterpret_cast<uint32_t*>(d0 + k) = w0;
    *reinterpret_cast<uint32_t*>(d1 + k) = w1;
  };
  float amax = 0.f;
  if (K <= 128 * kRegVec) {
    float4 v[kRegVec];
#pragma unroll
    for (int i = 0; i < kRegVec; ++i) {
      const int k = lane * 4 + 128 * i;
      v[i] = k < K ? load4(x + k) : make_float4(0.f, 0.f, 0.f, 0.f);
      amax = fmaxf(amax, abs_max4(v[i]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float inv = amax > 0.f ? 127.f / amax : 0.f;
#pragma unroll
    for (int i = 0; i < kRegVec; ++i) {
      const int k = lane * 4 + 128 * i;
      if (k < K) emit(k, v[i], inv);
    }
  } else {
    for (int k = lane * 4; k < K; k += 128) amax = fmaxf(amax, abs_max4(load4(x + k)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float inv = amax > 0.f ? 127.f / amax : 0.f;
    for (int k = lane * 4; k < K; k += 128) emit(k, load4(x + k), inv);
  }
  if (lane == 0) scale[row] = amax / 127.f;
}

template <typename XT>
__global__ void __launch_bounds__(256) slice_rows_kernel(const XT* __restrict__ src, int rows, int K,
                                                         int8_t* __restrict__ s0, int8_t* __restrict__ s1,
                                                         float* __restrict__ scale) {
  chain_wait();
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row < rows) slice_row_warp(src, row, K, s0, s1, scale, threadIdx.x & 31);
}

// ---------------------------------------------------------------------------
// the GEMM
// ---------------------------------------------------------------------------

// ---------------------------------------------------------------------------
// the GEMM
// ---------------------------------------------------------------------------

// TT = tokens per work item (128 for prefill, 16 for decode batches).
// A tile: 128 weight rows x 128 bytes of K per stage (mode 0: 64 gate rows,
// then the same 64 columns' up rows). B tile: slice 0 of TT token rows, then
// slice 1 of the same rows, so ONE MMA with N = TT + npad covers both slices
// and reads A once. The accumulator holds slice 0 in columns [0, TT) and
// slice 1 in [TT, 2 TT).
//
// CG = CTAs per item (1: one SM; 2: an SM pair, cta_group::2). Per stage a CTA
// holds its 128 weight rows and, on one SM, both slices (N = TT + npad), on a
// pair only its own slice (CTA r: slice r; the pair's MMA has N = 2 TT).
//
// A stage holds kKC 128-byte K chunks (each a 128-byte-swizzled tile of its
// own): [A chunk 0][A chunk 1].. then [B chunk 0][B chunk 1]..
template <int MODE, int TT, int CG>
struct TcGeom {
  static constexpr int kKC = 2;                  // 128-byte K chunks per stage
  static constexpr int kAChunkBytes = 16384;     // 128 weight rows x 128 bytes
  static constexpr int kABytes = kKC * kAChunkBytes;
  static constexpr int kBSliceBytes = TT * 128;  // one slice, one chunk
  static constexpr int kBChunkBytes = (3 - CG) * kBSliceBytes;
  static constexpr int kBBytes = kKC * kBChunkBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTxBytes = CG * kStageBytes;  // bytes completing on the (CTA 0) full barrier per stage
  // 3 stages of 64 KB on pairs; 5 of 40 KB for 16-token tiles, whose
  // throughput is set by copies in flight (a stage's turn-around is a
  // DRAM round trip plus its MMAs)
  static constexpr int kStages = (TT >= 128 ? 196608 : 204800) / kStageBytes;
  static constexpr int kCtaUnits = MODE == 0 ? 64 : 128;  // this CTA's intermediate columns / hidden rows
  static constexpr int kUnits = CG * kCtaUnits;           // per item
  static constexpr size_t kRingBytes = (size_t)kStages * kStageBytes;
  static constexpr size_t kXchBytes = MODE == 0 ? 4 * 2 * 16 * 32 * 4 : 0;  // gate/up exchange
  static constexpr int kChunks = (TT + 31) / 32;  // 16-token TMEM chunks per epilogue warp
  // Accumulators: 2 TT columns each (both slices; on a pair, one slice per
  // CTA). 128-token tiles double-buffer 256 columns; 16-token tiles keep a
  // ring of 16, so the MMAs run up to 15 items ahead of the epilogue (whose
  // first item, with every cache cold, takes several items' time).
  static constexpr int kAccCols = 2 * TT;
  static constexpr int kAccBufs = kTcTmemCols / kAccCols;
  static_assert(kAccBufs >= 2 && kAccBufs <= 16, "accumulator ring");
  // + 1024: the kernel rounds the dynamic shared memory base up to 1024 bytes
  static constexpr size_t kSmem = 1024 + kRingBytes + kXchBytes + 2048 + sizeof(struct TcPlanCache);
  static_assert(kSmem <= 232448, "shared memory per CTA");
};

template <int MODE, int TT, int CG>
__device__ __forceinline__ bool tc_item(const TcArgs& t, const TcPlanCache* pc, int item, TcItem& it) {
  using Geo = TcGeom<MODE, TT, CG>;
  return tc_item_at<MODE, 128 * Geo::kKC, Geo::kUnits, TT>(t, pc, item, it);
}

template <int MODE, int TT, int CG>
__global__ void __launch_bounds__(kTcThreads, 1) tc_expert_gemm_kernel(const __grid_constant__ TcMaps maps, TcArgs t) {
  using Geo = TcGeom<MODE, TT, CG>;
  constexpr int S = Geo::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* xch = reinterpret_cast<float*>(smem + Geo::kRingBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Geo::kRingBytes + Geo::kXchBytes);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + Geo::kAccBufs;
  uint64_t* drain_bar = acc_empty + Geo::kAccBufs;
  uint64_t* xfull = drain_bar + 1;   // [pair*2 + half][buffer]: u values written
  uint64_t* xempty = xfull + 8;      // [pair*2 + half][buffer]: u values consumed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xempty + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  TcPlanCache* pc = reinterpret_cast<TcPlanCache*>(smem + Geo::kRingBytes + Geo::kXchBytes + 2048);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // pair kernels: CTA 0 of the cluster issues the MMAs; items go to pairs
  const uint32_t rank = CG == 2 ? cluster_rank() : 0u;
  const bool leader = rank == 0;
  const int first_item = CG == 2 ? (int)cluster_id() : (int)blockIdx.x;
  const int item_stride = CG == 2 ? (int)cluster_count() : (int)gridDim.x;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < Geo::kAccBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], CG * kTcEpiWarps);  // one arrival per epilogue warp of each CTA
    }
    mbar_init(drain_bar, 1);
    for (int i = 0; i < 8; ++i) {
      mbar_init(&xfull[i], 1);
      mbar_init(&xempty[i], 1);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kTcTmaWarp && lane == 0) prefetch_maps(maps, t.maps_used);
  // Decode tiles: the next kernel (slices or combine, a few small CTAs that
  // fit beside this one) may launch early and wait in its chain_wait, so it
  // starts the moment this grid completes. The down GEMM lets the combine
  // launch now; the gate/up GEMM lets the slice launch only after its own
  // wait, i.e. once the dispatch (and with it the plan) is complete, so the
  // down GEMM launched after the slice reads the plan before its wait.
  if constexpr (TT == 16 && MODE == 1) chain_trigger();
  // Decode tiles: a CTA loads its first item's first weight stages before
  // its wait, while the kernels before it still run. Gate/up: the shared
  // expert's items come first in both schedules and are laid out from the
  // launch's sizes alone, so CTAs whose first item is one of them do. Down:
  // the plan is complete (above), so every CTA reads it first and does. The
  // full barriers get the weight bytes without an arrival; the producer adds
  // the activation bytes and arrives after the wait, and checks that the
  // plan agrees.
  // producer: first-item k-blocks whose weights are in flight, and where
  // their activation rows start (down: the row; gate/up: the token tile)
  int pre_n = 0, pre_kb0 = 0, pre_row = 0, pre_sh = 1;
  bool plan_read = false;
  if constexpr (TT == 16) {
    __syncthreads();  // the barriers are initialised
    if constexpr (MODE == 1) {
      tc_cache_plan<true>(t, pc);
      __syncthreads();
      plan_read = true;
      if (warp == kTcTmaWarp) {
        TcItem p;
        if (tc_item<MODE, TT, CG>(t, pc, first_item, p) && p.valid) {
          pre_n = min(p.nkb, S);
          pre_kb0 = p.kb0;
          pre_row = p.brow0;
          pre_sh = p.shared;
          if (lane == 0) {
            const uint64_t pol = l2_evict_first();
#pragma unroll 1
            for (int kb = 0; kb < pre_n; ++kb) {
              uint8_t* st = smem + kb * Geo::kStageBytes;
              mbar_expect_tx_only(&full[kb], Geo::kABytes);
#pragma unroll 1
              for (int c = 0; c < Geo::kKC; ++c) {
                const int x = ((p.kb0 + kb) * Geo::kKC + c) * 128;
                uint8_t* sa = st + c * Geo::kAChunkBytes;
                if (p.shared)
                  tma_w2d<CG>(sa, &maps.a_shared[0], &full[kb], 0u, x, p.unit0, pol);
                else
                  tma_w3d<CG>(sa, &maps.a_routed[0], &full[kb], 0u, x, p.unit0, p.slot, pol);
              }
            }
          }
        }
        __syncwarp();
      }
    } else if (warp == kTcTmaWarp && t.pre_shared && first_item < tc_shared_items<MODE, Geo::kUnits, TT>(t)) {
      TcItem p;
      tc_item_local<MODE, 128 * Geo::kKC, Geo::kUnits, TT>(t, true, t.g.n, first_item, p);
      pre_n = min(p.nkb, S);
      pre_kb0 = p.kb0;
      pre_row = p.tok0;
      if (lane == 0) {
        const uint64_t pol = l2_evict_first();
#pragma unroll 1
        for (int kb = 0; kb < pre_n; ++kb) {
          uint8_t* st = smem + kb * Geo::kStageBytes;
          mbar_expect_tx_only(&full[kb], Geo::kABytes);
#pragma unroll 1
          for (int c = 0; c < Geo::kKC; ++c) {
            const int x = ((p.kb0 + kb) * Geo::kKC + c) * 128;
            uint8_t* sa = st + c * Geo::kAChunkBytes;
            tma_w2d<CG>(sa, &maps.a_shared[0], &full[kb], 0u, x, p.unit0, pol);
            if (MODE == 0) tma_w2d<CG>(sa + 8192, &maps.a_shared[1], &full[kb], 0u, x, p.unit0, pol);
          }
        }
      }
      __syncwarp();
    }
  }
  // everything above touched only this CTA's shared memory (and read the
  // weights, and on decode down the complete plan); the operands come from
  // the kernels before this one
  chain_wait();
  if constexpr (TT == 16 && MODE == 0) chain_trigger();
  if (!plan_read) tc_cache_plan(t, pc);
  if constexpr (CG == 2) {
    // the peer's loads and arrivals target CTA 0's barriers: both CTAs'
    // barriers are initialised, and both CTAs running, before either goes on
    __syncthreads();
    cluster_sync();
  }
  // one warp of each CTA allocates TMEM (on a pair, the two warps collectively)
  if (warp == kTcMmaWarp) tmem_alloc<CG>(tmem_slot, kTcTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total = pc->total;

  if (warp == kTcTmaWarp) {
    // ---------------- TMA producer (lane 0 issues; the warp moves in step) ----------------
    // decode streams each weight byte once: evict-first, so the L2 keeps the
    // small kernels' code and data between replays
    const uint64_t wpol = TT == 16 ? l2_evict_first() : 0ull;
    uint32_t kc = 0;  // k-blocks issued so far
    bool ok = true;
    int skip = 0;  // k-blocks of the first item issued here, before the loop
    if (pre_n > 0) {
      // gate/up: the plan must make the shared expert the first group with
      // this CTA's first item among its items (the geometry then follows
      // from the launch's sizes, as above); if not (an inconsistent tally
      // leaves no items), report it, let the copies land (the arrivals
      // complete the phases) and stop. Down read the plan before issuing.
      bool same = true;
      if constexpr (MODE == 0)
        same = pc->num_active > 0 && pc->group[0] == t.g.E && first_item < pc->item_start[1] &&
               pc->rows[0] == t.g.n;
      if (!same) {
        ok = false;
        if (lane == 0) {
          atomicOr(&t.plan_rw->error, 8);
          *abort_flag = 1;
          for (int s = 0; s < pre_n; ++s) mbar_arrive(&full[s]);
          for (int s = 0; s < pre_n; ++s) mbar_drain(&full[s], 0, 100000000ull);
        }
        __syncwarp();
      } else {
        // the activation tiles of the stages in flight, straight after the
        // wait (this code runs once per launch, from a cold cache: short)
        const int brow0 = MODE == 0 ? pc->nk + pre_row : pre_row;
        const CUtensorMap* b = (MODE == 1 && pre_sh) ? maps.b_shared : maps.b_routed;
        if (lane == 0) {
#pragma unroll 1
          for (int kb = 0; kb < pre_n; ++kb) {
            uint8_t* sb = smem + kb * Geo::kStageBytes + Geo::kABytes;
            mbar_expect_tx(&full[kb], Geo::kTxBytes - Geo::kABytes);
#pragma unroll 1
            for (int c = 0; c < Geo::kKC; ++c) {
              const int x = ((pre_kb0 + kb) * Geo::kKC + c) * 128;
              tma_2d<CG>(sb + c * Geo::kBChunkBytes, &b[0], &full[kb], 0u, x, brow0);
              tma_2d<CG>(sb + c * Geo::kBChunkBytes + Geo::kBSliceBytes, &b[1], &full[kb], 0u, x, brow0);
            }
          }
        }
        __syncwarp();
        skip = pre_n;
        kc = pre_n;
      }
    }
    for (int item = first_item; ok && item < total; item += item_stride) {
      TcItem it;
      if (!tc_item<MODE, TT, CG>(t, pc, item, it)) break;
      if (!it.valid) continue;
      const int arow = it.unit0 + (int)rank * Geo::kCtaUnits;  // this CTA's first weight row
      for (int kb = item == first_item ? skip : 0; kb < it.nkb; ++kb, ++kc) {
        const int s = kc % S;
        const uint32_t ph = (kc / S) & 1;
        bool w = true;
        w = warp_wait(&empty[s], ph ^ 1, abort_flag, lane, t.wait_ns);
        if (!w) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t* st = smem + s * Geo::kStageBytes;
          // CTA 0 expects the whole pair's bytes; the peer's copies may land
          // before that (the barrier's transaction count goes negative until
          // then, and the phase cannot complete without CTA 0's arrival)
          if (leader) mbar_expect_tx(&full[s], Geo::kTxBytes);
          const uint32_t fc = CG == 2 ? mapa_shared(smem_u32(&full[s]), 0) : 0u;
          const CUtensorMap* b = (MODE == 1 && it.shared) ? maps.b_shared : maps.b_routed;
#pragma unroll(TT == 16 ? 1 : Geo::kKC)
          for (int c = 0; c < Geo::kKC; ++c) {
            // chunks past K read as zeros (out-of-bounds fill) and add nothing
            const int x = ((it.kb0 + kb) * Geo::kKC + c) * 128;
            uint8_t* sa = st + c * Geo::kAChunkBytes;
            uint8_t* sb = st + Geo::kABytes + c * Geo::kBChunkBytes;
            if (MODE == 0) {
              if (it.shared) {
                tma_w2d<CG>(sa, &maps.a_shared[0], &full[s], fc, x, arow, wpol);
                tma_w2d<CG>(sa + 8192, &maps.a_shared[1], &full[s], fc, x, arow, wpol);
              } else {
                tma_w3d<CG>(sa, &maps.a_routed[0], &full[s], fc, x, arow, it.slot, wpol);
                tma_w3d<CG>(sa + 8192, &maps.a_routed[1], &full[s], fc, x, arow, it.slot, wpol);
              }
            } else {
              if (it.shared)
                tma_w2d<CG>(sa, &maps.a_shared[0], &full[s], fc, x, arow, wpol);
              else
                tma_w3d<CG>(sa, &maps.a_routed[0], &full[s], fc, x, arow, it.slot, wpol);
            }
            if (CG == 1) {
              tma_2d<CG>(sb, &b[0], &full[s], fc, x, it.brow0);
              tma_2d<CG>(sb + Geo::kBSliceBytes, &b[1], &full[s], fc, x, it.brow0);
            } else {
              tma_2d<CG>(sb, &b[rank], &full[s], fc, x, it.brow0);
            }
          }
        }
        __syncwarp();
      }
    }
    if (!ok && lane == 0) {
      if (leader) {
        // aborted: let every stage this CTA's barriers track land before the CTA exits
        for (int s = 0; s < S; ++s) {
          if (kc > (uint32_t)s) {
            const uint32_t last = kc - 1 - ((kc - 1 - s) % S);
            mbar_drain(&full[s], (last / S) & 1, 100000000ull);
          }
        }
      } else {
        // the peer's copies complete on CTA 0's barriers, which this CTA
        // cannot wait on: give those in flight 1 ms to land
        const unsigned long long t0 = globaltimer();
        while (globaltimer() - t0 < 1000000ull) {
        }
      }
    }
    __syncwarp();
  } else if (warp == kTcMmaWarp && leader) {
    // ---------------- MMA issuer (lane 0 issues; the warp moves in step) ----------------
    uint32_t kc = 0, ic = 0;
    bool ok = true;
    for (int item = first_item; ok && item < total; item += item_stride) {
      TcItem it;
      if (!tc_item<MODE, TT, CG>(t, pc, item, it)) break;
      if (!it.valid) continue;
      const int ab = ic % Geo::kAccBufs;
      const uint32_t aph = (ic / Geo::kAccBufs) & 1;
      bool w = true;
      w = warp_wait(&acc_empty[ab], aph ^ 1, abort_flag, lane, t.wait_ns);
      if (!w) break;
      tc_fence_after();
      const uint32_t d = tmem_base + ab * Geo::kAccCols;
      const uint32_t idesc = CG == 1 ? idesc_i8(128, TT + it.npad) : idesc_i8(256, 2 * TT);
      for (int kb = 0; kb < it.nkb; ++kb, ++kc) {
        const int s = kc % S;
        const uint32_t ph = (kc / S) & 1;
        w = warp_wait(&full[s], ph, abort_flag, lane, t.wait_ns);
        if (!w) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t st = smem_u32(smem + s * Geo::kStageBytes);
          if constexpr (TT == 16) {
            // one MMA per iteration: short code for a launch that runs it cold
#pragma unroll 1
            for (int q = 0; q < 4 * Geo::kKC; ++q) {
              const int c = q >> 2, ks = q & 3;
              const uint32_t sa = st + c * Geo::kAChunkBytes, sb = st + Geo::kABytes + c * Geo::kBChunkBytes;
              mma_i8<CG>(d, umma_desc_sw128(sa + ks * 32), umma_desc_sw128(sb + ks * 32), idesc,
                         (kb > 0 || q > 0) ? 1u : 0u);
            }
          } else {
#pragma unroll
            for (int c = 0; c < Geo::kKC; ++c) {
              const uint32_t sa = st + c * Geo::kAChunkBytes, sb = st + Geo::kABytes + c * Geo::kBChunkBytes;
#pragma unroll
              for (int ks = 0; ks < 4; ++ks)
                mma_i8<CG>(d, umma_desc_sw128(sa + ks * 32), umma_desc_sw128(sb + ks * 32), idesc,
                           (kb > 0 || c > 0 || ks > 0) ? 1u : 0u);
            }
          }
          umma_commit<CG>(&empty[s]);  // frees the stage (in both CTAs of a pair) once these MMAs have read it
        }
        __syncwarp();
      }
      if (!ok) break;
      // accumulator ready for the epilogue(s); the stall test hook withholds the last item's
      if (lane == 0 && !(t.stall_last && item == total - 1)) umma_commit<CG>(&acc_full[ab]);
      __syncwarp();
      ++ic;
    }
    if (lane == 0) {
      // every MMA issued by this thread has finished before TMEM is released
      umma_commit<CG>(drain_bar);
      mbar_drain(drain_bar, 0, 100000000ull);
    }
    __syncwarp();
  } else if (warp >= kTcEpiWarp0) {
    // ---------------- epilogue (warps 4..11) ----------------
    // Warp w reads TMEM lanes 32*(w%4)..+31 and every other 16-token chunk
    // (half = (w-4)/4). Mode 0: lanes 0..63 hold gate rows, 64..127 the up
    // rows of the same columns; the up warp of each pair hands u to the gate
    // warp through shared memory (named barrier per pair and half).
    const int quad = warp & 3;
    const int half = (warp - kTcEpiWarp0) >> 2;
    const int pair = quad & 1;
    const bool up_warp = MODE == 0 && quad >= 2;
    const int xpb = (pair * 2 + half) * 2;  // exchange barriers of this pair and half
    uint32_t ic = 0, chunk = 0;
    bool alive = true;
    for (int item = first_item; item < total; item += item_stride) {
      TcItem it;
      if (!tc_item<MODE, TT, CG>(t, pc, item, it)) break;
      if (!it.valid) {
        if (threadIdx.x == kTcEpiWarp0 * 32) atomicOr(&t.plan_rw->error, 4);
        continue;
      }
      // this thread's weight row: mode 0 -> intermediate column `col` of gate (or up);
      // mode 1 -> hidden row
      const int col = it.unit0 + (int)rank * Geo::kCtaUnits + (MODE == 0 ? pair * 32 + lane : quad * 32 + lane);
      const bool row_ok = col < it.units;
      const uint8_t* rec = it.shared ? t.g.shared_record : t.arena + (size_t)it.slot * t.record_bytes;
      const RecordGeom geo{ER_FMT_INT8, t.g.H, it.shared ? t.g.Is : t.g.I, 1};
      const int which = MODE == 0 ? (up_warp ? 1 : 0) : 2;
      const float* xsc = (MODE == 1 && it.shared) ? t.xscale_s : t.xscale_r;
      const float* tokw = it.shared ? t.g.gate_sig : t.g.perm_w;
      // the row scale and the item's per-token scales (and, for down, routing
      // weights) are fetched before the wait for the accumulator, so their
      // latency hides behind the item's MMAs; lane l holds token 32 i + l
      const float sw = row_ok ? __ldg(reinterpret_cast<const float*>(rec + geo.scale_offset(which)) + col) : 0.f;
      float xs_r[Geo::kChunks], tw_r[Geo::kChunks];
#pragma unroll
      for (int i = 0; i < Geo::kChunks; ++i) {
        const int tk = 32 * i + lane;
        const bool ok = tk < it.nvalid;
        xs_r[i] = ok ? __ldg(xsc + it.brow0 + tk) : 0.f;
        tw_r[i] = (MODE == 1 && ok) ? __ldg(tokw + it.brow0 + tk) : 0.f;
      }
      const int ab = ic % Geo::kAccBufs;
      const uint32_t aph = (ic / Geo::kAccBufs) & 1;
      if (!warp_wait(&acc_full[ab], aph, abort_flag, lane, t.wait_ns)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ab * Geo::kAccCols + ((uint32_t)(quad * 32) << 16);
      const int ld_out = MODE == 0 ? (it.shared ? t.g.Is : t.g.I) : t.g.H;
      float* out_base = it.shared ? t.out_s + (size_t)it.part * t.g.n * t.g.H : t.out_r;
      const int orow0 = (MODE == 0 && it.shared) ? it.tok0 : it.brow0;
      if constexpr (TT == 16) {
        // 16-token tiles run a few items per launch, so their epilogue code
        // mostly runs cold, fetched from memory (the first item's took ~20 us
        // unrolled): loops that are not unrolled, one TMEM column per load,
        // keep it short. Warps of half h take tokens 8h .. 8h + 7; gate warps
        // park their values in the exchange buffer's upper rows until the up
        // values arrive.
        const int b = chunk & 1;
        const uint32_t use_ph = (chunk >> 1) & 1;
        float* xb = xch + (xpb + b) * (16 * 32);
        if (MODE == 0 && up_warp && !warp_wait(&xempty[xpb + b], use_ph ^ 1, abort_flag, lane, t.wait_ns)) break;
#pragma unroll 1
        for (int j = 0; j < 8; ++j) {
          const int tk = half * 8 + j;
          const uint32_t v0 = tmem_ld1(tbase + tk), v1 = tmem_ld1(tbase + TT + tk);
          const float xs = __shfl_sync(0xffffffffu, xs_r[0], tk);
          const float tw = MODE == 1 ? __shfl_sync(0xffffffffu, tw_r[0], tk) : 0.f;
          tmem_ld_wait();
          const float val = fmaf((float)(int)v1, 1.f / 256.f, (float)(int)v0) * (xs * sw);
          if (MODE == 0)
            xb[(up_warp ? j : 8 + j) * 32 + lane] = val;
          else if (row_ok && tk < it.nvalid)
            out_base[(size_t)(orow0 + tk) * ld_out + col] = val * tw;
        }
        if (MODE == 0) {
          __syncwarp();
          if (up_warp) {
            if (lane == 0) mbar_arrive(&xfull[xpb + b]);
          } else {
            if (!warp_wait(&xfull[xpb + b], use_ph, abort_flag, lane, t.wait_ns)) break;
#pragma unroll 1
            for (int j = 0; j < 8; ++j) {
              const int tk = half * 8 + j;
              const float g = xb[(8 + j) * 32 + lane], u = xb[j * 32 + lane];
              if (row_ok && tk < it.nvalid)
                out_base[(size_t)(orow0 + tk) * ld_out + col] = __fdividef(g, 1.f + __expf(-g)) * u;  // silu(g) * u
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&xempty[xpb + b]);
          }
        }
        ++chunk;
      } else {
#pragma unroll 1
      for (int ci = 0; ci < Geo::kChunks; ++ci) {
        const int c0 = half * 16 + 32 * ci;  // tokens c0 .. c0 + 15: lanes half*16 .. +15 of xs_r[ci]
        if (c0 >= it.npad) break;
        uint32_t v0[16], v1[16];
        tmem_ld16(tbase + c0, v0);
        tmem_ld16(tbase + TT + c0, v1);
        float xsc_ci = xs_r[0], tw_ci = tw_r[0];  // register select, no local-memory indexing
#pragma unroll
        for (int i = 1; i < Geo::kChunks; ++i)
          if (ci == i) {
            xsc_ci = xs_r[i];
            tw_ci = tw_r[i];
          }
        float xs[16], tw[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          xs[j] = __shfl_sync(0xffffffffu, xsc_ci, half * 16 + j);
          tw[j] = MODE == 1 ? __shfl_sync(0xffffffffu, tw_ci, half * 16 + j) : 0.f;
        }
        tmem_ld_wait();
        float val[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) val[j] = fmaf((float)(int)v1[j], 1.f / 256.f, (float)(int)v0[j]) * (xs[j] * sw);
        if (MODE == 0) {
          // hand u from the up warp to the gate warp of the pair: double-buffered,
          // every wait bounded like the pipeline's
          const int b = chunk & 1;
          const uint32_t use_ph = (chunk >> 1) & 1;
          float* xb = xch + (xpb + b) * (16 * 32);
          if (up_warp) {
            if (!warp_wait(&xempty[xpb + b], use_ph ^ 1, abort_flag, lane, t.wait_ns)) {
              alive = false;
              break;
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) xb[j * 32 + lane] = val[j];
            __syncwarp();
            if (lane == 0) mbar_arrive(&xfull[xpb + b]);
          } else {
            if (!warp_wait(&xfull[xpb + b], use_ph, abort_flag, lane, t.wait_ns)) {
              alive = false;
              break;
            }
            float act[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float g = val[j], u = xb[j * 32 + lane];
              // SiLU(g) * u = g / (1 + e^-g) * u with the fast exponential and the
              // fast divide (2 ulp; a correctly rounded reciprocal here costs a
              // fifth of the kernel's time). g << 0 gives e^-g = inf and 0.
              act[j] = row_ok ? __fdividef(g, 1.f + __expf(-g)) * u : 0.f;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&xempty[xpb + b]);
            if (row_ok) {
              float* dst = out_base + (size_t)(orow0 + c0) * ld_out + col;
#pragma unroll
              for (int j = 0; j < 16; ++j)
                if (c0 + j < it.nvalid) dst[(size_t)j * ld_out] = act[j];
            }
          }
        } else if (row_ok) {
          float* dst = out_base + (size_t)(orow0 + c0) * ld_out + col;
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c0 + j < it.nvalid) dst[(size_t)j * ld_out] = val[j] * tw[j];
        }
        ++chunk;
      }
      }
      if (!alive) break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader)
          mbar_arrive(&acc_empty[ab]);
        else
          mbar_arrive_remote(mapa_shared(smem_u32(&acc_empty[ab]), 0));
      }
      ++ic;
    }
  }

  tc_fence_before();
  __syncthreads();
  // neither CTA of a pair leaves while the other may still arrive on its
  // barriers or (CTA 0's MMAs) use its shared memory and TMEM
  if constexpr (CG == 2) cluster_sync();
  tc_fence_after();
  if (*abort_flag && threadIdx.x == 0) atomicOr(&t.plan_rw->error, 8);
  if (warp == kTcMmaWarp) tmem_dealloc<CG>(tmem_base, kTcTmemCols);
}

// ---------------------------------------------------------------------------
// host side: tensor maps and launches
// ---------------------------------------------------------------------------

// clusters of 2 CTAs; chained to the kernel before (chain_wait) when `chained`
static void pair_launch_config(cudaLaunchConfig_t* cfg, cudaLaunchAttribute* attr, int pairs, size_t smem,
                               cudaStream_t st, bool chained) {
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  memset(cfg, 0, sizeof(*cfg));
  cfg->gridDim = dim3(2 * pairs);
  cfg->blockDim = dim3(kTcThreads);
  cfg->dynamicSmemBytes = smem;
  cfg->stream = st;
  cfg->attrs = attr;
  cfg->numAttrs = chained ? 2 : 1;
}

// Per device and kernel: the shared-memory attribute, and for pair kernels how
// many SM pairs can be resident at once (the persistent grid's size).
template <int MODE, int TT, int CG>
static int configure_tc(int* resident_pairs) {
  static int done_dev = -1, pairs = 0;
  int dev = 0;
  if (int rc = cuda_check(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (done_dev != dev) {
    using Geo = TcGeom<MODE, TT, CG>;
    if (int rc = cuda_check(cudaFuncSetAttribute(tc_expert_gemm_kernel<MODE, TT, CG>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Geo::kSmem),
                            "tc smem attribute"))
      return rc;
    pairs = 0;
    if (CG == 2) {
      int sms = 148;
      if (int rc = er_device_sm_count(&sms)) return rc;
      cudaLaunchConfig_t cfg;
      cudaLaunchAttribute attr[2];
      pair_launch_config(&cfg, attr, sms / 2, Geo::kSmem, 0, false);
      if (int rc = cuda_check(cudaOccupancyMaxActiveClusters(&pairs, tc_expert_gemm_kernel<MODE, TT, CG>, &cfg),
                              "cudaOccupancyMaxActiveClusters"))
        return rc;
      if (pairs < 1)
        return fail(ER_ECUDA, "no SM pair can hold the tensor-core kernel (%zu bytes of shared memory)", Geo::kSmem);
    }
    done_dev = dev;
  }
  if (resident_pairs) *resident_pairs = pairs;
  return ER_OK;
}

template <int MODE, int TT, int CG>
static int launch_tc_mode(const TcMaps& maps, const TcArgs& t, long long items_bound, cudaStream_t st) {
  int resident_pairs = 0;
  if (int rc = configure_tc<MODE, TT, CG>(&resident_pairs)) return rc;
  const long long items = items_bound > 0 ? items_bound : 1;
  if constexpr (CG == 1) {
    int sms = 148;
    if (int rc = er_device_sm_count(&sms)) return rc;
    const int grid = (int)(items < sms ? items : sms);
    if (int rc = launch_chained(tc_expert_gemm_kernel<MODE, TT, CG>, dim3(grid), dim3(kTcThreads),
                                TcGeom<MODE, TT, CG>::kSmem, st, "tc_expert_gemm_kernel", maps, t))
      return rc;
  } else {
    // persistent: one cluster per resident SM pair, items strided over the pairs
    const int pairs = (int)(items < resident_pairs ? items : resident_pairs);
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[2];
    pair_launch_config(&cfg, attr, pairs, TcGeom<MODE, TT, CG>::kSmem, st, true);
    if (int rc = cuda_check(cudaLaunchKernelEx(&cfg, tc_expert_gemm_kernel<MODE, TT, CG>, maps, t),
                            "cudaLaunchKernelEx(tc pair)"))
      return rc;
  }
  return launch_check("tc_expert_gemm_kernel");
}

// Rows longer than a warp holds (K > 2048): one CTA of 256 threads per row,
// each thread holding kVec float4 of it, so the row is read once; the CTA
// reduces the row maximum through shared memory.
template <typename XT, int kVec>
__device__ __forceinline__ void slice_row_cta(const XT* __restrict__ src, int row, int K, int8_t* __restrict__ s0,
                                              int8_t* __restrict__ s1, float* __restrict__ scale) {
  __shared__ float red[8];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const XT* x = src + (size_t)row * K;
  float4 v[kVec];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int k = (tid + 256 * i) * 4;
    v[i] = k < K ? load4(x + k) : make_float4(0.f, 0.f, 0.f, 0.f);
    amax = fmaxf(amax, abs_max4(v[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (lane == 0) red[warp] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) amax = fmaxf(amax, red[w]);
  const float inv = amax > 0.f ? 127.f / amax : 0.f;
  int8_t* d0 = s0 + (size_t)row * K;
  int8_t* d1 = s1 + (size_t)row * K;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int k = (tid + 256 * i) * 4;
    if (k < K) {
      uint32_t w0, w1;
      slice4(v[i], inv, w0, w1);
      *reinterpret_cast<uint32_t*>(d0 + k) = w0;
      *reinterpret_cast<uint32_t*>(d1 + k) = w1;
    }
  }
  if (tid == 0) scale[row] = amax / 127.f;
}

template <typename XT, int kVec>
__global__ void __launch_bounds__(256) slice_long_rows_kernel(const XT* __restrict__ src, int K,
                                                              int8_t* __restrict__ s0, int8_t* __restrict__ s1,
                                                              float* __restrict__ scale) {
  chain_wait();
  slice_row_cta<XT, kVec>(src, blockIdx.x, K, s0, s1, scale);
}

// Both row sets of the down step's operand (the routed act rows, K = I, and
// the shared expert's, K = Is) in one launch: CTAs [0, a_blocks) slice set a,
// the rest set b; each set one warp per row (K <= 2048) or one CTA per row.
__device__ __forceinline__ void slice_set(const SliceSet& s, int b) {
  if (s.K <= 2048) {
    const int row = b * 8 + (threadIdx.x >> 5);
    if (row < s.rows) slice_row_warp(s.src, row, s.K, s.s0, s.s1, s.scale, threadIdx.x & 31);
  } else {
    slice_row_cta<float, 8>(s.src, b, s.K, s.s0, s.s1, s.scale);
  }
}

__global__ void __launch_bounds__(256) slice_sets_kernel(SliceSet a, int a_blocks, SliceSet b) {
  chain_trigger();  // the down GEMM's CTAs may start their prologue as SMs free up
  chain_wait();
  if ((int)blockIdx.x < a_blocks)
    slice_set(a, blockIdx.x);
  else
    slice_set(b, blockIdx.x - a_blocks);
}

static int slice_set_blocks(const SliceSet& s) { return s.rows <= 0 ? 0 : (s.K <= 2048 ? (s.rows + 7) / 8 : s.rows); }

int launch_slice_sets(const SliceSet& a, const SliceSet& b, cudaStream_t st) {
  for (const SliceSet* s : {&a, &b})
    if (s->rows > 0 && (s->K <= 0 || s->K % 4 || s->K > 8192))
      return fail(ER_EINVAL, "slice: row length %d (a multiple of 4 up to 8192)", s->K);
  const int ab = slice_set_blocks(a), bb = slice_set_blocks(b);
  if (ab + bb == 0) return ER_OK;
  return launch_chained(slice_sets_kernel, dim3(ab + bb), dim3(256), 0, st, "slice_sets_kernel", a, ab, b);
}

int launch_slice_rows(const void* src, int dtype, int rows, int K, int8_t* s0, int8_t* s1, float* scale,
                      cudaStream_t st) {
  if (rows <= 0) return ER_OK;
  if (K > 2048 && K <= 8192) {  // 256 threads x 8 float4 cover 8192 values
    if (dtype == ER_DTYPE_BF16)
      return launch_chained(slice_long_rows_kernel<__nv_bfloat16, 8>, dim3(rows), dim3(256), 0, st,
                            "slice_long_rows_kernel", (const __nv_bfloat16*)src, K, s0, s1, scale);
    return launch_chained(slice_long_rows_kernel<float, 8>, dim3(rows), dim3(256), 0, st, "slice_long_rows_kernel",
                          (const float*)src, K, s0, s1, scale);
  }
  const int blocks = (rows + 7) / 8;
  if (dtype == ER_DTYPE_BF16)
    return launch_chained(slice_rows_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, st, "slice_rows_kernel",
                          (const __nv_bfloat16*)src, rows, K, s0, s1, scale);
  return launch_chained(slice_rows_kernel<float>, dim3(blocks), dim3(256), 0, st, "slice_rows_kernel",
                        (const float*)src, rows, K, s0, s1, scale);
}

int launch_tc_grouped(const TcLaunch& L, cudaStream_t st) {
  const GroupArgs& a = L.g;
  const int TT = L.tok_tile;
  if (TT != 16 && TT != 128) return fail(ER_EINVAL, "tensor-core token tile %d (16 or 128)", TT);
  TcMaps maps;
  memset(&maps, 0, sizeof(maps));
  const RecordGeom rg{ER_FMT_INT8, a.H, a.I, 1};
  const RecordGeom sg{ER_FMT_INT8, a.H, a.Is, 1};
  const uint8_t* arena = static_cast<const uint8_t*>(L.arena);
  if (L.nk == 0 && !L.has_shared) return ER_OK;  // no rows at all
  const uint8_t* shr = a.shared_record;
  if (L.mode == 0) {
    // 64 gate rows + the same 64 up rows per item
    if (L.nk > 0) {
      if (int rc = make_map(&maps.a_routed[0], arena + rg.weight_offset(0), 3, a.H, a.I, L.arena_slots, a.H,
                            L.record_bytes, 64, "gate"))
        return rc;
      if (int rc = make_map(&maps.a_routed[1], arena + rg.weight_offset(1), 3, a.H, a.I, L.arena_slots, a.H,
                            L.record_bytes, 64, "up"))
        return rc;
    }
    if (L.has_shared) {
      if (int rc = make_map(&maps.a_shared[0], shr + sg.weight_offset(0), 2, a.H, a.Is, 1, a.H, 0, 64, "shared gate"))
        return rc;
      if (int rc = make_map(&maps.a_shared[1], shr + sg.weight_offset(1), 2, a.H, a.Is, 1, a.H, 0, 64, "shared up"))
        return rc;
    }
    const int rows_b = L.nk + L.n;
    if (int rc = make_map(&maps.b_routed[0], L.b0_r, 2, a.H, rows_b, 1, a.H, 0, TT, "x slice 0")) return rc;
    if (int rc = make_map(&maps.b_routed[1], L.b1_r, 2, a.H, rows_b, 1, a.H, 0, TT, "x slice 1")) return rc;
  } else {
    if (L.nk > 0)
      if (int rc = make_map(&maps.a_routed[0], arena + rg.weight_offset(2), 3, a.I, a.H, L.arena_slots, a.I,
                            L.record_bytes, 128, "down"))
        return rc;
    if (L.has_shared)
      if (int rc = make_map(&maps.a_shared[0], shr + sg.weight_offset(2), 2, a.Is, a.H, 1, a.Is, 0, 128, "shared down"))
        return rc;
    if (L.nk > 0) {
      if (int rc = make_map(&maps.b_routed[0], L.b0_r, 2, a.I, L.nk, 1, a.I, 0, TT, "act slice 0")) return rc;
      if (int rc = make_map(&maps.b_routed[1], L.b1_r, 2, a.I, L.nk, 1, a.I, 0, TT, "act slice 1")) return rc;
    }
    if (L.has_shared) {
      if (int rc = make_map(&maps.b_shared[0], L.b0_s, 2, a.Is, L.n, 1, a.Is, 0, TT, "shared act slice 0")) return rc;
      if (int rc = make_map(&maps.b_shared[1], L.b1_s, 2, a.Is, L.n, 1, a.Is, 0, TT, "shared act slice 1")) return rc;
    }
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
  t.shared_parts = L.mode == 1 && L.shared_parts > 1 ? L.shared_parts : 1;
  t.plan_rw = const_cast<Plan*>(a.plan);
  t.wait_ns = L.wait_ns ? L.wait_ns : kDefaultWaitNs;
  t.stall_last = L.stall_last;
  t.pre_shared = TT == 16 && L.has_shared && L.n > 0 && a.shared_record != nullptr;
  t.maps_used = maps_used_bits(maps);
  // 16-token tiles on single SMs, 128-token tiles on SM pairs (tc_cta_group)
  if (L.mode == 0)
    return TT == 16 ? launch_tc_mode<0, 16, 1>(maps, t, L.items_bound, st)
                    : launch_tc_mode<0, 128, 2>(maps, t, L.items_bound, st);
  return TT == 16 ? launch_tc_mode<1, 16, 1>(maps, t, L.items_bound, st)
                  : launch_tc_mode<1, 128, 2>(maps, t, L.items_bound, st);
}

}  // namespace er
