// er_tcg.cu -- tensor-core (tcgen05) grouped expert GEMM for int4 records with
// group scales: the store's symmetric int4 (value = nibble - 8) and the
// asymmetric GPTQ extension (value = nibble - zero point), fp16 scales per
// (row, group of G inputs).
//
// Reference arithmetic: runtime/int4_linear.py:37-71 (the fused kernel sums
// each group's products, then multiplies the partial sum by that group's
// scale) and bench/gptq_conversion_check.py:42-55 (value = (q - z) * s).
// Here the same order holds exactly: per group, an exact int32 tcgen05 sum of
// the integer codes (q - z) times the two int8 activation slices, then the
// group's scale applied to that partial sum in fp32.
//
// Design (one CTA per SM, persistent over the work items):
//  * TMA stages each 128-input k-block of the packed nibbles (64 bytes per
//    weight row) into shared memory, beside the activation slices (B, as in
//    er_tc.cu: slice 0 then slice 1 of the item's tokens, 128-byte swizzled).
//  * Four transform warps unpack each staged row into signed int8 codes
//    (q - z) and write them in the 128-byte-swizzled K-major layout the MMA
//    reads (the layout TMA would have produced), then release the stage to
//    the MMA issuer. The shared expert's int8 rows are loaded by TMA straight
//    into that layout; for them the transform warps only pass the stage on.
//  * The MMA issuer runs one accumulation per group (kind::i8, M = 128 weight
//    rows, N = both slices of the item's tokens) into a ring of TMEM
//    accumulators, so group g + 1 accumulates while the epilogue drains g.
//    The shared expert's items are one group spanning their K range.
//  * Eight epilogue warps drain every group: acc += s[row, g] * (D0 + D1/256)
//    in fp32 registers; at the item's end the token's slice scale (and, for
//    down, its routing weight or the shared expert's sigmoid gate) is
//    applied; gate/up items hand the up rows to the gate rows' warps and
//    write silu(gate) * up.
//  * Every mbarrier wait is bounded (the launch's wait bound): on expiry the
//    CTA raises its abort flag and an error bit in the plan, drains the
//    copies it issued, frees its TMEM and returns.
//  TT = tokens per item: 16 (decode batches) or 64.
#include "er_tc.cuh"

namespace er {

// Warp roles: 0..3 transform (one per SM sub-partition), 4..11 epilogue
// (warp w reads TMEM lanes 32 * (w % 4) .. +31; two warps per lane quadrant,
// each every other 16-token chunk), 14 MMA issuer and 15 TMA producer; 12
// and 13 have no role. A warp runs on sub-partition w % 4: the MMA and TMA
// warps share sub-partitions 2 and 3 with the gate/up epilogue's up-row
// warps, which only hand values over, not with the gate rows' SiLU math.
constexpr int kGXfmWarps = 4;
constexpr int kGEpiWarp0 = 4;
constexpr int kGEpiWarps = 8;
constexpr int kGMmaWarp = 14;
constexpr int kGTmaWarp = 15;
constexpr int kGThreads = 16 * 32;
static_assert(kGEpiWarp0 + kGEpiWarps <= 12 && kGMmaWarp % 4 == 2 && kGTmaWarp % 4 == 3, "warp roles");
static_assert(kGThreads >= kMaxExperts + 2, "tc_cache_plan reads one plan entry per thread");

template <int MODE, int TT>
struct TcgGeom {
  static constexpr int kABytes = 16384;             // 128 weight rows x 128 int8 codes (MMA operand)
  static constexpr int kBSliceBytes = TT * 128;     // one activation slice of the item's tokens
  static constexpr int kBBytes = 2 * kBSliceBytes;  // slice 0, then slice 1
  static constexpr int kPackBytes = 128 * 64;       // 128 weight rows x 64 bytes of packed nibbles
  static constexpr int kStageBytes = kABytes + kBBytes + kPackBytes;
  static constexpr int kStages = (196608 / kStageBytes) < 8 ? (196608 / kStageBytes) : 8;
  static constexpr int kSlotCols = 2 * TT;          // TMEM columns per accumulator (both slices)
  static constexpr int kSlots = 512 / kSlotCols;
  static constexpr int kUnits = MODE == 0 ? 64 : 128;  // intermediate columns / hidden rows per item
  static constexpr int kChunks = (TT + 31) / 32;       // 16-token chunks per epilogue warp
  static constexpr size_t kXchBytes = MODE == 0 ? 4 * 2 * 16 * 32 * 4 : 0;
  static constexpr int kMaxGroups = 64;               // scale groups per weight row (K / G) the kernel takes
  static constexpr size_t kZeroBytes = 128 * kMaxGroups;  // one item's zero points, [row][group]
  // two item buffers of zero points (bulk-copied with the item's first stage)
  static constexpr size_t kSmem =
      1024 + (size_t)kStages * kStageBytes + 2 * kZeroBytes + kXchBytes + 2048 + sizeof(TcPlanCache);
  static_assert(kStageBytes % 1024 == 0, "stages must keep 1024-byte alignment (128-byte swizzle)");
  static_assert(kSlots >= 2, "at least two accumulators");
};

// 8 int4 codes of one packed word (element 2b in the low nibble of byte b) ->
// two words of 4 signed int8 values (q - z), first element in the lowest byte.
// zz = the zero point in every byte (z <= 128). Per byte, 0x80 + q - z stays
// within 0x70..0x8f, so the subtraction never borrows across bytes, and
// flipping bit 7 gives q - z in two's complement.
__device__ __forceinline__ void unpack8(uint32_t w, uint32_t zz, uint32_t& o0, uint32_t& o1) {
  const uint32_t lo = w & 0x0f0f0f0fu, hi = (w >> 4) & 0x0f0f0f0fu;
  o0 = ((__byte_perm(lo, hi, 0x5140) | 0x80808080u) - zz) ^ 0x80808080u;
  o1 = ((__byte_perm(lo, hi, 0x7362) | 0x80808080u) - zz) ^ 0x80808080u;
}


// The K range of an item and the length of its accumulation groups: routed
// (int4) items accumulate per scale group, shared-expert (int8) items over
// their whole range.
struct TcgSpan {
  int kbeg, kend, gk, ngroups;
};
template <int MODE>
__device__ __forceinline__ TcgSpan tcg_span(const TcArgs& t, const TcItem& it) {
  const int K = MODE == 0 ? t.g.H : (it.shared ? t.g.Is : t.g.I);
  TcgSpan s;
  s.kbeg = it.kb0 * 128;
  s.kend = min(K, (it.kb0 + it.nkb) * 128);
  s.gk = it.shared ? (s.kend - s.kbeg) : t.g.group;
  s.ngroups = s.kend > s.kbeg ? (s.kend - s.kbeg + s.gk - 1) / s.gk : 0;
  return s;
}

template <int MODE, int TT>
__global__ void __launch_bounds__(kGThreads, 1) tcg_expert_gemm_kernel(const __grid_constant__ TcMaps maps, TcArgs t) {
  using Geo = TcgGeom<MODE, TT>;
  constexpr int S = Geo::kStages;
  constexpr int NS = Geo::kSlots;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* zbuf = smem + (size_t)S * Geo::kStageBytes;  // [2][128 rows][groups]: zero points of an item
  uint8_t* tail = zbuf + 2 * Geo::kZeroBytes;
  float* xch = reinterpret_cast<float*>(tail);
  uint64_t* full = reinterpret_cast<uint64_t*>(tail + Geo::kXchBytes);
  uint64_t* ready = full + S;
  uint64_t* empty = ready + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + NS;
  uint64_t* drain_bar = acc_empty + NS;
  uint64_t* xfull = drain_bar + 1;  // [pair*2 + half][buffer]: up values written
  uint64_t* xempty = xfull + 8;     // [pair*2 + half][buffer]: up values consumed
  uint64_t* zempty = xempty + 8;    // [buffer]: the transform is done with the item's zero points
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(zempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  TcPlanCache* pc = reinterpret_cast<TcPlanCache*>(tail + Geo::kXchBytes + 2048);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], kGXfmWarps);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NS; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kGEpiWarps);
    }
    mbar_init(drain_bar, 1);
    for (int i = 0; i < 8; ++i) {
      mbar_init(&xfull[i], 1);
      mbar_init(&xempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) mbar_init(&zempty[i], kGXfmWarps);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kGTmaWarp && lane == 0) prefetch_maps(maps, t.maps_used);
  if constexpr (TT == 16) chain_trigger();  // decode tiles: the next kernel may launch and wait meanwhile
  const int first_item = blockIdx.x, item_stride = gridDim.x;
  // decode tiles: a CTA whose first item is one of the int8 shared expert's
  // (first in both schedules, laid out from the launch's sizes) loads that
  // item's first weight stages before waiting for the routing, as in
  // tc_expert_gemm_kernel; the producer adds the activation bytes and
  // arrives once the plan is read, and checks that the plan agrees
  int pre_n = 0, pre_kb0 = 0, pre_tok0 = 0;
  if constexpr (TT == 16) {
    __syncthreads();  // the barriers are initialised
    if (warp == kGTmaWarp && t.pre_shared && first_item < tc_shared_items<MODE, Geo::kUnits, TT>(t)) {
      TcItem p;
      tc_item_local<MODE, 128, Geo::kUnits, TT>(t, true, t.g.n, first_item, p);
      pre_n = min(p.nkb, S);
      pre_kb0 = p.kb0;
      pre_tok0 = p.tok0;
      if (lane == 0) {
        const uint64_t pol = l2_evict_first();
#pragma unroll 1
        for (int kb = 0; kb < pre_n; ++kb) {
          uint8_t* sa = smem + (size_t)kb * Geo::kStageBytes;
          const int x = (p.kb0 + kb) * 128;
          mbar_expect_tx_only(&full[kb], Geo::kABytes);
          tma_w2d<1>(sa, &maps.a_shared[0], &full[kb], 0u, x, p.unit0, pol);
          if (MODE == 0) tma_w2d<1>(sa + 8192, &maps.a_shared[1], &full[kb], 0u, x, p.unit0, pol);
        }
      }
      __syncwarp();
    }
  }
  chain_wait();
  tc_cache_plan(t, pc);
  if (warp == kGMmaWarp) tmem_alloc<1>(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total = pc->total;
  const unsigned long long wait_ns = t.wait_ns;

  if (warp == kGTmaWarp) {
    // ---------------- TMA producer ----------------
    const uint64_t wpol = TT == 16 ? l2_evict_first() : 0ull;  // decode: weights streamed once, evicted first
    uint32_t kc = 0, zi = 0;  // k-blocks issued; items with zero points issued
    bool ok = true;
    int skip = 0;  // k-blocks of the first item issued here, before the loop
    if (pre_n > 0) {
      // the plan must make the shared expert the first group with this CTA's
      // first item among its items (the geometry then follows from the
      // launch's sizes); if not (an inconsistent tally leaves no items),
      // report it, let the copies land (the arrivals complete the phases)
      // and stop
      const bool same = pc->num_active > 0 && pc->group[0] == t.g.E && first_item < pc->item_start[1] &&
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
        const int brow0 = (MODE == 0 ? pc->nk : 0) + pre_tok0;
        const CUtensorMap* b = MODE == 1 ? maps.b_shared : maps.b_routed;
        if (lane == 0) {
#pragma unroll 1
          for (int kb = 0; kb < pre_n; ++kb) {
            uint8_t* sb = smem + (size_t)kb * Geo::kStageBytes + Geo::kABytes;
            const int x = (pre_kb0 + kb) * 128;
            mbar_expect_tx(&full[kb], Geo::kBBytes);
            tma_load_2d(sb, &b[0], &full[kb], x, brow0);
            tma_load_2d(sb + Geo::kBSliceBytes, &b[1], &full[kb], x, brow0);
          }
        }
        __syncwarp();
        skip = pre_n;
        kc = pre_n;
      }
    }
    for (int item = first_item; ok && item < total; item += item_stride) {
      TcItem it;
      if (!tc_item_at<MODE, 128, Geo::kUnits, TT>(t, pc, item, it)) break;
      if (!it.valid) continue;
      // asymmetric records: the item's zero points ([rows][groups], contiguous
      // in the record) ride on its first stage into a buffer the transform
      // releases when it is done with the item
      const bool zp = !it.shared && t.g.fmt == ER_FMT_INT4_ZP;
      uint8_t* zdst = zbuf + (zi & 1) * Geo::kZeroBytes;
      if (zp && !warp_wait(&zempty[zi & 1], ((zi >> 1) & 1) ^ 1, abort_flag, lane, wait_ns)) break;
      for (int kb = item == first_item ? skip : 0; kb < it.nkb; ++kb, ++kc) {
        const int s = kc % S;
        const uint32_t ph = (kc / S) & 1;
        bool w = true;
        w = warp_wait(&empty[s], ph ^ 1, abort_flag, lane, wait_ns);
        if (!w) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t* st = smem + (size_t)s * Geo::kStageBytes;
          uint8_t* sa = st;
          uint8_t* sb = st + Geo::kABytes;
          uint8_t* sp = sb + Geo::kBBytes;
          const int x = (it.kb0 + kb) * 128;  // first K element of the block
          if (it.shared) {
            mbar_expect_tx(&full[s], Geo::kABytes + Geo::kBBytes);
            if (MODE == 0) {
              tma_w2d<1>(sa, &maps.a_shared[0], &full[s], 0u, x, it.unit0, wpol);
              tma_w2d<1>(sa + 8192, &maps.a_shared[1], &full[s], 0u, x, it.unit0, wpol);
            } else {
              tma_w2d<1>(sa, &maps.a_shared[0], &full[s], 0u, x, it.unit0, wpol);
            }
          } else {
            // packed nibbles: 64 bytes per row per k-block, x / 2 a multiple of 64
            const RecordGeom rg{t.g.fmt, t.g.H, t.g.I, t.g.group};
            const int gpr = rg.cols(MODE == 0 ? 0 : 2) / t.g.group;  // groups per row
            // rows of the item inside its matrix (multiples of 16: so are the copies)
            const int nr = MODE == 0 ? min(64, t.g.I - it.unit0) : min(128, t.g.H - it.unit0);
            const uint32_t zbytes = (zp && kb == 0) ? (MODE == 0 ? 2u : 1u) * (uint32_t)(nr * gpr) : 0u;
            mbar_expect_tx(&full[s], Geo::kPackBytes + Geo::kBBytes + zbytes);
            const uint8_t* rec = t.arena + (size_t)it.slot * t.record_bytes;
            if (MODE == 0) {
              tma_w3d<1>(sp, &maps.a_routed[0], &full[s], 0u, x / 2, it.unit0, it.slot, wpol);
              tma_w3d<1>(sp + 4096, &maps.a_routed[1], &full[s], 0u, x / 2, it.unit0, it.slot, wpol);
              if (zbytes) {  // gate rows' zero points to buffer rows 0..63, up rows' to 64..127
                bulk_load(zdst, rec + rg.zero_offset(0) + (size_t)it.unit0 * gpr, nr * gpr, &full[s]);
                bulk_load(zdst + 64 * gpr, rec + rg.zero_offset(1) + (size_t)it.unit0 * gpr, nr * gpr, &full[s]);
              }
            } else {
              tma_w3d<1>(sp, &maps.a_routed[0], &full[s], 0u, x / 2, it.unit0, it.slot, wpol);
              if (zbytes) bulk_load(zdst, rec + rg.zero_offset(2) + (size_t)it.unit0 * gpr, nr * gpr, &full[s]);
            }
          }
          const CUtensorMap* b = (MODE == 1 && it.shared) ? maps.b_shared : maps.b_routed;
          tma_load_2d(sb, &b[0], &full[s], x, it.brow0);
          tma_load_2d(sb + Geo::kBSliceBytes, &b[1], &full[s], x, it.brow0);
        }
        __syncwarp();
      }
      zi += zp ? 1 : 0;
    }
    if (!ok && lane == 0) {
      // aborted: every stage issued so far lands before the CTA exits
      for (int s = 0; s < S; ++s) {
        if (kc > (uint32_t)s) {
          const uint32_t last = kc - 1 - ((kc - 1 - s) % S);
          mbar_drain(&full[s], (last / S) & 1, 100000000ull);
        }
      }
    }
    __syncwarp();
  } else if (warp < kGXfmWarps) {
    // ---------------- transform: packed nibbles -> swizzled int8 codes ----------------
    // Thread t owns 16-byte chunk c = t % 4 (inputs 32c .. 32c + 31 of the
    // block) of rows r0 + 32 q, q = 0..3, r0 = t / 4: a warp reads 512
    // contiguous bytes per step and its swizzled stores fill every bank.
    const int tid = threadIdx.x;
    const int c = tid & 3, r0 = tid >> 2;
    uint32_t kc = 0, zi = 0;  // k-blocks consumed; items with zero points consumed
    bool ok = true;
    for (int item = first_item; ok && item < total; item += item_stride) {
      TcItem it;
      if (!tc_item_at<MODE, 128, Geo::kUnits, TT>(t, pc, item, it)) break;
      if (!it.valid) continue;
      const int kfull = MODE == 0 ? t.g.H : t.g.I;  // inputs per row of the routed matrix
      const int gpr = kfull / t.g.group;              // scale groups per row
      // asymmetric records: the item's zero points arrive with its first
      // stage in buffer zi % 2 (rows as in the A tile)
      const bool zp = !it.shared && t.g.fmt == ER_FMT_INT4_ZP;
      const uint8_t* zsrc = zbuf + (zi & 1) * Geo::kZeroBytes;
      for (int kb = 0; kb < it.nkb; ++kb, ++kc) {
        const int s = kc % S;
        const uint32_t ph = (kc / S) & 1;
        bool w = true;
        w = warp_wait(&full[s], ph, abort_flag, lane, wait_ns);
        if (!w) {
          ok = false;
          break;
        }
        const int grp = zp ? min(((it.kb0 + kb) * 128 + 32 * c) / t.g.group, gpr - 1) : 0;
        __syncwarp();
        if (!it.shared) {
          const uint32_t st = smem_u32(smem + (size_t)s * Geo::kStageBytes);
          const uint32_t sp = st + Geo::kABytes + Geo::kBBytes;
          // decode launches run this a few dozen times per CTA, mostly cold: one row per iteration
#pragma unroll(TT == 16 ? 1 : 4)
          for (int q = 0; q < 4; ++q) {
            const int r = r0 + 32 * q;
            const uint32_t zz = zp ? (uint32_t)zsrc[r * gpr + grp] * 0x01010101u : 0x08080808u;
            const uint4 p = lds128(sp + r * 64 + c * 16);
            uint32_t o[8];
            unpack8(p.x, zz, o[0], o[1]);
            unpack8(p.y, zz, o[2], o[3]);
            unpack8(p.z, zz, o[4], o[5]);
            unpack8(p.w, zz, o[6], o[7]);
            // 128-byte swizzle: 16-byte chunk j of row r sits at chunk j ^ (r % 8)
            const uint32_t row = st + r * 128;
            sts128(row + (((2 * c) ^ (r & 7)) << 4), o[0], o[1], o[2], o[3]);
            sts128(row + (((2 * c + 1) ^ (r & 7)) << 4), o[4], o[5], o[6], o[7]);
          }
          fence_async_smem();  // the codes are read by tcgen05.mma (async proxy)
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ready[s]);
      }
      if (!ok) break;
      if (zp) {  // this warp no longer reads the item's zero points
        if (lane == 0) mbar_arrive(&zempty[zi & 1]);
        ++zi;
      }
    }
  } else if (warp == kGMmaWarp) {
    // ---------------- MMA issuer (lane 0 issues) ----------------
    uint32_t kc = 0, gc = 0;
    bool ok = true;
    for (int item = first_item; ok && item < total; item += item_stride) {
      TcItem it;
      if (!tc_item_at<MODE, 128, Geo::kUnits, TT>(t, pc, item, it)) break;
      if (!it.valid) continue;
      const TcgSpan sp = tcg_span<MODE>(t, it);
      const uint32_t idesc = idesc_i8(128, TT + it.npad);
      int gpos = 0;      // K elements of the current group issued so far
      uint32_t d = 0;    // its accumulator
      int slot = 0;
      // The whole warp runs the loop in step (waits polled by lane 0 and
      // broadcast); only the MMAs and commits are issued by lane 0. A
      // lane-0-only loop body with waits inside it cost over a thousand
      // cycles per stage in branch and reconvergence overhead.
      for (int kb = 0; ok && kb < it.nkb; ++kb, ++kc) {
        const int s = kc % S;
        const uint32_t ph = (kc / S) & 1;
        if (!warp_wait(&ready[s], ph, abort_flag, lane, wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t st = smem_u32(smem + (size_t)s * Geo::kStageBytes);
        const uint32_t sa = st, sb = st + Geo::kABytes;
        const int k0 = (it.kb0 + kb) * 128;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const int k = k0 + ks * 32;
          if (k < sp.kend) {
            if (gpos == 0) {
              slot = (int)(gc % NS);
              if (!warp_wait(&acc_empty[slot], ((gc / NS) & 1) ^ 1, abort_flag, lane, wait_ns)) {
                ok = false;
                break;
              }
              tc_fence_after();
              d = tmem_base + slot * Geo::kSlotCols;
            }
            if (lane == 0)
              mma_i8<1>(d, umma_desc_sw128(sa + ks * 32), umma_desc_sw128(sb + ks * 32), idesc, gpos > 0 ? 1u : 0u);
            gpos += 32;
            if (gpos == sp.gk || k + 32 >= sp.kend) {
              if (lane == 0) umma_commit<1>(&acc_full[slot]);  // this group's partial sums are ready
              ++gc;
              gpos = 0;
            }
          }
        }
        if (lane == 0) umma_commit<1>(&empty[s]);  // the stage is free once these MMAs have read it
        __syncwarp();
      }
    }
    if (lane == 0) {
      // every MMA issued by this thread has finished before TMEM is released
      umma_commit<1>(drain_bar);
      mbar_drain(drain_bar, 0, 100000000ull);
    }
    __syncwarp();
  } else if (warp >= kGEpiWarp0 && warp < kGEpiWarp0 + kGEpiWarps) {
    // ---------------- epilogue ----------------
    // Warp w reads TMEM lanes 32 (w % 4) .. +31 and every other 16-token
    // chunk (half). Mode 0: lanes 0..63 hold gate rows, 64..127 the up rows
    // of the same columns; each up warp hands its finished values to the gate
    // warp of the same columns and half through shared memory.
    const int quad = warp & 3;
    const int half = (warp - kGEpiWarp0) >> 2;
    const int pair = quad & 1;
    const bool up_warp = MODE == 0 && quad >= 2;
    const int xpb = (pair * 2 + half) * 2;
    uint32_t gc = 0, chunk = 0;
    bool alive = true;
    for (int item = first_item; alive && item < total; item += item_stride) {
      TcItem it;
      if (!tc_item_at<MODE, 128, Geo::kUnits, TT>(t, pc, item, it)) break;
      if (!it.valid) {
        if (threadIdx.x == kGEpiWarp0 * 32) atomicOr(&t.plan_rw->error, 4);
        continue;
      }
      const TcgSpan sp = tcg_span<MODE>(t, it);
      const int col = it.unit0 + (MODE == 0 ? pair * 32 + lane : quad * 32 + lane);
      const bool row_ok = col < it.units;
      const int which = MODE == 0 ? (up_warp ? 1 : 0) : 2;
      // per-group scale of this thread's weight row
      const uint8_t* rec = it.shared ? t.g.shared_record : t.arena + (size_t)it.slot * t.record_bytes;
      const __half* sg_row = nullptr;
      float s_row = 0.f;
      if (it.shared) {
        const RecordGeom sgeo{ER_FMT_INT8, t.g.H, t.g.Is, 1};
        s_row = row_ok ? __ldg(reinterpret_cast<const float*>(rec + sgeo.scale_offset(which)) + col) : 0.f;
      } else if (row_ok) {
        const RecordGeom rg{t.g.fmt, t.g.H, t.g.I, t.g.group};
        const int gpr = rg.cols(which) / t.g.group;
        sg_row = reinterpret_cast<const __half*>(rec + rg.scale_offset(which)) + (size_t)col * gpr + sp.kbeg / t.g.group;
      }
      auto group_scale = [&](int g) -> float {
        if (it.shared) return s_row;
        return sg_row ? __half2float(sg_row[g]) : 0.f;
      };
      // token slice scales and (down) routing weights: lane l holds token 32 i + l
      const float* xsc = (MODE == 1 && it.shared) ? t.xscale_s : t.xscale_r;
      const float* tokw = it.shared ? t.g.gate_sig : t.g.perm_w;
      float xs_r[Geo::kChunks], tw_r[Geo::kChunks];
#pragma unroll
      for (int i = 0; i < Geo::kChunks; ++i) {
        const int tk = 32 * i + lane;
        const bool ok = tk < it.nvalid;
        xs_r[i] = ok ? __ldg(xsc + it.brow0 + tk) : 0.f;
        tw_r[i] = (MODE == 1 && ok) ? __ldg(tokw + it.brow0 + tk) : 0.f;
      }
      if constexpr (TT == 16) {
        // 16-token tiles: warps of half h take tokens 8h .. 8h + 7, and the
        // code is kept short (loops not unrolled where their bodies are
        // long): a decode launch runs it once or twice per CTA, cold.
        const int tk0 = half * 8;
        float acc8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc8[j] = 0.f;
        constexpr int kGB = 16;
#pragma unroll 1
        for (int g0 = 0; alive && g0 < sp.ngroups; g0 += kGB) {
          float sc[kGB];
#pragma unroll
          for (int i = 0; i < kGB; ++i) sc[i] = g0 + i < sp.ngroups ? group_scale(g0 + i) : 0.f;
#pragma unroll 1
          for (int i = 0; i < kGB && g0 + i < sp.ngroups; ++i) {
            float s_i = sc[0];  // register select, no local-memory indexing
#pragma unroll
            for (int q = 1; q < kGB; ++q)
              if (i == q) s_i = sc[q];
            const int slot = (int)(gc % NS);
            if (!warp_wait(&acc_full[slot], (gc / NS) & 1, abort_flag, lane, wait_ns)) {
              alive = false;
              break;
            }
            tc_fence_after();
            const uint32_t tb = tmem_base + slot * Geo::kSlotCols + ((uint32_t)(quad * 32) << 16);
            uint32_t v0[8], v1[8];
            tmem_ld8(tb + tk0, v0);
            tmem_ld8(tb + TT + tk0, v1);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 8; ++j)
              acc8[j] = fmaf(s_i, fmaf((float)(int)v1[j], 1.f / 256.f, (float)(int)v0[j]), acc8[j]);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[slot]);
            ++gc;
          }
        }
        if (!alive) break;
        const int ld_out = MODE == 0 ? (it.shared ? t.g.Is : t.g.I) : t.g.H;
        float* out_base = it.shared ? t.out_s + (size_t)it.part * t.g.n * t.g.H : t.out_r;
        const int orow0 = (MODE == 0 && it.shared) ? it.tok0 : it.brow0;
        float val[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float xs = __shfl_sync(0xffffffffu, xs_r[0], tk0 + j);
          const float tw = MODE == 1 ? __shfl_sync(0xffffffffu, tw_r[0], tk0 + j) : 1.f;
          val[j] = acc8[j] * xs * tw;
        }
        if (MODE == 0) {
          const int b = chunk & 1;
          const uint32_t use_ph = (chunk >> 1) & 1;
          float* xb = xch + (xpb + b) * (16 * 32);
          if (up_warp) {
            if (!warp_wait(&xempty[xpb + b], use_ph ^ 1, abort_flag, lane, wait_ns)) break;
#pragma unroll
            for (int j = 0; j < 8; ++j) xb[j * 32 + lane] = val[j];
            __syncwarp();
            if (lane == 0) mbar_arrive(&xfull[xpb + b]);
          } else {
            if (!warp_wait(&xfull[xpb + b], use_ph, abort_flag, lane, wait_ns)) break;
#pragma unroll 1
            for (int j = 0; j < 8; ++j) {
              float gv = val[0];
#pragma unroll
              for (int q = 1; q < 8; ++q)
                if (j == q) gv = val[q];
              const float u = xb[j * 32 + lane];
              if (row_ok && tk0 + j < it.nvalid)
                out_base[(size_t)(orow0 + tk0 + j) * ld_out + col] = __fdividef(gv, 1.f + __expf(-gv)) * u;  // silu(g) * u
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&xempty[xpb + b]);
          }
        } else if (row_ok) {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (tk0 + j < it.nvalid) out_base[(size_t)(orow0 + tk0 + j) * ld_out + col] = val[j];
        }
        ++chunk;
        continue;
      }
      float acc[Geo::kChunks][16];
#pragma unroll
      for (int i = 0; i < Geo::kChunks; ++i)
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[i][j] = 0.f;
      // group scales in batches of kGB, all of a batch fetched before its
      // first accumulator wait (one latency per batch, not per group)
      constexpr int kGB = 16;
#pragma unroll 1
      for (int g0 = 0; alive && g0 < sp.ngroups; g0 += kGB) {
        float sc[kGB];
#pragma unroll
        for (int i = 0; i < kGB; ++i) sc[i] = g0 + i < sp.ngroups ? group_scale(g0 + i) : 0.f;
#pragma unroll
        for (int i = 0; i < kGB; ++i) {
          if (g0 + i >= sp.ngroups) break;
          const int slot = (int)(gc % NS);
          if (!warp_wait(&acc_full[slot], (gc / NS) & 1, abort_flag, lane, wait_ns)) {
            alive = false;
            break;
          }
          tc_fence_after();
          const uint32_t tb = tmem_base + slot * Geo::kSlotCols + ((uint32_t)(quad * 32) << 16);
#pragma unroll
          for (int ci = 0; ci < Geo::kChunks; ++ci) {
            const int c0 = half * 16 + 32 * ci;
            if (c0 < it.npad) {  // the same for the whole warp
              uint32_t v0[16], v1[16];
              tmem_ld16(tb + c0, v0);
              tmem_ld16(tb + TT + c0, v1);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 16; ++j)
                acc[ci][j] = fmaf(sc[i], fmaf((float)(int)v1[j], 1.f / 256.f, (float)(int)v0[j]), acc[ci][j]);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[slot]);
          ++gc;
        }
      }
      if (!alive) break;
      const int ld_out = MODE == 0 ? (it.shared ? t.g.Is : t.g.I) : t.g.H;
      float* out_base = it.shared ? t.out_s + (size_t)it.part * t.g.n * t.g.H : t.out_r;
      const int orow0 = (MODE == 0 && it.shared) ? it.tok0 : it.brow0;
#pragma unroll
      for (int ci = 0; ci < Geo::kChunks; ++ci) {
        const int c0 = half * 16 + 32 * ci;
        if (c0 >= it.npad) continue;
        float val[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float xs = __shfl_sync(0xffffffffu, xs_r[ci], half * 16 + j);
          const float tw = MODE == 1 ? __shfl_sync(0xffffffffu, tw_r[ci], half * 16 + j) : 1.f;
          val[j] = acc[ci][j] * xs * tw;
        }
        if (MODE == 0) {
          const int b = chunk & 1;
          const uint32_t use_ph = (chunk >> 1) & 1;
          float* xb = xch + (xpb + b) * (16 * 32);
          if (up_warp) {
            if (!warp_wait(&xempty[xpb + b], use_ph ^ 1, abort_flag, lane, wait_ns)) {
              alive = false;
              break;
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) xb[j * 32 + lane] = val[j];
            __syncwarp();
            if (lane == 0) mbar_arrive(&xfull[xpb + b]);
          } else {
            if (!warp_wait(&xfull[xpb + b], use_ph, abort_flag, lane, wait_ns)) {
              alive = false;
              break;
            }
            float act[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float gv = val[j], u = xb[j * 32 + lane];
              act[j] = row_ok ? __fdividef(gv, 1.f + __expf(-gv)) * u : 0.f;  // silu(g) * u
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
            if (c0 + j < it.nvalid) dst[(size_t)j * ld_out] = val[j];
        }
        ++chunk;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (*abort_flag && threadIdx.x == 0) atomicOr(&t.plan_rw->error, 8);
  if (warp == kGMmaWarp) tmem_dealloc<1>(tmem_base, 512);
}

template <int MODE, int TT>
static int launch_tcg_mode(const TcMaps& maps, const TcArgs& t, long long items_bound, cudaStream_t st) {
  using Geo = TcgGeom<MODE, TT>;
  static int done_dev = -1;
  int dev = 0;
  if (int rc = cuda_check(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (done_dev != dev) {
    if (int rc = cuda_check(cudaFuncSetAttribute(tcg_expert_gemm_kernel<MODE, TT>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Geo::kSmem),
                            "tcg smem attribute"))
      return rc;
    done_dev = dev;
  }
  int sms = 148;
  if (int rc = er_device_sm_count(&sms)) return rc;
  const long long items = items_bound > 0 ? items_bound : 1;
  const int grid = (int)(items < sms ? items : sms);
  if (int rc = launch_chained(tcg_expert_gemm_kernel<MODE, TT>, dim3(grid), dim3(kGThreads), Geo::kSmem, st,
                              "tcg_expert_gemm_kernel", maps, t))
    return rc;
  return launch_check("tcg_expert_gemm_kernel");
}

int launch_tcg_grouped(const TcLaunch& L, cudaStream_t st) {
  const GroupArgs& a = L.g;
  const int TT = L.tok_tile;
  if (TT != 16 && TT != 64) return fail(ER_EINVAL, "int4 tensor-core token tile %d (16 or 64)", TT);
  if (L.fmt != ER_FMT_INT4 && L.fmt != ER_FMT_INT4_ZP) return fail(ER_EINVAL, "int4 tensor-core path: format %d", L.fmt);
  if (L.group <= 0 || L.group % 32 || a.H % L.group || a.I % L.group)
    return fail(ER_EINVAL, "int4 tensor-core path: group %d must be a multiple of 32 dividing %d and %d", L.group, a.H,
                a.I);
  if (a.H / L.group > TcgGeom<0, 16>::kMaxGroups || a.I / L.group > TcgGeom<0, 16>::kMaxGroups)
    return fail(ER_EINVAL, "int4 tensor-core path: more than %d groups per row", TcgGeom<0, 16>::kMaxGroups);
  if (a.H % 128 || a.I % 32 || a.Is % 128)
    return fail(ER_EINVAL, "int4 tensor-core path: hidden %d (x128), inter %d (x32), shared inter %d (x128)", a.H, a.I,
                a.Is);
  if (L.nk == 0 && !L.has_shared) return ER_OK;
  if (L.mode == 1 && L.has_shared && L.shared_parts > 1) {
    // the shared expert's down tiles split in K parts of 128-input blocks: none may be empty
    const int blocks = (a.Is + 127) / 128, span = (blocks + L.shared_parts - 1) / L.shared_parts;
    if ((L.shared_parts - 1) * span >= blocks)
      return fail(ER_EINVAL, "int4 tensor-core path: %d shared-expert parts of %d k-blocks", L.shared_parts, blocks);
  }
  TcMaps maps;
  memset(&maps, 0, sizeof(maps));
  const RecordGeom rg{L.fmt, a.H, a.I, L.group};
  const RecordGeom sg{ER_FMT_INT8, a.H, a.Is, 1};
  const uint8_t* arena = static_cast<const uint8_t*>(L.arena);
  const uint8_t* shr = a.shared_record;
  if (L.mode == 0) {
    if (L.nk > 0) {  // packed gate / up rows: 64 rows x 64 bytes per box, unswizzled (the transform reads them)
      if (int rc = make_map(&maps.a_routed[0], arena + rg.weight_offset(0), 3, a.H / 2, a.I, L.arena_slots, a.H / 2,
                            L.record_bytes, 64, "int4 gate", 64, false))
        return rc;
      if (int rc = make_map(&maps.a_routed[1], arena + rg.weight_offset(1), 3, a.H / 2, a.I, L.arena_slots, a.H / 2,
                            L.record_bytes, 64, "int4 up", 64, false))
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
    if (L.nk > 0) {
      if (int rc = make_map(&maps.a_routed[0], arena + rg.weight_offset(2), 3, a.I / 2, a.H, L.arena_slots, a.I / 2,
                            L.record_bytes, 128, "int4 down", 64, false))
        return rc;
      if (int rc = make_map(&maps.b_routed[0], L.b0_r, 2, a.I, L.nk, 1, a.I, 0, TT, "act slice 0")) return rc;
      if (int rc = make_map(&maps.b_routed[1], L.b1_r, 2, a.I, L.nk, 1, a.I, 0, TT, "act slice 1")) return rc;
    }
    if (L.has_shared) {
      if (int rc = make_map(&maps.a_shared[0], shr + sg.weight_offset(2), 2, a.Is, a.H, 1, a.Is, 0, 128, "shared down"))
        return rc;
      if (int rc = make_map(&maps.b_shared[0], L.b0_s, 2, a.Is, L.n, 1, a.Is, 0, TT, "shared act slice 0")) return rc;
      if (int rc = make_map(&maps.b_shared[1], L.b1_s, 2, a.Is, L.n, 1, a.Is, 0, TT, "shared act slice 1")) return rc;
    }
  }
  TcArgs t;
  memset(&t, 0, sizeof(t));
  t.g = a;
  t.g.fmt = L.fmt;
  t.g.group = L.group;
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
  t.stall_last = 0;
  t.pre_shared = TT == 16 && L.has_shared && L.n > 0 && a.shared_record != nullptr;
  t.maps_used = maps_used_bits(maps);
  if (L.mode == 0)
    return TT == 16 ? launch_tcg_mode<0, 16>(maps, t, L.items_bound, st) : launch_tcg_mode<0, 64>(maps, t, L.items_bound, st);
  return TT == 16 ? launch_tcg_mode<1, 16>(maps, t, L.items_bound, st) : launch_tcg_mode<1, 64>(maps, t, L.items_bound, st);
}

}  // namespace er
