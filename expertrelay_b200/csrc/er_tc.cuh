// er_tc.cuh -- pieces shared by the tcgen05 grouped expert GEMMs (er_tc.cu:
// int8 records; er_tcg.cu: group-scaled int4 records): PTX wrappers for
// mbarriers, TMA, tcgen05 MMA / TMEM, the launch arguments, the work-item
// lookup over the routing plan, and tensor-map encoding.
#pragma once

#include <cuda.h>
#include <string.h>

#include "er_internal.cuh"

namespace er {

constexpr unsigned long long kDefaultWaitNs = 2000000000ull;  // 2 s: bound of every mbarrier wait

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
// raise the phase's expected transaction bytes without arriving
__device__ __forceinline__ void mbar_expect_tx_only(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
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
// try_wait with a suspend hint: the thread sleeps until the phase completes
// (it is woken then) or hint_ns pass, instead of spinning on the barrier and
// taking issue slots from the warps that do the work.
__device__ __forceinline__ bool mbar_test_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// The waiting part of mbar_wait, out of line: inlined, its loop made every
// call cost over a hundred cycles more even when the phase had already
// completed (measured), and the pipelines make several such calls per stage.
static __device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                            unsigned long long limit_ns) {
  const unsigned long long t0 = globaltimer();
  const uint32_t hint = (uint32_t)(limit_ns / 16 < 100000ull ? limit_ns / 16 + 1 : 100000ull);
  for (;;) {
    if (mbar_test_sleep(bar, parity, hint)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > limit_ns) {
      *abort_flag = 1;
      return false;
    }
  }
}
// Bounded wait for the phase with `parity` to complete. Returns false (and
// raises the CTA's abort flag) after limit_ns, or as soon as it sees that
// another role already aborted (within one suspend hint, <= 100 us).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned long long limit_ns) {
  if (mbar_test(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, abort_flag, limit_ns);
}
// The whole warp waits (every lane tests the barrier, so the warp's control
// flow stays uniform: a lane-0 wait inside a divergent branch cost several
// times more per call), then agrees on lane 0's outcome; the warp syncs so
// every lane's later accesses are ordered after the acquire.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int lane,
                                          unsigned long long limit_ns) {
  (void)lane;
  bool w = mbar_wait(bar, parity, abort_flag, limit_ns);
  w = __shfl_sync(0xffffffffu, (int)w, 0) != 0;
  __syncwarp();
  return w;
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
// Untiled bulk copy of `bytes` from global memory into this CTA's shared
// memory, completing on `bar` (src, dst and bytes multiples of 16). A plain
// load of this GPU's memory; no multicast.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// Pair forms: the tile lands in this CTA's shared memory and completes on the
// barrier at shared::cluster address `bar` (CTA 0's full barrier). Plain
// loads of this GPU's memory; no multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int x, int y,
                                                 int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}
// L2 policy for streamed weights (decode): evicted first, so the small
// kernels' code and data stay in L2 across the weight stream
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void tma_load_2d_ef(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                               uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, %4}], "
      "[%2], %5;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d_ef(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                               uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, %4, "
      "%5}], [%2], %6;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "l"(pol)
      : "memory");
}
// weight tiles: with the evict-first policy on single SMs when `pol` is nonzero
template <int CG>
__device__ __forceinline__ void tma_w2d(void* dst, const CUtensorMap* map, uint64_t* bar, uint32_t bar_c, int x, int y,
                                        uint64_t pol) {
  if constexpr (CG == 1) {
    if (pol)
      tma_load_2d_ef(dst, map, bar, x, y, pol);
    else
      tma_load_2d(dst, map, bar, x, y);
  } else {
    tma_load_2d_pair(dst, map, bar_c, x, y);
  }
}
template <int CG>
__device__ __forceinline__ void tma_w3d(void* dst, const CUtensorMap* map, uint64_t* bar, uint32_t bar_c, int x, int y,
                                        int z, uint64_t pol) {
  if constexpr (CG == 1) {
    if (pol)
      tma_load_3d_ef(dst, map, bar, x, y, z, pol);
    else
      tma_load_3d(dst, map, bar, x, y, z);
  } else {
    tma_load_3d_pair(dst, map, bar_c, x, y, z);
  }
}
template <int CG>
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, uint64_t* bar, uint32_t bar_c, int x, int y) {
  if constexpr (CG == 1)
    tma_load_2d(dst, map, bar, x, y);
  else
    tma_load_2d_pair(dst, map, bar_c, x, y);
}
template <int CG>
__device__ __forceinline__ void tma_3d(void* dst, const CUtensorMap* map, uint64_t* bar, uint32_t bar_c, int x, int y,
                                       int z) {
  if constexpr (CG == 1)
    tma_load_3d(dst, map, bar, x, y, z);
  else
    tma_load_3d_pair(dst, map, bar_c, x, y, z);
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

template <int CG>
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  if constexpr (CG == 1)
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// Arrive on `bar` once every MMA issued so far by this thread has completed.
// Pair kernels arrive on the barrier at the same offset in both CTAs.
template <int CG>
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  if constexpr (CG == 1)
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
  else
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"((uint16_t)3)
        : "memory");
}
template <int CG>
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
  if constexpr (CG == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  } else {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
}
template <int CG>
__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t cols) {
  if constexpr (CG == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols));
  else
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols));
}

// ---- clusters (SM pairs)
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// shared::cluster address of the variable at shared::cta address `a` in CTA `rank`
__device__ __forceinline__ uint32_t mapa_shared(uint32_t a, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
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
// Eight consecutive TMEM columns per lane.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
// One TMEM column (32-bit) per lane.
__device__ __forceinline__ uint32_t tmem_ld1(uint32_t taddr) {
  uint32_t r;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
  return r;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}
// Orders this thread's earlier generic-proxy shared-memory writes before later
// async-proxy reads of them (operands written by threads, read by tcgen05.mma).
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------
// launch arguments and the work-item lookup
// ---------------------------------------------------------------------------

struct TcMaps {
  CUtensorMap a_routed[2];  // mode 0: gate, up (64-row boxes) over the arena; mode 1: down in [0]
  CUtensorMap a_shared[2];  // the same for the shared-expert record (2-D)
  CUtensorMap b_routed[2];  // activation slices 0 / 1 of the routed rows (mode 0: all nk + n rows)
  CUtensorMap b_shared[2];  // mode 1: activation slices of the shared rows
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
  float* out_s;              // mode 0: act shared [n, Is]; mode 1: shared_parts partial y shared [n, H]
  int shared_parts;          // mode 1: K parts of each shared-expert tile (1: no split)
  Plan* plan_rw;             // error bits
  unsigned long long wait_ns;  // bound of every mbarrier wait (kDefaultWaitNs unless a test shortens it)
  uint32_t maps_used;        // bit i: map i of TcMaps (a_routed 0-1, a_shared 2-3, b_routed 4-5, b_shared 6-7)
                             // is encoded (prefetched at the kernel's start)
  int pre_shared;            // 16-token tiles: the shared expert runs in this launch (its items come first), so
                             // CTAs whose first item is one of its load that item's first weight stages
                             // before waiting for the kernels before them
  int stall_last;            // test hook: nonzero -> the MMA issuer never completes the accumulator of the
                             // launch's last item, so its epilogue wait runs out (that item is its CTA's
                             // last: no copy is in flight when the wait gives up)
};

// The plan's schedule, copied into shared memory once per CTA so that the
// per-item lookups of every role (a binary search over the item prefix,
// then the group's rows and record) cost no global-memory round trips.
// Entries are indexed by active position a, not by group id.
struct TcPlanCache {
  int total;       // work items of this schedule
  int num_active;  // active groups (the shared expert, then the routed experts)
  int nk;
  int item_start[kMaxExperts + 2];
  int group[kMaxExperts + 1];   // group id (E = shared expert)
  int rows[kMaxExperts + 1];    // tokens of the group
  int offset[kMaxExperts + 1];  // first expert-sorted position (routed groups)
  int slot[kMaxExperts + 1];    // arena slot of the group's record; -1 outside the arena
};

struct TcItem {
  int g, shared, valid;
  int unit0;   // first unit of the tile (mode 0: intermediate column; mode 1: hidden row)
  int tok0;    // first token of the tile within the group
  int nvalid;  // tokens in the tile
  int npad;    // tokens rounded up to 16
  int brow0;   // first B row in the operand matrix
  int slot;    // arena slot of the routed record
  int units;
  int kb0, nkb;  // the item's k-blocks: [kb0, kb0 + nkb)
  int part;      // mode 1 shared items: which K part (partial output) the item computes
};

// Copies the schedule `t.sched` of the plan into `pc` (every thread takes
// part; at least kMaxExperts + 2 threads; a __syncthreads must follow before
// any lookup). One round of loads: every entry that can be active is read
// together with num_active (the dispatch wrote each active group's rows,
// range and record by active position; entries past num_active are read and
// dropped). Group ids are clamped to 0..E. L2: loads that bypass L1 (for a
// kernel that reads the plan before its griddepcontrol.wait).
template <bool L2 = false>
__device__ __forceinline__ void tc_cache_plan(const TcArgs& t, TcPlanCache* pc) {
  const Plan* P = t.g.plan;
  const int E = t.g.E;
  const int a = threadIdx.x;
  auto ld = [](const int* q) { return L2 ? __ldcg(q) : *q; };
  const int na_raw = ld(&P->num_active);
  const int nk = ld(&P->nk);
  const int start = a < kMaxExperts + 2 ? ld(&P->item_start[t.sched][a]) : 0;
  const bool in_list = a < kMaxExperts + 1;
  const int g_raw = in_list ? ld(&P->active[a]) : E;
  const int rows_raw = in_list ? ld(&P->act_rows[a]) : 0;
  const int off_raw = in_list ? ld(&P->act_off[a]) : 0;
  const uint64_t addr = in_list ? (L2 ? __ldcg(&P->act_rec[a]) : P->act_rec[a]) : 0ull;
  const int na = min(na_raw, kMaxExperts + 1);
  const int g = g_raw < 0 ? 0 : (g_raw > E ? E : g_raw);
  const bool shared = g == E;
  const bool live = a < na;
  if (a <= na) pc->item_start[a] = start;
  if (a == na) pc->total = start;
  if (live) {
    pc->group[a] = g;
    pc->rows[a] = rows_raw;
    pc->offset[a] = shared ? 0 : off_raw;
    int slot = 0;
    if (!shared) {
      const uint64_t base = (uint64_t)t.arena;
      slot = -1;  // record outside the arena: reported, never loaded
      if (addr >= base && (addr - base) % t.record_bytes == 0 && (addr - base) / t.record_bytes < (uint64_t)t.arena_slots)
        slot = (int)((addr - base) / t.record_bytes);
    }
    pc->slot[a] = slot;
  }
  if (a == 0) {
    pc->num_active = na;
    pc->nk = nk;
  }
}

// Item `local` of a group with `rows` tokens (shared: the shared expert):
// its token tile and output-unit tile, and its k-blocks of KBLK K elements
// (the shared expert's down tiles in `t.shared_parts` K parts). Depends on
// the launch's sizes only, not on the plan.
template <int MODE, int KBLK, int UNITS, int TT>
__device__ __forceinline__ void tc_item_local(const TcArgs& t, bool shared, int rows, int local, TcItem& it) {
  it.shared = shared;
  const int inter = it.shared ? t.g.Is : t.g.I;
  it.units = MODE == 0 ? inter : t.g.H;
  const int K = MODE == 0 ? t.g.H : inter;
  const int blocks = (K + KBLK - 1) / KBLK;
  const int ntiles = (it.units + UNITS - 1) / UNITS;
  int tile = local;
  it.kb0 = 0;
  it.nkb = blocks;
  it.part = 0;
  if (MODE == 1 && it.shared && t.shared_parts > 1) {
    // the K parts of one tile are adjacent items (different CTAs); part p
    // covers k-blocks [p span, min(blocks, (p + 1) span)), none empty
    const int span = (blocks + t.shared_parts - 1) / t.shared_parts;
    tile = local / t.shared_parts;
    it.part = local % t.shared_parts;
    it.kb0 = it.part * span;
    it.nkb = min(blocks - it.kb0, span);
  }
  it.tok0 = (tile / ntiles) * TT;
  it.unit0 = (tile % ntiles) * UNITS;
  it.nvalid = min(TT, rows - it.tok0);
  it.npad = (it.nvalid + 15) & ~15;
}

// Work items of the shared expert (the first group of every schedule when it
// runs), from the launch's sizes; the same count as the plan's scan.
template <int MODE, int UNITS, int TT>
__device__ __forceinline__ int tc_shared_items(const TcArgs& t) {
  const int units = MODE == 0 ? t.g.Is : t.g.H;
  const int parts = (MODE == 1 && t.shared_parts > 1) ? t.shared_parts : 1;
  return ((t.g.n + TT - 1) / TT) * ((units + UNITS - 1) / UNITS) * parts;
}

// Locate work item `item`: the group (binary search over the item prefix),
// then tc_item_local. UNITS = output units per item. Returns false past the
// last item.
template <int MODE, int KBLK, int UNITS, int TT>
__device__ __forceinline__ bool tc_item_at(const TcArgs& t, const TcPlanCache* pc, int item, TcItem& it) {
  const int na = pc->num_active;
  if (item >= pc->total || na <= 0) return false;
  int lo = 0, hi = na - 1;  // largest a with item_start[a] <= item
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (pc->item_start[mid] <= item)
      lo = mid;
    else
      hi = mid - 1;
  }
  const int g = pc->group[lo];
  it.g = g;
  tc_item_local<MODE, KBLK, UNITS, TT>(t, g == t.g.E, pc->rows[lo], item - pc->item_start[lo], it);
  if (MODE == 0)
    it.brow0 = (it.shared ? pc->nk : pc->offset[lo]) + it.tok0;
  else
    it.brow0 = pc->offset[lo] + it.tok0;
  it.slot = it.shared ? 0 : pc->slot[lo];
  it.valid = it.slot >= 0;
  return true;
}

// Prefetch the encoded tensor maps into the TMA unit's descriptor cache (one
// lane), so the first copies do not wait for the descriptor fetch; the maps
// are kernel parameters, so this may run before the kernel waits for the
// one before it.
__device__ __forceinline__ void prefetch_maps(const TcMaps& maps, uint32_t used) {
  const CUtensorMap* m = &maps.a_routed[0];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (used & (1u << i)) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m + i)) : "memory");
}

// bits of TcArgs::maps_used for the maps a launch encoded
inline uint32_t maps_used_bits(const TcMaps& maps) {
  uint32_t bits = 0;
  const unsigned char* p = reinterpret_cast<const unsigned char*>(&maps);
  for (int i = 0; i < 8; ++i) {
    bool any = false;
    for (size_t b = 0; b < sizeof(CUtensorMap) && !any; ++b) any = p[i * sizeof(CUtensorMap) + b] != 0;
    if (any) bits |= 1u << i;
  }
  return bits;
}

// ---------------------------------------------------------------------------
// host side: tensor maps
// ---------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
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

// uint8 tensor map, K innermost (contiguous), box box_k x box_rows [x 1]:
// 128-byte swizzle for MMA operand tiles (box_k = 128), none for staged tiles.
inline int make_map(CUtensorMap* m, const void* base, int rank, uint64_t k, uint64_t rows, uint64_t slots,
                    uint64_t row_stride, uint64_t slot_stride, uint32_t box_rows, const char* what,
                    uint32_t box_k = 128, bool swizzle = true) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(ER_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (((uintptr_t)base & 15) || (row_stride & 15) || (rank == 3 && (slot_stride & 15)))
    return fail(ER_EINVAL, "tensor map %s: base and strides must be 16-byte aligned", what);
  if (box_k % 16 || (swizzle && box_k != 128))
    return fail(ER_EINVAL, "tensor map %s: box width %u bytes", what, box_k);
  const cuuint64_t dims[3] = {k, rows, slots};
  const cuuint64_t strides[2] = {row_stride, slot_stride};
  const cuuint32_t box[3] = {box_k, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, (cuuint32_t)rank, const_cast<void*>(base), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ER_ECUDA, "cuTensorMapEncodeTiled(%s) failed (%d)", what, (int)r);
  return ER_OK;
}

}  // namespace er
