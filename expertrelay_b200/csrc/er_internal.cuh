// er_internal.cuh -- internal types and launchers shared by the .cu files.
#pragma once

#include "er_common.cuh"

namespace er {

constexpr int kRouterTok = 8;  // tokens per router CTA

// A schedule enumerates work items over the active groups. Group g < E is
// routed expert g (its tokens in expert-sorted order), group E is the shared
// expert (all n tokens). Item count of group g = mtiles(g) * ntiles(g).
struct SchedSpec {
  int bm;      // tokens per item (0: all tokens of the group in one item)
  int bn;      // output units per item
  int which;   // 0: gate/up (units = intermediate columns), 1: down (units = hidden rows)
  int ks = 1;  // down only: parts the shared expert's K is split into (partial outputs)
};

constexpr int kNumSched = 2;

// Routing plan in the workspace. `tally`, `cursor` and `error` are cleared
// (kPlanClear ints from `tally`) before the top-k kernel counts into `tally`;
// the dispatch kernel turns the counts into groups and schedules and claims
// expert-sorted positions through `cursor`. Every kernel that reports a
// problem sets its bit of `error` with atomicOr, so no report is lost.
struct Plan {
  int n, E, k, nk;
  int num_active;                      // groups with at least one token (shared first)
  int counts[kMaxExperts + 1];         // tokens per group (counts[E] = n)
  int offsets[kMaxExperts + 1];        // first expert-sorted position of each routed group
  int active[kMaxExperts + 1];         // active group ids: the shared expert first, then routed ascending
  int item_start[kNumSched][kMaxExperts + 2];  // prefix of items over active groups
  // by active position, for the tensor-core kernels' one-round plan read:
  // the group's tokens, first expert-sorted position and record address (0
  // for the shared expert, or when the dispatch was given no expert table)
  int act_rows[kMaxExperts + 1];
  int act_off[kMaxExperts + 1];
  unsigned long long act_rec[kMaxExperts + 1];
  SchedSpec sched[kNumSched];
  int tally[kMaxExperts];              // (token, slot) pairs routed to each expert
  int cursor[kMaxExperts];             // positions of each expert's range claimed so far
  // bits: 1 an expert id out of range, 2 tallies and ids disagree (or do not
  // add up to n * k), 4 a record outside the arena, 8 a tensor-core wait
  // gave up; the combine writes NaN rows when any is set
  int error;
};
constexpr int kPlanClear = 2 * kMaxExperts + 1;  // tally, cursor and error, contiguous

// Everything a grouped expert kernel needs to find a group's tokens and weights.
struct GroupArgs {
  const Plan* plan;
  const uint64_t* expert_records;  // device [E]
  const uint8_t* shared_record;
  int fmt;                         // routed format (shared is ER_FMT_INT8)
  int H, I, Is, group, E, n;
  const int32_t* perm_token;       // [nk] token of each expert-sorted position
  const float* perm_w;             // [nk] routing weight of each position
  const float* gate_sig;           // [n] sigmoid(shared gate logit)
};

struct GroupView {
  const uint8_t* rec;
  int fmt, inter, rows, row0;
  bool shared;
};

__device__ __forceinline__ GroupView group_view(const GroupArgs& a, int g) {
  GroupView v;
  v.shared = (g == a.E);
  v.rec = v.shared ? a.shared_record : reinterpret_cast<const uint8_t*>(a.expert_records[g]);
  v.fmt = v.shared ? ER_FMT_INT8 : a.fmt;
  v.inter = v.shared ? a.Is : a.I;
  v.rows = a.plan->counts[g];
  v.row0 = v.shared ? 0 : a.plan->offsets[g];
  return v;
}

// Locate work item `item` of schedule `s`: returns the group id and the
// item's index inside the group, or -1 past the end.
__device__ __forceinline__ int find_item(const Plan* P, int s, int item, int* local) {
  const int na = P->num_active;
  if (item >= P->item_start[s][na]) return -1;
  int lo = 0, hi = na - 1;  // largest a with item_start[a] <= item
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (P->item_start[s][mid] <= item)
      lo = mid;
    else
      hi = mid - 1;
  }
  *local = item - P->item_start[s][lo];
  return P->active[lo];
}

// Two int8 slices of four values: with inv = 127 / max|x| of the row,
// x ~= (x0 + x1 / 256) / inv, x0 = rint(x inv), x1 = rint((x inv - x0) 256)
// clamped to +-127. Packs the low bytes, first value in the lowest byte.
__device__ __forceinline__ void slice4(float4 v, float inv, uint32_t& w0, uint32_t& w1) {
  const float f[4] = {v.x, v.y, v.z, v.w};
  int i0[4], i1[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float y = f[j] * inv;
    const float q0 = rintf(y);
    i0[j] = (int)q0;
    i1[j] = max(-127, min(127, __float2int_rn((y - q0) * 256.f)));
  }
  w0 = __byte_perm(__byte_perm(i0[0], i0[1], 0x0040), __byte_perm(i0[2], i0[3], 0x0040), 0x5410);
  w1 = __byte_perm(__byte_perm(i1[0], i1[1], 0x0040), __byte_perm(i1[2], i1[3], 0x0040), 0x5410);
}

__device__ __forceinline__ float abs_max4(float4 v) {
  return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
}

// launchers (each returns an ER_* status)
// Router logits; large batches write kRouterKSplit partial sums (K slices)
// into logits / gate_logit (each n*E / n apart), *nparts says how many.
constexpr int kRouterKSplit = 4;
// partial logits the router writes for a batch of n tokens and `rows` weight
// rows (E, plus one for the shared gate): K slices for the tiled kernel
// (more than 64 tokens, at most 64 rows), one set otherwise
inline int router_parts(int n, int rows) { return (n <= 64 || rows > 64) ? 1 : kRouterKSplit; }
// `tally` (optional, `ntally` ints) is cleared for the top-k kernel's counts.
// Batches of more than 64 tokens with at most 64 router rows run on the
// tensor cores (er_router_tc.cu), which set bit 8 of `error` (optional) if
// one of their waits gives up.
int launch_router_logits(const void* h, int h_dtype, int n, int H, const float* wr, const float* wg, int E,
                         float* logits, float* gate_logit, int* nparts, int* tally, int ntally, cudaStream_t st,
                         int* error = nullptr);
// the tensor-core router (er_router_tc.cu): whether it takes the batch, and its launch
bool router_tc_ok(int n, int H, int E, const void* wr, const void* wg);
int launch_router_tc(const void* h, int h_dtype, int n, int H, const float* wr, const float* wg, int E, float* logits,
                     float* gate_logit, int* tally, int ntally, int* error, cudaStream_t st);
// The top-k step's inputs and outputs: softmax + top-k over the sum of
// `nparts` partial logits (and the sigmoid of `gparts` partial shared-gate
// logits).
struct TopkArgs {
  const float* logits;      // [nparts][n][E] partial logits, added in order
  int nparts, gparts;       // logit / shared-gate partials
  int norm;                 // renormalise the k weights to sum 1
  int64_t* idx64;           // optional [n, k] ids
  int32_t* idx32;           // optional [n, k] ids
  float* wout;              // optional [n, k] weights
  const float* gate_logit;  // optional [gparts][n] shared-gate partial logits
  float* gate_sig;          // optional [n] sigmoid of their sum
  float* logits_sum;        // optional [n, E] summed logits
  int* tally;               // optional [E] counts of the selected (token, slot) pairs per expert
};
int launch_router_topk(const TopkArgs& a, int n, int E, int k, cudaStream_t st);
// Batches of at most this many tokens run the top-k inside the dispatch kernel.
constexpr int kFusedTopkMaxTok = 16;
// The plan (groups, ranges, work-item schedules; the shared expert, all n
// tokens, is the first group when `shared` is nonzero) from plan->tally, and
// the scatter of the (token, slot) pairs to expert-sorted positions; `records`
// (nullable): the expert table, copied into the plan by active position
// (perm_token, perm_w, pos_of). With s0 non-null also slices each token's h
// row once and writes the slices to its k routed positions and, when
// `shared` is nonzero, to shared row nk + t. With `topk` non-null (n <=
// kFusedTopkMaxTok) the kernel first runs that top-k step itself, whose
// idx32 / wout / tally must be idx / w / plan->tally.
int launch_dispatch(const void* h, int h_dtype, const int32_t* idx, const float* w, int n, int k, int E, int H, int I,
                    int Is, const SchedSpec* specs, int shared, Plan* plan, const uint64_t* records,
                    int32_t* perm_token, float* perm_w, int32_t* pos_of, int8_t* s0, int8_t* s1, float* scale,
                    const TopkArgs* topk, cudaStream_t st);
// Upper bound of the items a schedule can produce (host side, for grid sizing).
long long sched_items_bound(const SchedSpec& s, int n, int k, int E, int H, int I, int Is);

int launch_gemv_grouped(const GroupArgs& a, int sched, int mode, const void* x, int x_dtype, float* act_r,
                        float* act_s, float* out_r, float* out_s, long long items_bound, cudaStream_t st);
int launch_gemm_simt_grouped(const GroupArgs& a, int sched, int mode, const void* x, int x_dtype,
                             float* act_r, float* act_s, float* out_r, float* out_s,
                             long long items_bound, cudaStream_t st);
// out[t] = sum over t's k slots, in ascending expert id (idx), of y_r[pos_of[t * k + j]]
// (+ the `parts` partial shared rows y_s[p * n + t], in order, when y_s is not
// NULL); rows of NaN when *error is nonzero
int launch_combine(const float* y_r, const float* y_s, int parts, const int32_t* pos_of, const int32_t* idx, int n,
                   int k, int H, const int* error, float* out, cudaStream_t st);
// the same with the row results and the output in ER_DTYPE_F32 or ER_DTYPE_BF16
int launch_combine_dt(const void* y_r, int r_dtype, const float* y_s, int parts, const int32_t* pos_of,
                      const int32_t* idx, int n, int k, int H, const int* error, void* out, int o_dtype,
                      cudaStream_t st);
// per-expert counts of ids[0..m) into tally[E] (nclear ints from tally cleared
// first); out-of-range ids are not counted
int launch_tally(const int32_t* ids, int m, int E, int* tally, int nclear, cudaStream_t st);
// gate_sig[t] = sigmoid(sum of the nparts partial shared-gate logits of token t)
int launch_gate_sigmoid(const float* gate_logit, int nparts, int n, float* gate_sig, cudaStream_t st);

// rows [0, rows) of a [rows, K] fp32 matrix to slice (the same outputs as launch_slice_rows)
struct SliceSet {
  const float* src;
  int rows, K;
  int8_t *s0, *s1;
  float* scale;
};

// tcgen05 grouped GEMM (er_tc.cu)
struct TcLaunch {
  GroupArgs g;
  int mode, sched;
  const void* arena;           // routed records, arena_slots x record_bytes
  int arena_slots;
  size_t record_bytes;
  int nk, n;
  int tok_tile;                // tokens per work item: 16 (decode batches) or 128
  const int8_t *b0_r, *b1_r;   // B slices: mode 0 all nk + n rows of h; mode 1 routed act rows
  const int8_t *b0_s, *b1_s;   // mode 1: shared act rows
  int has_shared;              // the shared expert is one of the groups (its maps are needed)
  const float *xscale_r, *xscale_s;
  float *out_r, *out_s;        // mode 1: out_s holds shared_parts partial [n, H] outputs
  int shared_parts;            // mode 1: K parts of the shared expert's down items (the schedule's ks)
  long long items_bound;
  int fmt, group;              // routed record format and int4 group size (the shared expert is int8)
  unsigned long long wait_ns;  // mbarrier wait bound (0: the default)
  int stall_last;              // test hook (er_tc_test_stall): withhold the last item's accumulator
};
int launch_tc_grouped(const TcLaunch& L, cudaStream_t st);
// the same for int4 routed records (group-scaled; er_tcg.cu); the shared expert stays int8
int launch_tcg_grouped(const TcLaunch& L, cudaStream_t st);
// two int8 slices and a scale per row of a [rows, K] fp32 / bf16 matrix
int launch_slice_rows(const void* src, int dtype, int rows, int K, int8_t* s0, int8_t* s1, float* scale,
                      cudaStream_t st);
// two such sets in one launch (K up to 8192 each)
int launch_slice_sets(const SliceSet& a, const SliceSet& b, cudaStream_t st);
// tokens per tcgen05 work item: 16 when every group fits (n <= 16), else 128
// for int8 records (SM pairs) and 64 for int4 records (single SMs)
inline int tc_tok_tile(int n, int fmt = ER_FMT_INT8) { return n <= 16 ? 16 : (fmt == ER_FMT_INT8 ? 128 : 64); }
// whether the int4 tensor-core path takes these shapes (groups in whole
// 32-input MMA steps, rows in whole 16-byte TMA strides)
inline bool tcg_shapes_ok(int H, int I, int Is, int group) {
  return group > 0 && group % 32 == 0 && H % group == 0 && I % group == 0 && H % 128 == 0 && I % 32 == 0 &&
         Is % 128 == 0 && H / group <= 64 && I / group <= 64;
}
constexpr int kTcKBlock = 256;  // K elements per tcgen05 pipeline stage
// Decode tiles split the shared expert's down product (K = Is, Is / I times a
// routed expert's) into parts of about a routed expert's K, so its items take
// no longer than the others; the parts' outputs are added by the combine.
// Every part is non-empty: ks = ceil(blocks / ceil(blocks / wanted)).
inline int tc_shared_parts(int tok_tile, int I, int Is) {
  if (tok_tile > 16) return 1;
  const int blocks = (Is + kTcKBlock - 1) / kTcKBlock;
  const int want = Is / I > 1 ? Is / I : 1;
  const int span = (blocks + want - 1) / want;
  return (blocks + span - 1) / span;
}
// CTAs per work item: 128-token tiles run on an SM pair (tcgen05 cta_group::2,
// M = 256), 16-token tiles on one SM.
inline int tc_cta_group(int tok_tile) { return tok_tile >= 128 ? 2 : 1; }
// intermediate columns per gate/up item (64 gate + 64 up rows per CTA)
inline int tc_units_gu(int tok_tile) { return 64 * tc_cta_group(tok_tile); }
// hidden rows per down item (128 per CTA)
inline int tc_units_dn(int tok_tile) { return 128 * tc_cta_group(tok_tile); }

// GEMV schedule geometry (er_gemv.cu): units per item
constexpr int kGemvWarps = 8;
constexpr int kGemvRowsPerWarp = 8;          // weight rows per warp
constexpr int kGemvUnitsGU = kGemvWarps * kGemvRowsPerWarp / 2;  // 32 intermediate columns (gate+up rows)
constexpr int kGemvUnitsDN = kGemvWarps * kGemvRowsPerWarp;      // 64 output rows
constexpr int kGemvMaxTok = 8;               // tokens per pass
// SIMT GEMM tile (er_gemm_simt.cu)
constexpr int kSimtBM = 64;
constexpr int kSimtBN = 64;

}  // namespace er
