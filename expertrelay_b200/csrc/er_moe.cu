// er_moe.cu -- the MoE block (runtime/qwen_moe.py:293-359) as a fixed sequence
// of device launches with no host synchronisation, so a call can be captured
// in a CUDA graph:
//   K1 router logits (+ shared-gate logit) -> K1 softmax/top-k (+ per-expert counts)
//   K2 plan: expert ranges and work-item schedules -> dispatch: expert-sorted
//      (token, slot) positions (and, for the tensor-core path, h's int8 slices)
//   K3 gate/up + SwiGLU, K3 down (grouped GEMV, SIMT GEMM or tcgen05 GEMM)
//   K4 combine in ascending expert order + gated shared expert
// The same runner serves two parts of the block for expert parallelism:
// er_moe_rows (routed experts on rows that already carry an expert id and a
// weight: K2-K4 with one slot per row and no shared expert) and er_moe_shared
// (the gated shared expert alone: K1's shared gate, K2-K4 with no routed slot).
#include "er_internal.cuh"

namespace er {

enum RunMode { kBlock = 0, kRows = 1, kShared = 2 };

// Test hooks of the tensor-core path (er_tc_test_stall): the bound of every
// mbarrier wait (0: the kernels' default) and which int8 launch withholds
// its last item's accumulator (0 none, 1 gate/up, 2 down).
static unsigned long long g_tc_test_wait_ns = 0;
static int g_tc_test_stall = 0;

struct Run {
  int mode;
  const void* h;  // tokens (kRows: the rows)
  int h_dtype;
  int n;
  const float* logits_in;
  void* y;
  int y_dtype;    // ER_DTYPE_F32, or (kRows) ER_DTYPE_BF16
  float* logits_out;
  int64_t* topk_idx_out;
  float* topk_w_out;
  const int32_t* row_expert;  // kRows
  const float* row_weight;    // kRows
  int path;
  void* const* stage_events;
  int* launch_count;
};

// routed slots per token and whether the shared expert runs
static int run_k(const er_moe_weights* w, int mode) { return mode == kBlock ? w->top_k : (mode == kRows ? 1 : 0); }
static bool run_shared(int mode) { return mode != kRows; }

// partial outputs of the shared expert's down product (K parts of its tiles)
static int shared_parts(const er_moe_weights* w, int n, int path) {
  return path == ER_PATH_TC ? tc_shared_parts(tc_tok_tile(n, w->expert_fmt), w->inter, w->shared_inter) : 1;
}

struct WsLayout {
  size_t logits, gate_logit, gate_sig, idx32, topw, plan, perm_token, perm_w, pos_of, act_r, act_s, y_r, y_s;
  // tensor-core path: int8 activation slices and their row scales
  size_t xs0, xs1, xscale, as0_r, as1_r, ascale_r, as0_s, as1_s, ascale_s;
  size_t total;
};

static WsLayout ws_layout(const er_moe_weights* w, int n, int path, int mode) {
  WsLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  const size_t nk = (size_t)n * run_k(w, mode);
  const size_t ns = run_shared(mode) ? (size_t)n : 0;  // rows through the shared expert
  const size_t nl = mode == kBlock ? (size_t)n : 0;    // rows with router logits
  // partial sums of K slices: the router rows with the shared gate (block), or
  // the shared gate alone (given router logits, or the shared expert), which
  // is split whenever a batch is
  L.logits = take((size_t)router_parts(n, w->num_experts + 1) * nl * w->num_experts * 4);
  L.gate_logit = take((size_t)router_parts(n, 1) * ns * 4);
  L.gate_sig = take(ns * 4);
  L.idx32 = take(mode == kBlock ? nk * 4 : 0);
  L.topw = take(mode == kBlock ? nk * 4 : 0);
  L.plan = take(sizeof(Plan));
  L.perm_token = take(nk * 4);
  L.perm_w = take(nk * 4);
  L.pos_of = take(nk * 4);
  L.act_r = take(nk * w->inter * 4);
  L.act_s = take(ns * w->shared_inter * 4);
  L.y_r = take(nk * w->hidden * 4);
  L.y_s = take(shared_parts(w, n, path) * ns * w->hidden * 4);
  if (path == ER_PATH_TC) {
    const size_t rows = nk + ns;
    L.xs0 = take(rows * w->hidden);
    L.xs1 = take(rows * w->hidden);
    L.xscale = take(rows * 4);
    L.as0_r = take(nk * w->inter);
    L.as1_r = take(nk * w->inter);
    L.ascale_r = take(nk * 4);
    L.as0_s = take(ns * w->shared_inter);
    L.as1_s = take(ns * w->shared_inter);
    L.ascale_s = take(ns * 4);
  }
  L.total = off;
  return L;
}

static int validate(const er_moe_weights* w, int mode) {
  if (!w) return fail(ER_EINVAL, "er_moe: null weights");
  if (w->hidden <= 0 || w->hidden % 16)
    return fail(ER_EINVAL, "er_moe: hidden %d must be a positive multiple of 16", w->hidden);
  if (w->inter <= 0 || w->inter % 16 || w->shared_inter <= 0 || w->shared_inter % 16)
    return fail(ER_EINVAL, "er_moe: inter %d / shared_inter %d must be positive multiples of 16", w->inter,
                w->shared_inter);
  if (w->num_experts < 1 || w->num_experts > kMaxExperts)
    return fail(ER_EINVAL, "er_moe: num_experts %d outside 1..%d", w->num_experts, kMaxExperts);
  if (mode == kBlock && (w->top_k < 1 || w->top_k > kMaxTopK || w->top_k > w->num_experts))
    return fail(ER_EINVAL, "er_moe: top_k %d outside 1..min(%d, num_experts)", w->top_k, kMaxTopK);
  if (w->expert_fmt != ER_FMT_INT8 && w->expert_fmt != ER_FMT_INT4 && w->expert_fmt != ER_FMT_INT4_ZP)
    return fail(ER_EINVAL, "er_moe: unknown expert format %d", w->expert_fmt);
  if (w->expert_fmt != ER_FMT_INT8) {
    if (w->group <= 0 || w->group % 16 || w->hidden % w->group || w->inter % w->group)
      return fail(ER_EINVAL, "er_moe: int4 group %d must be a multiple of 16 dividing hidden %d and inter %d",
                  w->group, w->hidden, w->inter);
  }
  if (mode == kBlock && !w->router_w) return fail(ER_EINVAL, "er_moe: null router weights");
  if (mode != kShared && !w->expert_records) return fail(ER_EINVAL, "er_moe: null expert record table");
  if (mode != kRows && (!w->shared_gate_w || !w->shared_record))
    return fail(ER_EINVAL, "er_moe: null shared-expert weights");
  if (((uintptr_t)w->router_w | (uintptr_t)w->shared_gate_w) & 15)
    return fail(ER_EINVAL, "er_moe: router / shared-gate weights must be 16-byte aligned");
  if ((uintptr_t)w->shared_record & 255) return fail(ER_EINVAL, "er_moe: shared record must be 256-byte aligned");
  return ER_OK;
}

// whether the tensor-core path takes this block's records: int8, or int4
// whose groups and rows fit its tiles
static bool tc_format_ok(const er_moe_weights* w) {
  return w->expert_fmt == ER_FMT_INT8 || tcg_shapes_ok(w->hidden, w->inter, w->shared_inter, w->group);
}

// AUTO: the tensor-core path when it can run (records in an arena, a format
// it takes), else the weight-streaming GEMV for decode batches and the SIMT
// GEMM beyond.
static int pick_path(const er_moe_weights* w, int path, int n) {
  if (path != ER_PATH_AUTO) return path;
  if (tc_format_ok(w) && w->record_arena && w->arena_slots > 0) return ER_PATH_TC;
  return n <= kGemvMaxTok ? ER_PATH_GEMV : ER_PATH_GEMM;
}

static int run_moe(const er_moe_weights* w, const Run& r, void* workspace, size_t workspace_bytes, cudaStream_t st) {
  const int mode = r.mode;
  if (int rc = validate(w, mode)) return rc;
  const int n = r.n;
  if (n < 0) return fail(ER_EINVAL, "er_moe: negative row count");
  if (n == 0) return ER_OK;
  if (!r.h || !r.y) return fail(ER_EINVAL, "er_moe: null input or output");
  if (r.h_dtype != ER_DTYPE_F32 && r.h_dtype != ER_DTYPE_BF16)
    return fail(ER_EINVAL, "er_moe: unknown activation dtype %d", r.h_dtype);
  if (((uintptr_t)r.h | (uintptr_t)r.y) & 15)
    return fail(ER_EINVAL, "er_moe: inputs and outputs must be 16-byte aligned");
  if (mode == kRows && (!r.row_expert || !r.row_weight))
    return fail(ER_EINVAL, "er_moe_rows: null expert ids or weights");
  if (r.y_dtype != ER_DTYPE_F32 && !(mode == kRows && r.y_dtype == ER_DTYPE_BF16))
    return fail(ER_EINVAL, "er_moe: output dtype %d (fp32; bf16 for er_moe_rows)", r.y_dtype);
  const int path = pick_path(w, r.path, n);
  if (path != ER_PATH_GEMV && path != ER_PATH_GEMM && path != ER_PATH_TC)
    return fail(ER_EINVAL, "er_moe: unknown path %d", r.path);
  if (path == ER_PATH_TC) {
    if (!tc_format_ok(w))
      return fail(ER_EINVAL,
                  "er_moe: the tensor-core path takes int8 records, or int4 records whose group (%d) is a multiple "
                  "of 32 dividing hidden and inter, with hidden and shared inter multiples of 128",
                  w->group);
    if (mode != kShared && (!w->record_arena || w->arena_slots < 1 || ((uintptr_t)w->record_arena & 15)))
      return fail(ER_EINVAL, "er_moe: the tensor-core path needs the record arena (record_arena, arena_slots)");
  }
  const WsLayout L = ws_layout(w, n, path, mode);
  if (!workspace || workspace_bytes < L.total)
    return fail(ER_ENOSPACE, "er_moe: workspace %zu bytes, need %zu", workspace_bytes, L.total);
  if ((uintptr_t)workspace & 255) return fail(ER_EINVAL, "er_moe: workspace must be 256-byte aligned");

  char* ws = static_cast<char*>(workspace);
  int launches = 0;
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  if (r.stage_events)
    if (int rc = cuda_check(cudaStreamIsCapturing(st, &capture), "cudaStreamIsCapturing")) return rc;
  auto mark = [&](int i) -> int {
    if (!r.stage_events) return ER_OK;
    // under stream capture the record becomes an external event node, so the
    // graph's replays timestamp the stages too; outside capture a plain record
    const unsigned flags = capture == cudaStreamCaptureStatusActive ? cudaEventRecordExternal : cudaEventRecordDefault;
    return cuda_check(cudaEventRecordWithFlags((cudaEvent_t)r.stage_events[i], st, flags), "cudaEventRecord");
  };
  if (int rc = mark(0)) return rc;
  const int H = w->hidden, E = w->num_experts, k = run_k(w, mode);
  const bool shared = run_shared(mode);
  const size_t nk = (size_t)n * k;
  float* logits = reinterpret_cast<float*>(ws + L.logits);
  float* gate_logit = reinterpret_cast<float*>(ws + L.gate_logit);
  float* gate_sig = shared ? reinterpret_cast<float*>(ws + L.gate_sig) : nullptr;
  Plan* plan = reinterpret_cast<Plan*>(ws + L.plan);
  int32_t* perm_token = reinterpret_cast<int32_t*>(ws + L.perm_token);
  float* perm_w = reinterpret_cast<float*>(ws + L.perm_w);
  int32_t* pos_of = reinterpret_cast<int32_t*>(ws + L.pos_of);
  float* act_r = reinterpret_cast<float*>(ws + L.act_r);
  float* act_s = reinterpret_cast<float*>(ws + L.act_s);
  float* y_r = reinterpret_cast<float*>(ws + L.y_r);
  float* y_s = shared ? reinterpret_cast<float*>(ws + L.y_s) : nullptr;
  const int32_t* idx32 = nullptr;  // expert id of each (token, slot)
  const float* topw = nullptr;     // its routing weight
  TopkArgs topk{};                 // the block's top-k step
  bool fused_topk = false;         // run by the dispatch kernel (small batches)

  // K1: routing (the block), the shared gate alone, or the rows' expert counts
  if (mode == kBlock) {
    int32_t* idx = reinterpret_cast<int32_t*>(ws + L.idx32);
    float* wts = reinterpret_cast<float*>(ws + L.topw);
    const float* lg = logits;
    int nparts = 1, gparts = 1;
    float* logits_sum = r.logits_out;
    if (r.logits_in) {
      if (int rc = launch_router_logits(r.h, r.h_dtype, n, H, nullptr, w->shared_gate_w, 0, nullptr, gate_logit,
                                        &gparts, plan->tally, kPlanClear, st))
        return rc;
      lg = r.logits_in;  // one whole set of logits
      if (logits_sum == r.logits_in) logits_sum = nullptr;
    } else {
      if (int rc = launch_router_logits(r.h, r.h_dtype, n, H, w->router_w, w->shared_gate_w, E, logits, gate_logit,
                                        &nparts, plan->tally, kPlanClear, st, &plan->error))
        return rc;
      gparts = nparts;
    }
    topk.logits = lg;
    topk.nparts = nparts;
    topk.gparts = gparts;
    topk.norm = w->norm_topk_prob;
    topk.idx64 = r.topk_idx_out;
    topk.idx32 = idx;
    topk.wout = wts;
    topk.gate_logit = gate_logit;
    topk.gate_sig = gate_sig;
    topk.logits_sum = logits_sum;
    topk.tally = plan->tally;
    fused_topk = n <= kFusedTopkMaxTok;
    if (!fused_topk) {
      if (int rc = launch_router_topk(topk, n, E, k, st)) return rc;
      launches += 1;
    }
    launches += 1;
    idx32 = idx;
    topw = wts;
  } else if (mode == kShared) {
    int gparts = 1;
    if (int rc = launch_router_logits(r.h, r.h_dtype, n, H, nullptr, w->shared_gate_w, 0, nullptr, gate_logit,
                                      &gparts, nullptr, 0, st))
      return rc;
    if (int rc = launch_gate_sigmoid(gate_logit, gparts, n, gate_sig, st)) return rc;
    if (int rc = cuda_check(cudaMemsetAsync(plan->tally, 0, (size_t)kPlanClear * sizeof(int), st), "clear tally"))
      return rc;
    launches += 2;
  } else {
    if (int rc = launch_tally(r.row_expert, n, E, plan->tally, kPlanClear, st)) return rc;
    launches += 1;
    idx32 = r.row_expert;
    topw = r.row_weight;
  }

  // K2: plan + dispatch
  SchedSpec specs[kNumSched];
  if (path == ER_PATH_GEMV) {
    specs[0] = SchedSpec{0, kGemvUnitsGU, 0};
    specs[1] = SchedSpec{0, kGemvUnitsDN, 1};
  } else if (path == ER_PATH_TC) {
    const int tt = tc_tok_tile(n, w->expert_fmt);
    specs[0] = SchedSpec{tt, tc_units_gu(tt), 0};
    specs[1] = SchedSpec{tt, tc_units_dn(tt), 1, shared_parts(w, n, path)};
  } else {
    specs[0] = SchedSpec{kSimtBM, kSimtBN, 0};
    specs[1] = SchedSpec{kSimtBM, kSimtBN, 1};
  }
  if (int rc = mark(1)) return rc;
  int8_t* xs0 = path == ER_PATH_TC ? reinterpret_cast<int8_t*>(ws + L.xs0) : nullptr;
  int8_t* xs1 = path == ER_PATH_TC ? reinterpret_cast<int8_t*>(ws + L.xs1) : nullptr;
  float* xscale = path == ER_PATH_TC ? reinterpret_cast<float*>(ws + L.xscale) : nullptr;
  if (int rc = launch_dispatch(r.h, r.h_dtype, idx32, topw, n, k, E, H, w->inter, w->shared_inter, specs, shared,
                               plan, static_cast<const uint64_t*>(w->expert_records), perm_token, perm_w, pos_of, xs0,
                               xs1, xscale, fused_topk ? &topk : nullptr, st))
    return rc;
  launches += 1;
  if (mode == kBlock && r.topk_w_out) {
    if (int rc = cuda_check(cudaMemcpyAsync(r.topk_w_out, topw, nk * 4, cudaMemcpyDeviceToDevice, st),
                            "copy top-k weights"))
      return rc;
  }
  if (int rc = mark(2)) return rc;

  GroupArgs ga;
  ga.plan = plan;
  ga.expert_records = w->expert_records;
  ga.shared_record = static_cast<const uint8_t*>(w->shared_record);
  ga.fmt = w->expert_fmt;
  ga.H = H;
  ga.I = w->inter;
  ga.Is = w->shared_inter;
  ga.group = w->expert_fmt == ER_FMT_INT8 ? 1 : w->group;
  ga.E = E;
  ga.n = n;
  ga.perm_token = perm_token;
  ga.perm_w = perm_w;
  ga.gate_sig = gate_sig;

  const long long b0 = sched_items_bound(specs[0], n, k, E, H, w->inter, w->shared_inter);
  const long long b1 = sched_items_bound(specs[1], n, k, E, H, w->inter, w->shared_inter);
  // one int8 instance (the shared expert and int8 routed experts), plus one
  // instance of the routed format when it is int4
  const int per_stage = (w->expert_fmt == ER_FMT_INT8 || path == ER_PATH_TC) ? 1 : 2;
  if (path == ER_PATH_TC) {
    int8_t* as0_r = reinterpret_cast<int8_t*>(ws + L.as0_r);
    int8_t* as1_r = reinterpret_cast<int8_t*>(ws + L.as1_r);
    float* ascale_r = reinterpret_cast<float*>(ws + L.ascale_r);
    int8_t* as0_s = reinterpret_cast<int8_t*>(ws + L.as0_s);
    int8_t* as1_s = reinterpret_cast<int8_t*>(ws + L.as1_s);
    float* ascale_s = reinterpret_cast<float*>(ws + L.ascale_s);
    TcLaunch tl{};
    tl.g = ga;
    tl.arena = w->record_arena;
    tl.arena_slots = w->arena_slots;
    tl.fmt = w->expert_fmt;
    tl.group = w->expert_fmt == ER_FMT_INT8 ? 1 : w->group;
    tl.record_bytes = er_record_bytes(w->expert_fmt, H, w->inter, w->group);
    tl.nk = (int)nk;
    tl.n = shared ? n : 0;
    tl.has_shared = shared;
    tl.tok_tile = tc_tok_tile(n, w->expert_fmt);
    tl.wait_ns = g_tc_test_wait_ns;
    tl.stall_last = 0;
    tl.mode = 0;
    tl.sched = 0;
    tl.b0_r = xs0;
    tl.b1_r = xs1;
    tl.xscale_r = xscale;
    tl.out_r = act_r;
    tl.out_s = act_s;
    tl.items_bound = b0;
    tl.stall_last = g_tc_test_stall == 1;
    if (int rc = (tl.fmt == ER_FMT_INT8 ? launch_tc_grouped : launch_tcg_grouped)(tl, st)) return rc;
    if (int rc = mark(3)) return rc;
    if (nk > 0 || shared) {
      const SliceSet routed{act_r, (int)nk, w->inter, as0_r, as1_r, ascale_r};
      const SliceSet shared_rows{act_s, shared ? n : 0, w->shared_inter, as0_s, as1_s, ascale_s};
      if (int rc = launch_slice_sets(routed, shared_rows, st)) return rc;
      launches += 1;
    }
    tl.mode = 1;
    tl.sched = 1;
    tl.b0_r = as0_r;
    tl.b1_r = as1_r;
    tl.b0_s = as0_s;
    tl.b1_s = as1_s;
    tl.xscale_r = ascale_r;
    tl.xscale_s = ascale_s;
    tl.out_r = y_r;
    tl.out_s = y_s;
    tl.shared_parts = specs[1].ks;
    tl.items_bound = b1;
    tl.stall_last = g_tc_test_stall == 2;
    if (int rc = (tl.fmt == ER_FMT_INT8 ? launch_tc_grouped : launch_tcg_grouped)(tl, st)) return rc;
  } else if (path == ER_PATH_GEMV) {
    if (int rc = launch_gemv_grouped(ga, 0, 0, r.h, r.h_dtype, act_r, act_s, nullptr, nullptr, b0, st)) return rc;
    if (int rc = mark(3)) return rc;
    if (int rc = launch_gemv_grouped(ga, 1, 1, nullptr, ER_DTYPE_F32, act_r, act_s, y_r, y_s, b1, st)) return rc;
  } else {
    if (int rc = launch_gemm_simt_grouped(ga, 0, 0, r.h, r.h_dtype, act_r, act_s, nullptr, nullptr, b0, st))
      return rc;
    if (int rc = mark(3)) return rc;
    if (int rc = launch_gemm_simt_grouped(ga, 1, 1, nullptr, ER_DTYPE_F32, act_r, act_s, y_r, y_s, b1, st))
      return rc;
  }
  launches += 2 * per_stage;
  if (int rc = mark(4)) return rc;
  // K4
  if (int rc = launch_combine_dt(y_r, ER_DTYPE_F32, y_s, specs[1].ks, pos_of, idx32, n, k, H, &plan->error, r.y,
                                 r.y_dtype, st))
    return rc;
  launches += 1;
  if (r.launch_count) *r.launch_count += launches;
  return mark(5);
}

}  // namespace er

using namespace er;

extern "C" int er_tc_test_stall(unsigned long long wait_ns, int stall) {
  if (stall < 0 || stall > 2) return fail(ER_EINVAL, "er_tc_test_stall: stall %d (0 none, 1 gate/up, 2 down)", stall);
  g_tc_test_wait_ns = wait_ns;
  g_tc_test_stall = stall;
  return ER_OK;
}

extern "C" int er_moe_error_bits(const er_moe_weights* w, int n, int path, const void* workspace, int* bits,
                                 void* stream) {
  if (!bits) return fail(ER_EINVAL, "er_moe_error_bits: null output");
  *bits = 0;
  if (int rc = validate(w, kBlock)) return rc;
  if (n <= 0) return ER_OK;
  if (!workspace) return fail(ER_EINVAL, "er_moe_error_bits: null workspace");
  const WsLayout L = ws_layout(w, n, pick_path(w, path, n), kBlock);
  const Plan* plan = reinterpret_cast<const Plan*>(static_cast<const char*>(workspace) + L.plan);
  cudaStream_t st = (cudaStream_t)stream;
  if (int rc = cuda_check(cudaMemcpyAsync(bits, &plan->error, sizeof(int), cudaMemcpyDeviceToHost, st),
                          "er_moe_error_bits: copy"))
    return rc;
  return cuda_check(cudaStreamSynchronize(st), "er_moe_error_bits: sync");
}

extern "C" size_t er_moe_workspace_bytes(const er_moe_weights* w, int n, int path) {
  if (validate(w, kBlock) != ER_OK || n < 0) return 0;
  return ws_layout(w, n, pick_path(w, path, n), kBlock).total;
}

extern "C" int er_moe_block(const er_moe_weights* w, const er_moe_io* io, void* workspace, size_t workspace_bytes,
                            void* stream) {
  if (!io) return fail(ER_EINVAL, "er_moe_block: null io");
  Run r{};
  r.mode = kBlock;
  r.h = io->h;
  r.h_dtype = io->h_dtype;
  r.n = io->n;
  r.logits_in = io->logits_in;
  r.y = io->y;
  r.logits_out = io->logits_out;
  r.topk_idx_out = io->topk_idx_out;
  r.topk_w_out = io->topk_w_out;
  r.path = io->path;
  r.stage_events = io->stage_events;
  r.launch_count = io->launch_count;
  return run_moe(w, r, workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" size_t er_moe_rows_workspace_bytes(const er_moe_weights* w, int m, int path) {
  if (validate(w, kRows) != ER_OK || m < 0) return 0;
  return ws_layout(w, m, pick_path(w, path, m), kRows).total;
}

extern "C" int er_moe_rows(const er_moe_weights* w, const er_moe_rows_io* io, void* workspace, size_t workspace_bytes,
                           void* stream) {
  if (!io) return fail(ER_EINVAL, "er_moe_rows: null io");
  Run r{};
  r.mode = kRows;
  r.h = io->x;
  r.h_dtype = io->x_dtype;
  r.n = io->m;
  r.y = io->y;
  r.row_expert = io->expert;
  r.row_weight = io->weight;
  r.y_dtype = io->y_dtype;
  r.path = io->path;
  r.launch_count = io->launch_count;
  return run_moe(w, r, workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" size_t er_moe_shared_workspace_bytes(const er_moe_weights* w, int n, int path) {
  if (validate(w, kShared) != ER_OK || n < 0) return 0;
  return ws_layout(w, n, pick_path(w, path, n), kShared).total;
}

extern "C" int er_moe_shared(const er_moe_weights* w, const void* h, int h_dtype, int n, float* y, int path,
                             void* workspace, size_t workspace_bytes, void* stream) {
  Run r{};
  r.mode = kShared;
  r.h = h;
  r.h_dtype = h_dtype;
  r.n = n;
  r.y = y;
  r.path = path;
  return run_moe(w, r, workspace, workspace_bytes, (cudaStream_t)stream);
}

extern "C" int er_moe_combine(const void* y_rows, int rows_dtype, const int32_t* pos_of, const int32_t* idx,
                              const float* y_shared, int n, int k, int hidden, float* y, void* stream) {
  if (n < 0 || k < 0 || k > kMaxTopK || hidden <= 0 || hidden % 4)
    return fail(ER_EINVAL, "er_moe_combine: n %d, k %d (<= %d), hidden %d (a multiple of 4)", n, k, kMaxTopK, hidden);
  if (rows_dtype != ER_DTYPE_F32 && rows_dtype != ER_DTYPE_BF16)
    return fail(ER_EINVAL, "er_moe_combine: rows dtype %d", rows_dtype);
  if (n == 0) return ER_OK;
  if (!y || (k > 0 && (!y_rows || !pos_of || !idx))) return fail(ER_EINVAL, "er_moe_combine: null argument");
  if ((((uintptr_t)y_shared | (uintptr_t)y) & 15) || ((uintptr_t)y_rows & (rows_dtype == ER_DTYPE_BF16 ? 7 : 15)))
    return fail(ER_EINVAL, "er_moe_combine: rows must be aligned (16 bytes; 8 for bf16 rows)");
  return launch_combine_dt(y_rows, rows_dtype, y_shared, 1, pos_of, idx, n, k, hidden, nullptr, y, ER_DTYPE_F32,
                           (cudaStream_t)stream);
}
