// er_moe.cu -- er_moe_block: the whole MoE block (runtime/qwen_moe.py:293-359)
// as a fixed sequence of device launches with no host synchronisation, so
// the call can be captured in a CUDA graph:
//   K1 router logits (+ shared-gate logit) -> K1 softmax/top-k (+ per-expert counts)
//   K2 plan: expert ranges and work-item schedules -> dispatch: expert-sorted
//      (token, slot) positions (and, for the tensor-core path, h's int8 slices)
//   K3 gate/up + SwiGLU, K3 down (grouped GEMV for decode, GEMM otherwise)
//   K4 combine in ascending expert order + gated shared expert
#include "er_internal.cuh"

namespace er {

struct WsLayout {
  size_t logits, gate_logit, gate_sig, idx32, topw, plan, perm_token, perm_w, pos_of, act_r, act_s, y_r, y_s;
  // tensor-core path: int8 activation slices and their row scales
  size_t xs0, xs1, xscale, as0_r, as1_r, ascale_r, as0_s, as1_s, ascale_s;
  size_t total;
};

static WsLayout ws_layout(const er_moe_weights* w, int n, int path) {
  WsLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  const size_t nk = (size_t)n * w->top_k;
  L.logits = take((size_t)kRouterKSplit * n * w->num_experts * 4);  // partial sums of K slices
  L.gate_logit = take((size_t)kRouterKSplit * n * 4);
  L.gate_sig = take((size_t)n * 4);
  L.idx32 = take(nk * 4);
  L.topw = take(nk * 4);
  L.plan = take(sizeof(Plan));
  L.perm_token = take(nk * 4);
  L.perm_w = take(nk * 4);
  L.pos_of = take(nk * 4);
  L.act_r = take(nk * w->inter * 4);
  L.act_s = take((size_t)n * w->shared_inter * 4);
  L.y_r = take(nk * w->hidden * 4);
  L.y_s = take((size_t)n * w->hidden * 4);
  if (path == ER_PATH_TC) {
    const size_t rows = nk + n;
    L.xs0 = take(rows * w->hidden);
    L.xs1 = take(rows * w->hidden);
    L.xscale = take(rows * 4);
    L.as0_r = take(nk * w->inter);
    L.as1_r = take(nk * w->inter);
    L.ascale_r = take(nk * 4);
    L.as0_s = take((size_t)n * w->shared_inter);
    L.as1_s = take((size_t)n * w->shared_inter);
    L.ascale_s = take((size_t)n * 4);
  }
  L.total = off;
  return L;
}

static int validate(const er_moe_weights* w) {
  if (!w) return fail(ER_EINVAL, "er_moe: null weights");
  if (w->hidden <= 0 || w->hidden % 16)
    return fail(ER_EINVAL, "er_moe: hidden %d must be a positive multiple of 16", w->hidden);
  if (w->inter <= 0 || w->inter % 16 || w->shared_inter <= 0 || w->shared_inter % 16)
    return fail(ER_EINVAL, "er_moe: inter %d / shared_inter %d must be positive multiples of 16", w->inter,
                w->shared_inter);
  if (w->num_experts < 1 || w->num_experts > kMaxExperts)
    return fail(ER_EINVAL, "er_moe: num_experts %d outside 1..%d", w->num_experts, kMaxExperts);
  if (w->top_k < 1 || w->top_k > kMaxTopK || w->top_k > w->num_experts)
    return fail(ER_EINVAL, "er_moe: top_k %d outside 1..min(%d, num_experts)", w->top_k, kMaxTopK);
  if (w->expert_fmt != ER_FMT_INT8 && w->expert_fmt != ER_FMT_INT4 && w->expert_fmt != ER_FMT_INT4_ZP)
    return fail(ER_EINVAL, "er_moe: unknown expert format %d", w->expert_fmt);
  if (w->expert_fmt != ER_FMT_INT8) {
    if (w->group <= 0 || w->group % 16 || w->hidden % w->group || w->inter % w->group)
      return fail(ER_EINVAL, "er_moe: int4 group %d must be a multiple of 16 dividing hidden %d and inter %d",
                  w->group, w->hidden, w->inter);
  }
  if (!w->router_w || !w->shared_gate_w || !w->expert_records || !w->shared_record)
    return fail(ER_EINVAL, "er_moe: null weight pointer");
  if (((uintptr_t)w->router_w | (uintptr_t)w->shared_gate_w) & 15)
    return fail(ER_EINVAL, "er_moe: router / shared-gate weights must be 16-byte aligned");
  if ((uintptr_t)w->shared_record & 255) return fail(ER_EINVAL, "er_moe: shared record must be 256-byte aligned");
  return ER_OK;
}

static int pick_path(int path, int n) {
  if (path != ER_PATH_AUTO) return path;
  return n <= kGemvMaxTok ? ER_PATH_GEMV : ER_PATH_GEMM;
}

}  // namespace er

using namespace er;

extern "C" size_t er_moe_workspace_bytes(const er_moe_weights* w, int n, int path) {
  if (validate(w) != ER_OK || n < 0) return 0;
  return ws_layout(w, n, pick_path(path, n)).total;
}

extern "C" int er_moe_block(const er_moe_weights* w, const er_moe_io* io, void* workspace, size_t workspace_bytes,
                            void* stream) {
  if (int rc = validate(w)) return rc;
  if (!io) return fail(ER_EINVAL, "er_moe_block: null io");
  const int n = io->n;
  if (n < 0) return fail(ER_EINVAL, "er_moe_block: negative n");
  if (n == 0) return ER_OK;
  if (!io->h || !io->y) return fail(ER_EINVAL, "er_moe_block: null h or y");
  if (io->h_dtype != ER_DTYPE_F32 && io->h_dtype != ER_DTYPE_BF16)
    return fail(ER_EINVAL, "er_moe_block: unknown activation dtype %d", io->h_dtype);
  if (((uintptr_t)io->h | (uintptr_t)io->y) & 15) return fail(ER_EINVAL, "er_moe_block: h and y must be 16-byte aligned");
  const int path = pick_path(io->path, n);
  if (path != ER_PATH_GEMV && path != ER_PATH_GEMM && path != ER_PATH_TC)
    return fail(ER_EINVAL, "er_moe_block: unknown path %d", io->path);
  if (path == ER_PATH_TC) {
    if (w->expert_fmt != ER_FMT_INT8)
      return fail(ER_EINVAL, "er_moe_block: the tensor-core path takes int8 expert records");
    if (!w->record_arena || w->arena_slots < 1 || ((uintptr_t)w->record_arena & 15))
      return fail(ER_EINVAL, "er_moe_block: the tensor-core path needs the record arena (record_arena, arena_slots)");
  }
  const WsLayout L = ws_layout(w, n, path);
  if (!workspace || workspace_bytes < L.total)
    return fail(ER_ENOSPACE, "er_moe_block: workspace %zu bytes, need %zu", workspace_bytes, L.total);
  if ((uintptr_t)workspace & 255) return fail(ER_EINVAL, "er_moe_block: workspace must be 256-byte aligned");

  cudaStream_t st = (cudaStream_t)stream;
  char* ws = static_cast<char*>(workspace);
  int launches = 0;
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  if (io->stage_events)
    if (int rc = cuda_check(cudaStreamIsCapturing(st, &capture), "cudaStreamIsCapturing")) return rc;
  auto mark = [&](int i) -> int {
    if (!io->stage_events) return ER_OK;
    // under stream capture the record becomes an external event node, so the
    // graph's replays timestamp the stages too; outside capture a plain record
    const unsigned flags = capture == cudaStreamCaptureStatusActive ? cudaEventRecordExternal : cudaEventRecordDefault;
    return cuda_check(cudaEventRecordWithFlags((cudaEvent_t)io->stage_events[i], st, flags), "cudaEventRecord");
  };
  if (int rc = mark(0)) return rc;
  const int H = w->hidden, E = w->num_experts, k = w->top_k;
  float* logits = reinterpret_cast<float*>(ws + L.logits);
  float* gate_logit = reinterpret_cast<float*>(ws + L.gate_logit);
  float* gate_sig = reinterpret_cast<float*>(ws + L.gate_sig);
  int32_t* idx32 = reinterpret_cast<int32_t*>(ws + L.idx32);
  float* topw = reinterpret_cast<float*>(ws + L.topw);
  Plan* plan = reinterpret_cast<Plan*>(ws + L.plan);
  int32_t* perm_token = reinterpret_cast<int32_t*>(ws + L.perm_token);
  float* perm_w = reinterpret_cast<float*>(ws + L.perm_w);
  int32_t* pos_of = reinterpret_cast<int32_t*>(ws + L.pos_of);
  float* act_r = reinterpret_cast<float*>(ws + L.act_r);
  float* act_s = reinterpret_cast<float*>(ws + L.act_s);
  float* y_r = reinterpret_cast<float*>(ws + L.y_r);
  float* y_s = reinterpret_cast<float*>(ws + L.y_s);

  // K1: router (or only the shared-gate row when the caller supplies logits)
  const float* lg = logits;
  int nparts = 1, gparts = 1;
  float* logits_sum = io->logits_out;
  if (io->logits_in) {
    if (int rc = launch_router_logits(io->h, io->h_dtype, n, H, nullptr, w->shared_gate_w, 0, nullptr, gate_logit,
                                      &gparts, plan->tally, E, st))
      return rc;
    lg = io->logits_in;  // one whole set of logits
    if (logits_sum == io->logits_in) logits_sum = nullptr;
  } else {
    if (int rc = launch_router_logits(io->h, io->h_dtype, n, H, w->router_w, w->shared_gate_w, E, logits, gate_logit,
                                      &nparts, plan->tally, E, st))
      return rc;
    gparts = nparts;
  }
  if (int rc = launch_router_topk(lg, nparts, gparts, n, E, k, w->norm_topk_prob, io->topk_idx_out, idx32, topw,
                                  gate_logit, gate_sig, logits_sum, plan->tally, st))
    return rc;
  launches += 2;
  if (io->topk_w_out) {
    if (int rc = cuda_check(cudaMemcpyAsync(io->topk_w_out, topw, (size_t)n * k * 4, cudaMemcpyDeviceToDevice, st),
                            "copy top-k weights"))
      return rc;
  }

  // K2: plan
  SchedSpec specs[kNumSched];
  if (path == ER_PATH_GEMV) {
    specs[0] = SchedSpec{0, kGemvUnitsGU, 0};
    specs[1] = SchedSpec{0, kGemvUnitsDN, 1};
  } else if (path == ER_PATH_TC) {
    specs[0] = SchedSpec{tc_tok_tile(n), tc_units_gu(tc_tok_tile(n)), 0};
    specs[1] = SchedSpec{tc_tok_tile(n), tc_units_dn(tc_tok_tile(n)), 1};
  } else {
    specs[0] = SchedSpec{kSimtBM, kSimtBN, 0};
    specs[1] = SchedSpec{kSimtBM, kSimtBN, 1};
  }
  if (int rc = mark(1)) return rc;
  if (int rc = launch_plan(n, k, E, H, w->inter, w->shared_inter, specs, plan, st)) return rc;
  const size_t nk = (size_t)n * k;
  int8_t* xs0 = path == ER_PATH_TC ? reinterpret_cast<int8_t*>(ws + L.xs0) : nullptr;
  int8_t* xs1 = path == ER_PATH_TC ? reinterpret_cast<int8_t*>(ws + L.xs1) : nullptr;
  float* xscale = path == ER_PATH_TC ? reinterpret_cast<float*>(ws + L.xscale) : nullptr;
  if (int rc = launch_dispatch(io->h, io->h_dtype, idx32, topw, n, k, E, H, plan, perm_token, perm_w, pos_of, xs0, xs1,
                               xscale, st))
    return rc;
  launches += 2;
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
    tl.record_bytes = er_record_bytes(ER_FMT_INT8, H, w->inter, 0);
    tl.nk = (int)nk;
    tl.n = n;
    tl.tok_tile = tc_tok_tile(n);
    tl.mode = 0;
    tl.sched = 0;
    tl.b0_r = xs0;
    tl.b1_r = xs1;
    tl.xscale_r = xscale;
    tl.out_r = act_r;
    tl.out_s = act_s;
    tl.items_bound = b0;
    if (int rc = launch_tc_grouped(tl, st)) return rc;
    if (int rc = mark(3)) return rc;
    if (int rc = launch_slice_rows(act_r, ER_DTYPE_F32, (int)nk, w->inter, as0_r, as1_r, ascale_r, st)) return rc;
    if (int rc = launch_slice_rows(act_s, ER_DTYPE_F32, n, w->shared_inter, as0_s, as1_s, ascale_s, st)) return rc;
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
    tl.items_bound = b1;
    if (int rc = launch_tc_grouped(tl, st)) return rc;
    launches += 2;  // the two act slice launches; the two GEMMs are counted below
  } else if (path == ER_PATH_GEMV) {
    if (int rc = launch_gemv_grouped(ga, 0, 0, io->h, io->h_dtype, act_r, act_s, nullptr, nullptr, b0, st)) return rc;
    if (int rc = mark(3)) return rc;
    if (int rc = launch_gemv_grouped(ga, 1, 1, nullptr, ER_DTYPE_F32, act_r, act_s, y_r, y_s, b1, st)) return rc;
  } else {
    if (int rc = launch_gemm_simt_grouped(ga, 0, 0, io->h, io->h_dtype, act_r, act_s, nullptr, nullptr, b0, st))
      return rc;
    if (int rc = mark(3)) return rc;
    if (int rc = launch_gemm_simt_grouped(ga, 1, 1, nullptr, ER_DTYPE_F32, act_r, act_s, y_r, y_s, b1, st))
      return rc;
  }
  launches += 2 * per_stage;
  if (int rc = mark(4)) return rc;
  // K4
  if (int rc = launch_combine_plan(y_r, y_s, pos_of, idx32, n, k, H, plan, io->y, st)) return rc;
  launches += 1;
  if (io->launch_count) *io->launch_count += launches;
  return mark(5);
}
