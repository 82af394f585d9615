/*
 * expertrelay_b200.h -- C ABI of libexpertrelay_b200.so, the sm_100a (B200)
 * implementation of ExpertRelay's MoE-block hot path.
 *
 * Every entry point takes plain pointers and sizes (device pointers unless
 * stated), an optional CUDA stream (NULL = legacy default stream), returns
 * an int status (ER_OK = 0) and never allocates device memory: callers pass
 * any scratch space as a workspace pointer, sized by the matching *_bytes()
 * query. On failure er_last_error() returns a message for the calling
 * thread. Launches are asynchronous on `stream`; a kernel fault surfaces as
 * ER_ECUDA on a later call or synchronisation.
 *
 * Reference interfaces replaced (paths inside the ExpertRelay project):
 *   er_linear_f32      runtime/backends.py:57-59, 86-88   Backend.linear
 *   er_int8_linear     runtime/backends.py:47-51, 78-81   Backend.int8_linear
 *                      runtime/int8_linear.py:106-138     int8_linear()
 *   er_int4_linear     runtime/backends.py:53-55, 83-84   Backend.int4_linear
 *                      runtime/int4_linear.py:88-122      int4_linear()
 *   er_attention       runtime/backends.py:61-67, 90-95   Backend.attention
 *   er_router_topk     runtime/qwen_moe.py:303-308        router softmax + top-k
 *   er_dequant_int8    store/quantize.py:45-46            dequantize_rowwise_int8
 *   er_dequant_int4    store/int4.py:142-144              dequantize_groupwise_int4
 *   er_moe_block       runtime/qwen_moe.py:293-359        QwenMoe._moe
 *   er_record_*        store/layout.py:53-115, store/int4.py:165-244
 *                                                         expert record layouts
 *   er_cache_*         cache/expert_cache.py:92-402       CachedExpertSource (HBM slots)
 *   er_trace_*         runtime/expert_trace.py:34-135     ExpertTraceWriter records
 *   er_rms_norm, er_rope_kv, er_embed_int8
 *                      runtime/qwen_moe.py:121-138, 250-270, weights.py:62-64
 *                                                         decoder-layer norm, RoPE + KV cache, embedding
 *   er_store_*         store/unbuffered_io.py:135-149,    one aligned read per expert record
 *                      store/expert_reader.py:92-101      (ExpertStoreReader.read_into)
 */
#ifndef EXPERTRELAY_B200_H
#define EXPERTRELAY_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ER_API __attribute__((visibility("default")))
#else
#define ER_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define ER_OK 0
#define ER_EINVAL 1    /* bad argument: shape, alignment, null pointer, size */
#define ER_ECUDA 2     /* a CUDA runtime call or launch failed */
#define ER_ETIMEOUT 3  /* a bounded device-side wait gave up */
#define ER_ENOSPACE 4  /* workspace (or fixed scratch) too small */
#define ER_EIO 5       /* a file read failed or came up short */

/* ---- activation dtypes ------------------------------------------------- */
#define ER_DTYPE_F32 0
#define ER_DTYPE_BF16 1

/* ---- routed-expert record formats (store/layout.py, store/int4.py) ----- */
#define ER_FMT_INT8 0      /* [gate q][up q][down q][gate s f32][up s][down s][pad] */
#define ER_FMT_INT4 1      /* [gate p][up p][down p][gate s f16][up s][down s][pad], value = nibble - 8 */
#define ER_FMT_INT4_ZP 2   /* ER_FMT_INT4 + [gate z u8][up z][down z] after the scales, value = nibble - z */

/* ---- expert-matrix execution paths ------------------------------------- */
#define ER_PATH_AUTO 0     /* the tensor-core path for records in an arena of a format it takes; else
                              stream weights (GEMV) for small n, tiled GEMM otherwise */
#define ER_PATH_GEMV 1     /* weight-streaming grouped GEMV, any n (slow for large n) */
#define ER_PATH_GEMM 2     /* tiled grouped GEMM, fp32 FMA (exact-fp32 path) */
#define ER_PATH_TC 3       /* tcgen05 grouped GEMM: int8 weights (int4 records: codes q - z, unpacked in
                              shared memory) x two int8 activation slices, int32 accumulate (int4: per
                              scale group, the group scale applied to each partial sum) */

/* library identity / diagnostics */
ER_API int er_version(void);                 /* e.g. 100 = 0.1.0 */
ER_API const char* er_last_error(void);      /* message of the last failure on this thread */
ER_API int er_device_sm_count(int* sms);     /* SMs of the current device */

/* ---- record layout queries (store/layout.py:74-100, store/int4.py:194-220) ---- */
/* byte size of one padded expert record (a multiple of 4096) */
ER_API size_t er_record_bytes(int fmt, int hidden, int inter, int group);
/* byte offset inside a record of matrix `which` (0 gate, 1 up, 2 down);
 * part 0 = weights, 1 = scales, 2 = zero points (ER_FMT_INT4_ZP only) */
ER_API size_t er_record_offset(int fmt, int hidden, int inter, int group, int which, int part);

/* ---- Backend protocol ops (runtime/backends.py:44-67) ----------------------
 * x [m, in] with row stride ldx elements (>= in), y [m, out] contiguous.
 * bias may be NULL. All fp32 unless stated. */
ER_API int er_linear_f32(const float* x, long long ldx, const float* w, const float* bias, float* y,
                  int m, int out, int in, void* stream);
ER_API int er_int8_linear(const float* x, long long ldx, const int8_t* q, const float* scales,
                   const float* bias, float* y, int m, int out, int in, void* stream);
/* packed uint8 [out, in/2] (even input column in the low nibble), scales f16 bits
 * [out, in/group]; zeros (uint8 [out, in/group], 0..16) or NULL for the fixed 8 */
ER_API int er_int4_linear(const float* x, long long ldx, const uint8_t* packed, const uint16_t* scales_f16,
                   const uint8_t* zeros, int group, const float* bias, float* y, int m, int out,
                   int in, void* stream);
/* q [n, heads, d], keys/values [kv, heads, d], allowed [n, kv] (uint8 0/1) -> out [n, heads, d];
 * scores scaled by d^-0.5, softmax in fp32 */
ER_API int er_attention(const float* q, const float* keys, const float* values, const uint8_t* allowed,
                 float* out, int n, int kv, int heads, int d, void* stream);

/* ---- weight reconstruction (bit-exact fp32) ---------------------------- */
ER_API int er_dequant_int8(const int8_t* q, const float* scales, float* w, int rows, int cols, void* stream);
ER_API int er_dequant_int4(const uint8_t* packed, const uint16_t* scales_f16, const uint8_t* zeros, int group,
                    float* w, int rows, int cols, void* stream);

/* ---- router (runtime/qwen_moe.py:303-308) ----------------------------------
 * logits [n, E] fp32 -> top-k expert ids (largest first, exact ties to the lower id)
 * and their softmax probabilities (no renormalisation). idx64 or idx32 may be NULL. */
ER_API int er_router_topk(const float* logits, int n, int num_experts, int k, int64_t* idx64, int32_t* idx32,
                   float* probs_out, void* stream);
/* Routing straight from the tokens (runtime/qwen_moe.py:303-308): the router
 * logits h @ router_w^T at fp32 accuracy (h fp32 or bf16, [n, hidden];
 * router_w fp32 [num_experts, hidden]: fp32 FMA for up to 64 tokens, tensor
 * cores beyond, on exact tf32 hi/lo splits with fp32 accumulation), then
 * softmax + top-k as er_router_topk;
 * logits_out [n, E] optional. scratch: device memory of
 * er_route_scratch_bytes(n, num_experts) bytes for the K-slice partial
 * logits. */
ER_API size_t er_route_scratch_bytes(int n, int num_experts);
ER_API int er_route(const void* h, int h_dtype, int n, int hidden, const float* router_w, int num_experts, int k,
                    int norm_topk_prob, float* scratch, size_t scratch_bytes, float* logits_out, int32_t* idx32,
                    float* w_out, void* stream);

/* ---- the MoE block (runtime/qwen_moe.py:293-359) ------------------------- */
typedef struct er_moe_weights {
  int hidden;                  /* H (2048) */
  int num_experts;             /* E (60), <= 256 */
  int top_k;                   /* k (4), <= 8 */
  int inter;                   /* routed intermediate size I (1408) */
  int shared_inter;            /* shared-expert intermediate size (5632) */
  int expert_fmt;              /* ER_FMT_* of the routed-expert records */
  int group;                   /* int4 group size along the input dim (128), ignored for int8 */
  int norm_topk_prob;          /* 0 for Qwen1.5-MoE (weights are not renormalised) */
  const float* router_w;       /* [E, H] fp32 (mlp.gate.weight) */
  const float* shared_gate_w;  /* [H] fp32 (mlp.shared_expert_gate.weight) */
  const uint64_t* expert_records; /* DEVICE array [E] of record base addresses (4096-aligned) */
  const void* shared_record;   /* the shared expert as an ER_FMT_INT8 record with inter = shared_inter */
  /* optional (required by ER_PATH_TC): the routed records sit in one array of
   * arena_slots records of er_record_bytes() each starting here (e.g. the HBM
   * expert cache), and every expert_records[e] points at one of its slots */
  const void* record_arena;
  int arena_slots;
} er_moe_weights;

typedef struct er_moe_io {
  const void* h;               /* [n, H] activations, dtype h_dtype */
  int h_dtype;                 /* ER_DTYPE_F32 / ER_DTYPE_BF16 */
  int n;                       /* tokens */
  const float* logits_in;      /* optional [n, E]: use these router logits instead of h @ Wr^T */
  float* y;                    /* [n, H] fp32 output */
  float* logits_out;           /* optional [n, E] */
  int64_t* topk_idx_out;       /* optional [n, k] */
  float* topk_w_out;           /* optional [n, k] */
  int path;                    /* ER_PATH_* */
  /* optional instrumentation (NULL to skip): ER_MOE_STAGES + 1 cudaEvent_t handles,
   * recorded on the stream before the router and after each stage (router, plan,
   * gate/up, down, combine), so stage i took elapsed(events[i], events[i + 1]) */
  void* const* stage_events;
  int* launch_count;           /* optional: incremented by the number of kernels launched */
} er_moe_io;

#define ER_MOE_STAGES 5        /* router, plan, gate/up, down, combine */

ER_API size_t er_moe_workspace_bytes(const er_moe_weights* w, int n, int path);
/* er_moe_block for callers that cannot allocate device memory (no counterpart
 * in the reference): same weights and io, no workspace argument. The scratch
 * is a fixed 8 MiB device array inside the library, held on each GPU from the
 * first call there until exit; batches needing more (er_moe_workspace_bytes)
 * fail with ER_ENOSPACE. At Qwen1.5-MoE-A2.7B shapes up to 96 tokens fit on
 * the GEMV / SIMT GEMM paths and up to 64 on the tensor-core path (which
 * ER_PATH_AUTO picks for int8 records in an arena: its int8 operand slices
 * need room). The
 * first call on a device sets up the array's address: make it before any
 * stream capture. All calls share the array, so calls that overlap on the GPU
 * race and must be serialised by the caller. */
ER_API int er_moe_block_noalloc(const er_moe_weights* w, const er_moe_io* io, void* stream);
/* Test hook of the tensor-core path (no counterpart in the reference, whose
 * CPU path has no device waits): every later er_moe_block call bounds each
 * mbarrier wait of its tensor-core kernels by wait_ns (0: the default, 2 s)
 * and, with stall = 1 (gate/up) or 2 (down), the int8 kernel of that step
 * never completes its last work item's accumulator, so that item's epilogue
 * wait runs out: the kernel returns, the plan's error bit 8 is set and the
 * block writes NaN rows. (0, 0) restores normal operation. Process-wide,
 * not thread-safe; for tests of the bounded-wait error path only. */
ER_API int er_tc_test_stall(unsigned long long wait_ns, int stall);
/* The error bits the last er_moe_block call on this workspace (same w, n and
 * path) left in its plan, read after the stream's work: 0 when it ran clean;
 * 1 an expert id out of range, 2 inconsistent routing counts, 4 a record
 * outside the arena, 8 a tensor-core wait gave up. Any of them made the
 * block write NaN rows. Synchronises the stream. No counterpart in the
 * reference (its CPU path raises instead). */
ER_API int er_moe_error_bits(const er_moe_weights* w, int n, int path, const void* workspace, int* bits,
                             void* stream);
ER_API int er_moe_block(const er_moe_weights* w, const er_moe_io* io, void* workspace, size_t workspace_bytes,
                 void* stream);

/* ---- the block in parts, for expert parallelism ---------------------------
 * One rank holds experts [lo, hi) of every layer; tokens stay on their rank.
 * The reference runs on one process (runtime/qwen_moe.py:340-359); these
 * split its routed sum and shared expert so that routed rows can travel to
 * the rank holding their expert (one collective each way) and back. */
typedef struct er_moe_rows_io {
  const void* x;               /* [m, H] rows, dtype x_dtype */
  int x_dtype;
  int m;
  const int32_t* expert;       /* [m] expert of each row: 0 .. num_experts-1 of `w` (this rank's experts) */
  const float* weight;         /* [m] routing weight of each row */
  void* y;                     /* [m, H] = weight * down(silu(gate x) * up x) (qwen_moe.py:345-349), dtype y_dtype */
  int path;                    /* ER_PATH_* */
  int* launch_count;           /* optional */
  int y_dtype;                 /* ER_DTYPE_F32 (0, the default) or ER_DTYPE_BF16: results rounded to bf16 halve
                                  the bytes sent back to the tokens' ranks */
} er_moe_rows_io;
/* routed experts on pre-routed rows (w->router_w and the shared weights unused) */
ER_API size_t er_moe_rows_workspace_bytes(const er_moe_weights* w, int m, int path);
ER_API int er_moe_rows(const er_moe_weights* w, const er_moe_rows_io* io, void* workspace, size_t workspace_bytes,
                       void* stream);
/* y [n, H] = sigmoid(h . w_g) * shared(h) (qwen_moe.py:353-359; w->router_w and
 * the routed records unused) */
ER_API size_t er_moe_shared_workspace_bytes(const er_moe_weights* w, int n, int path);
ER_API int er_moe_shared(const er_moe_weights* w, const void* h, int h_dtype, int n, float* y, int path,
                         void* workspace, size_t workspace_bytes, void* stream);
/* y[t] = sum over t's k slots in ascending expert id (idx [n, k]) of
 * y_rows[pos_of[t * k + j]] (+ y_shared[t] when not NULL): the reference's
 * np.add.at order (qwen_moe.py:340-349) and its final sum (:359), in fp32;
 * y_rows in rows_dtype (ER_DTYPE_F32 or ER_DTYPE_BF16) */
ER_API int er_moe_combine(const void* y_rows, int rows_dtype, const int32_t* pos_of, const int32_t* idx,
                          const float* y_shared, int n, int k, int hidden, float* y, void* stream);

/* ---- expert-parallel exchange buffers -------------------------------------
 * owner[e] = rank holding global expert e, local[e] = its index there. */
/* counts[r] = (token, slot) pairs of idx [n, k] whose expert lives on rank r */
ER_API int er_ep_count(const int32_t* idx, int n, int k, const int32_t* owner, int num_experts, int ranks,
                       int32_t* counts, void* stream);
/* Packs the send buffers, destination rank by destination rank: rank r's
 * rows occupy [offsets[r], offsets[r] + counts[r]) (offsets: device, the
 * exclusive prefix of er_ep_count's counts). For pair (t, j) at position p:
 * x_send[p] = h[t] (dtype h_dtype), expert_send[p * meta_stride] =
 * local[idx[t, j]], weight_send[p * meta_stride] = w[t, j], pos_of[t * k + j]
 * = p (meta_stride 2 with weight_send = expert_send + 1 interleaves the id
 * and the weight's bits, so both travel in one exchange). cursor: device
 * scratch of `ranks` ints. Rows of one destination are in no particular
 * order. */
ER_API int er_ep_pack(const void* h, int h_dtype, int hidden, const int32_t* idx, const float* w, int n, int k,
                      const int32_t* owner, const int32_t* local, int num_experts, int ranks, const int32_t* offsets,
                      int32_t* cursor, void* x_send, int32_t* expert_send, float* weight_send, int meta_stride,
                      int32_t* pos_of, void* stream);

/* ------------------------------------------------------------------------
 * HBM expert cache: replaces CachedExpertSource (cache/expert_cache.py:92-402).
 *
 * A fixed number of slots, each one store record (record_bytes), in one
 * device arena; keys are (layer, expert). Records come from pinned host
 * memory (er_cache_set_source) by cudaMemcpyAsync on the cache's own copy
 * stream, each fill followed by the slot's ready event; a stream that uses a
 * slot waits on that event, so an expert whose copy is still in flight is
 * waited for, never copied twice (expert_cache.py:271-279). Eviction takes the
 * least recently used ready slot that the current layer does not hold and
 * that is not pinned (expert_cache.py:172-191); a refill waits on the slot's
 * last-use event, so kernels still reading the old record finish first.
 * Not thread-safe per cache: one host thread drives it, like the reference's
 * forward pass.
 * ---------------------------------------------------------------------- */
typedef struct er_cache er_cache;

/* cumulative counters, the fields of SourceStats (runtime/weights.py:170-193) */
typedef struct er_cache_stats {
  long long loads;                     /* experts handed to the forward pass (er_cache_acquire) */
  long long bytes_read;                /* bytes of demand fills */
  long long demand_reads;              /* fills started by er_cache_acquire */
  long long cache_hits;                /* resident, not from an unused prefetch */
  long long prefetch_hits;             /* resident thanks to a finished prefetch */
  long long prefetch_waits;            /* a prefetch's copy was still in flight: waited on it */
  long long prefetches_issued;
  long long prefetch_reads;            /* prefetch copies seen complete */
  long long prefetch_bytes;
  long long prefetches_wasted;         /* prefetched, evicted before any use */
  long long prefetches_cancelled;      /* always 0: a copy in the stream is not withdrawn */
  long long prefetches_skipped_full;   /* no evictable slot */
  long long prefetches_skipped_budget; /* over max_new_reads */
} er_cache_stats;

#define ER_CACHE_DRY 1 /* bookkeeping only: no device memory, copies or events; fills complete at once */

#define ER_SLOT_FREE 0
#define ER_SLOT_LOADING 1
#define ER_SLOT_READY 2

/* slots >= min_free_slots (else ER_ENOSPACE, the reference's CacheTooSmall,
 * expert_cache.py:104-113). arena: caller-owned device memory of
 * slots * record_bytes, 256-byte aligned, or NULL to let the cache allocate it.
 * record_bytes: a multiple of 256. */
ER_API int er_cache_create(int slots, size_t record_bytes, int min_free_slots, void* arena, int flags,
                           er_cache** out);
ER_API int er_cache_destroy(er_cache* c);
/* the arena's base address, slot count and record size; the copy stream (cudaStream_t) */
ER_API int er_cache_info(const er_cache* c, void** arena, int* slots, size_t* record_bytes, void** copy_stream);
/* host_records[layer * experts + expert]: pinned host address of that record */
ER_API int er_cache_set_source(er_cache* c, int layers, int experts, const void* const* host_records);
/* load now and never evict (the reference's `pinned`, expert_cache.py:150-158);
 * ER_ENOSPACE when fewer than min_free_slots slots would stay unpinned */
ER_API int er_cache_pin(er_cache* c, int layer, int expert);
/* The forward pass's loads for one layer (expert_cache.py:203-262, batched):
 * makes every listed expert resident (starting fills as needed), makes
 * `stream` wait for their copies, and writes each record's device address to
 * records_out[i]. The slots stay held until er_cache_end_layer(layer).
 * ER_ENOSPACE when no slot can be freed (CacheTooSmall). */
ER_API int er_cache_acquire(er_cache* c, int layer, const int* experts, int count, void* stream,
                            uint64_t* records_out);
/* Background loads (expert_cache.py:264-294): touches the (layer, expert)
 * pairs in keep[2 * keep_count] and each listed expert already resident;
 * starts at most max_new_reads fills (< 0: no limit) into free or evictable
 * slots, counting skips like the reference. */
ER_API int er_cache_prefetch(er_cache* c, int layer, const int* experts, int count, const int* keep, int keep_count,
                             int max_new_reads);
/* done with `layer` for this call (expert_cache.py:296-305): releases its held
 * slots; their last use is recorded on `stream` for later refills */
ER_API int er_cache_end_layer(er_cache* c, int layer, void* stream);
/* Change the slot count between forward calls (expert_cache.py:307-354):
 * waits for copies in flight and for kernels using the slots, keeps the pinned
 * experts and then the most recently used ones, and moves them into a new
 * arena of `slots` slots: `new_arena` (caller-owned from then on; the caller
 * frees the old one after the call) or, when NULL, one the cache allocates
 * (only if it allocated the old one). ER_ENOSPACE (nothing changed) when the
 * pinned experts plus min_free_slots would not fit; ER_EINVAL while a layer
 * holds slots. */
ER_API int er_cache_resize(er_cache* c, int slots, void* new_arena, int* slots_out);
/* slot and ER_SLOT_* state of a key (slot -1 when absent); polls its copy */
ER_API int er_cache_lookup(er_cache* c, int layer, int expert, int* slot, int* state);
ER_API int er_cache_stats_get(er_cache* c, er_cache_stats* out);

/* ---- expert-usage trace (runtime/expert_trace.py) ----
 * Record bytes of one (token, layer) record (record_dtype, expert_trace.py:
 * 34-65: 10 + 7 top_k + 4 num_experts); 0 when num_experts >= 255 (u8 ids)
 * or top_k is outside 1..8. */
ER_API size_t er_trace_record_bytes(int num_experts, int top_k);
/* One layer's records of a forward call (ExpertTraceWriter.layer,
 * expert_trace.py:114-135), written on the device into `records` (the call's
 * n * num_layers records, token major): positions / tokens [n] u32, logits
 * [n, E] f32 (stored f16), experts [n, k] int64 (experts_are_i64) or int32,
 * weights [n, k] f32, fate_logits [n, E] f32 or NULL (the Fate logits given
 * with the previous layer: stored f16 and their top-k; NULL: NO_EXPERT and
 * zeros). prev_in / prev_out: [num_layers, k] u8 previous-token experts
 * before and after this call (distinct buffers unless n == 1). */
ER_API int er_trace_pack_layer(void* records, int n, int num_layers, int layer, const uint32_t* positions,
                               const uint32_t* tokens, int phase, const float* logits, const void* experts,
                               int experts_are_i64, const float* weights, const float* fate_logits,
                               const uint8_t* prev_in, uint8_t* prev_out, int num_experts, int top_k, void* stream);

/* ---- the decoder layer's other parts (runtime/qwen_moe.py) ----
 * x_out = x + add (when add is not NULL; x_out may be x), h = weight * x_out /
 * sqrt(mean(x_out^2) + eps) per row of `hidden` fp32 values (rms_norm, :121-123,
 * with the residual add before it fused). */
ER_API int er_rms_norm(const float* x, const float* add, const float* weight, float eps, int n, int hidden,
                       float* x_out, float* h, void* stream);
/* RoPE (rope_tables and the rotation, :126-138, 255-256; inv_freq = 1 /
 * theta^(2i/d)) for positions pos0 .. pos0 + n - 1. qkv: n rows (stride ld
 * floats) of the fused projection [q heads*d | k kv_heads*d | v kv_heads*d];
 * the rotated q goes to q_out [n, heads, d], the rotated k and the v to rows
 * pos0.. of the layer's caches [max_seq, kv_heads, d] (:264-270; ER_EINVAL
 * when pos0 + n > max_seq, like the reference's ValueError). */
ER_API int er_rope_kv(const float* qkv, long long ld, float* q_out, int n, int heads, int kv_heads, int head_dim,
                      int pos0, float theta, float* k_cache, float* v_cache, int max_seq, void* stream);
/* out[t] = q[ids[t]] * scales[ids[t]] (Int8Matrix.dequantized_rows,
 * runtime/weights.py:62-64); an id outside [0, vocab) sets *bad and a NaN row */
ER_API int er_embed_int8(const int8_t* q, const float* scales, long long vocab, int hidden, const int64_t* ids, int n,
                         float* out, int* bad, void* stream);

/* ---- expert store reads (store/unbuffered_io.py, store/expert_reader.py) ----
 * experts.bin opened for reads that bypass the page cache (O_DIRECT; with
 * ER_STORE_BUFFERED, or on a filesystem without O_DIRECT, plain reads). A
 * read is offset / size / destination all multiples of 4096 (ER_EINVAL
 * otherwise, "unaligned unbuffered read" as the reference), into HOST memory
 * (normally pinned), and fails with ER_EIO on an I/O error or a short read. */
typedef struct er_store er_store;
#define ER_STORE_BUFFERED 1
ER_API int er_store_open(const char* path, int flags, er_store** out);
ER_API int er_store_close(er_store* s);
ER_API int er_store_info(const er_store* s, uint64_t* file_bytes, int* direct);
ER_API int er_store_read(er_store* s, uint64_t offset, uint64_t nbytes, void* dst);
/* count reads of nbytes each (offsets[i] -> dsts[i]) on up to `threads` threads;
 * on a failed read, *failed (when given) receives its index i, else -1, so the
 * caller can name the expert whose read failed (cache/expert_cache.py:281-282) */
ER_API int er_store_read_many(er_store* s, int count, const uint64_t* offsets, uint64_t nbytes, void* const* dsts,
                              int threads, int* failed);

#ifdef __cplusplus
}
#endif

#endif /* EXPERTRELAY_B200_H */
