/*
 * specfit_b200 — C ABI of the B200 (sm_100a) MoE verification path.
 *
 * Every entry point takes plain device pointers, sizes, dtype codes and a
 * cudaStream_t passed as `void*` (NULL = the legacy default stream).  None of
 * them allocates device memory except sf_ipc_alloc (the shared region of the
 * peer-memory exchange): scratch buffers ("workspace") are passed in by the
 * caller.  All device work is enqueued asynchronously on the given
 * stream; the return value is a status code (SF_OK on success), and on
 * failure sf_last_error() returns a message for the calling thread.
 *
 * Interface map to the SpecFit reference (paths inside the SpecFit tree;
 * "transformers/..." = transformers/models/qwen3_moe/modeling_qwen3_moe.py):
 *   sf_router_topk        Qwen3MoeTopKRouter.forward            transformers/...:263-272
 *   sf_moe_dispatch       grouping in Qwen3OffloadedExperts     src/specfit/runtime/qwen3_offloaded_experts.py:111-122,173-178
 *   sf_moe_gather         hidden_states[route_tokens], weights  src/specfit/runtime/qwen3_offloaded_experts.py:189-190
 *   sf_grouped_swiglu     _expert_forward + mul_(w), per expert src/specfit/runtime/qwen3_offloaded_experts.py:38-62,126-138,194-198
 *   sf_grouped_swiglu_gathered  the gather (:189-190) + sf_grouped_swiglu in one call
 *   sf_moe_combine        index_add_ reduction                  src/specfit/runtime/qwen3_offloaded_experts.py:144-163,200-202
 *   sf_slot_fill_batch    slot.tensor.copy_(source)             src/specfit/runtime/gpu_expert_cache.py:556-561
 *   sf_tree_attention     SDPA under the tree mask              transformers/...:156-195 with the mask of
 *                                                               src/specfit/runtime/eagle3_types.py:450-473
 *   sf_specfit_select     exact_specfit_selection               src/specfit/specfit_exact.py:58-94
 *   sf_ep_*               (none: the reference is single-GPU, scripts/run_specfit_main_comparison.py:465)
 *   sf_add_rmsnorm        residual add + Qwen3MoeRMSNorm        transformers/...:Qwen3MoeRMSNorm.forward,
 *                                                               Qwen3MoeDecoderLayer.forward (residual adds)
 *   sf_qk_norm_rope       q_norm/k_norm + apply_rotary_pos_emb  transformers/...:Qwen3MoeAttention.forward
 *                         + cache update (write k, v rows)
 *   sf_kv_compact         _compact_tree_cache                   src/specfit/runtime/eagle3_tree.py:833-858
 *   sf_logsoftmax_topk    log_softmax + topk of a drafter level src/specfit/runtime/eagle3_tree.py:611-803
 *   sf_draft_level        one level of the candidate-pool build  src/specfit/runtime/eagle3_tree.py:611-803
 *   sf_rope_rows          rotary cos/sin rows                    transformers/...:Qwen3MoeRotaryEmbedding
 *   sf_linear_bf16        F.linear (q|k|v, o, lm_head, drafter)  transformers/...:Qwen3MoeAttention.forward,
 *                                                               Qwen3MoeForCausalLM.forward (lm_head)
 *                                                               (candidate-pool expansion)
 */
#ifndef SPECFIT_B200_H_
#define SPECFIT_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SF_API __attribute__((visibility("default")))
#else
#define SF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define SF_OK 0
#define SF_ERR_INVALID_ARGUMENT 1 /* maps to ValueError in the Python layer */
#define SF_ERR_CUDA 2             /* a CUDA runtime call failed */
#define SF_ERR_UNSUPPORTED 3      /* shape/dtype/device not supported */
#define SF_ERR_WORKSPACE 4        /* workspace too small */
#define SF_ERR_STATE 5            /* object state forbids the call (maps to RuntimeError) */
#define SF_ERR_NO_SLOT 6          /* every expert-cache slot is leased (NoEvictableSlotError) */

/* Element types. */
#define SF_DTYPE_F32 0
#define SF_DTYPE_BF16 1

/* Reduction order of sf_moe_combine. */
#define SF_REDUCE_MODEL_DTYPE 0 /* sequential adds rounded to the model dtype (reference index_add_) */
#define SF_REDUCE_F32 1         /* fp32 accumulation, one rounding at the end */

/* Implementation choice of sf_grouped_swiglu_ex. */
#define SF_SWIGLU_AUTO 0    /* tcgen05 path when the shape allows it, else SIMT */
#define SF_SWIGLU_SIMT 1    /* CUDA-core kernel, any shape, f32 or bf16 */
#define SF_SWIGLU_TCGEN05 2 /* tcgen05/TMEM + TMA kernel: bf16, H%128==0, I%64==0, <= 1024 experts */

/* Message describing the last failure on the calling thread ("" if none). */
SF_API const char* sf_last_error(void);

/* ABI version of this library (bumped on any signature change). */
SF_API int sf_abi_version(void);

/*
 * Sticky device-side status of the current device: 0, or the code of the first
 * barrier wait of a tcgen05 kernel (grouped SwiGLU, projection GEMM, tree
 * attention) that gave up after its one-second limit (each kernel's site
 * codes); that kernel then skipped its remaining work and returned.
 * Synchronous: reads (and with reset != 0 clears) the words.
 * No reference counterpart; the reference's GPU work is PyTorch library calls.
 */
SF_API int sf_device_status(int* status, int reset);

/*
 * Router: logits = hidden[T,H] @ router_weight[E,H]^T, rounded once to the
 * model dtype from an exact (fp64) dot product; probs = softmax(logits) in
 * fp32; top_k experts by (logit desc, expert id asc); weights = the top-k
 * probs, divided by their sum when norm_topk_prob.
 * Replaces Qwen3MoeTopKRouter.forward (transformers/...:263-272), which returns
 * (probs, weights, indices).  `logits_out` (nullable) receives the rounded
 * logits in the model dtype.  Requires E <= 1024, top_k <= 32, top_k <= E.
 * `workspace` must hold sf_router_topk_workspace_bytes(T, E) bytes.
 */
SF_API size_t sf_router_topk_workspace_bytes(int64_t tokens, int num_experts);
SF_API int sf_router_topk(const void* hidden, const void* router_weight, int dtype, int64_t tokens,
                   int hidden_size, int num_experts, int top_k, int norm_topk_prob,
                   float* probs, float* topk_weights, int64_t* topk_index, void* logits_out,
                   void* workspace, size_t workspace_bytes, void* stream);

/*
 * Allocation-free router: same contract and results as sf_router_topk, but it
 * takes no workspace and allocates nothing.  It is for callers that cannot
 * obtain device memory where they route: plugins loaded into a serving
 * engine that reserves the GPU's memory for its own pools at start-up (a
 * cudaMalloc there fails or fragments the engine's pool), hosts that bind
 * this library through a plain C FFI and have no device allocator to carve
 * a workspace from, and latency-critical paths where cudaMalloc's implicit
 * device-wide synchronisation would stall every other stream.  Its scratch
 * (the fp32 logits between the two router passes) is a 2 MiB array compiled
 * into the library, which every GPU that loads the library holds until the
 * process exits.
 *   - tokens * num_experts must not exceed sf_router_topk_noalloc_max_elems()
 *     (2^19); larger calls fail with SF_ERR_WORKSPACE and launch nothing.
 *   - The first call on a device looks up the array's device address with
 *     cudaGetSymbolAddress (a runtime query, no allocation) and keeps it for
 *     that device; make that first call before any stream capture.  The
 *     address belongs to the device's primary context: after
 *     cudaDeviceReset the kept address is stale, so do not call this entry
 *     point again in a process that has reset the device.
 *   - All calls on a device share the array: calls that may overlap on the
 *     GPU (different streams without ordering) race and must not be issued.
 *     Nothing in the array needs to start at zero; each call overwrites every
 *     element it later reads, and the array keeps the last call's contents.
 * No counterpart in the reference (its router is a PyTorch module that
 * allocates through the caching allocator).
 */
SF_API int64_t sf_router_topk_noalloc_max_elems(void);
SF_API int sf_router_topk_noalloc(const void* hidden, const void* router_weight, int dtype,
                                  int64_t tokens, int hidden_size, int num_experts, int top_k,
                                  int norm_topk_prob, float* probs, float* topk_weights,
                                  int64_t* topk_index, void* logits_out, void* stream);

/*
 * Dispatch: stable grouping of the T*K routes by expert id.
 *   counts[E], offsets[E+1] (exclusive prefix of counts),
 *   sorted_pos[T*K]: route positions t*K+k in ascending (expert, position)
 *     order == torch.sort(top_k_index.reshape(-1), stable=True).indices
 *     (qwen3_offloaded_experts.py:173); its per-expert blocks are the token
 *     groups of torch.where(top_k_index == e) (:120-122);
 *   inv_pos[T*K]: inverse permutation (route position -> sorted row);
 *   active[E]: experts with a non-empty group, ascending, -1 padded;
 *   num_active[1].
 * *error_flag (device int32) is set to 1 if an expert id lies outside
 * [0, E) (that route is dropped), else to 0.  Requires E <= 1024.
 */
SF_API int sf_moe_dispatch(const int64_t* topk_index, int64_t tokens, int top_k, int num_experts,
                    int32_t* counts, int32_t* offsets, int32_t* sorted_pos, int32_t* inv_pos,
                    int32_t* active, int32_t* num_active, int32_t* error_flag, void* stream);
/* sf_moe_dispatch that also adds num_active to *active_total (device int64,
 * optional: NULL skips it) -- a running count of expert hits kept on the
 * device without a separate launch. */
SF_API int sf_moe_dispatch_ex(const int64_t* topk_index, int64_t tokens, int top_k, int num_experts,
                              int32_t* counts, int32_t* offsets, int32_t* sorted_pos,
                              int32_t* inv_pos, int32_t* active, int32_t* num_active,
                              int32_t* error_flag, int64_t* active_total, void* stream);

/*
 * Gather: hidden_sorted[i,:] = hidden[sorted_pos[i] / K, :] and
 * weights_sorted[i] = (float) topk_weights.flat[sorted_pos[i]]
 * (qwen3_offloaded_experts.py:189-190).  weight_dtype may differ from dtype.
 */
SF_API int sf_moe_gather(const void* hidden, int dtype, int64_t tokens, int hidden_size,
                  const void* topk_weights, int weight_dtype, int top_k,
                  const int32_t* sorted_pos, void* hidden_sorted, float* weights_sorted,
                  void* stream);

/*
 * Grouped SwiGLU over the active experts of one layer.  For every active
 * expert e (active[0..*num_active)) and its rows r in [offsets[e], offsets[e+1]):
 *   g,u   = hidden_sorted[r] @ gate_e^T, @ up_e^T        (rounded to dtype)
 *   act   = silu(g) * u                                  (each op rounded)
 *   out   = act @ down_e^T                               (rounded to dtype)
 *   out_sorted[r] = round(out * weights_sorted[r])
 * Expert e's packed weights [gate(I*H) | up(I*H) | down(H*I)] start at
 * slot_storage + expert_slot[e] * slot_stride_elems (elements of dtype).
 * act_workspace holds rows*I elements of dtype.
 * Replaces _expert_forward (qwen3_offloaded_experts.py:38-62) and the
 * weighting mul_ (:132-138, :198), for all experts of a layer in one call.
 */
SF_API int sf_grouped_swiglu(const void* hidden_sorted, const float* weights_sorted, int dtype,
                      const int32_t* offsets, const int32_t* active, const int32_t* num_active,
                      const int32_t* expert_slot, const void* slot_storage, int64_t slot_count,
                      int64_t slot_stride_elems, int num_experts, int hidden_size,
                      int intermediate_size, int64_t rows, void* act_workspace, void* out_sorted,
                      void* stream);
SF_API int sf_grouped_swiglu_ex(const void* hidden_sorted, const float* weights_sorted, int dtype,
                         const int32_t* offsets, const int32_t* active, const int32_t* num_active,
                         const int32_t* expert_slot, const void* slot_storage, int64_t slot_count,
                         int64_t slot_stride_elems, int num_experts, int hidden_size,
                         int intermediate_size, int64_t rows, void* act_workspace,
                         void* out_sorted, int impl, void* stream);

/*
 * sf_moe_gather + sf_grouped_swiglu (tcgen05) in one call, without the
 * gathered copy: sorted row r reads hidden[sorted_pos[r] / top_k] (bf16
 * [tokens, hidden_size]) by TMA gather4 straight into the MMA tiles and is
 * weighted by topk_weights[sorted_pos[r]] (fp32 [tokens * top_k]); rows =
 * tokens * top_k.  Results equal the two calls bit for bit.  Returns
 * SF_ERR_UNSUPPORTED (no message) when the tcgen05 kernel does not apply
 * (not bf16-shaped as sf_grouped_swiglu's tcgen05 path requires, unaligned
 * buffers, or not an sm_100 device); the caller then gathers and calls
 * sf_grouped_swiglu.
 * Replaces the gather of qwen3_offloaded_experts.py:189-190 and
 * _expert_forward + mul_(w) (:38-62, :198) for all experts of a layer.
 */
SF_API int sf_grouped_swiglu_gathered(const void* hidden, int64_t tokens, const float* topk_weights,
                                      int top_k, const int32_t* sorted_pos, const int32_t* offsets,
                                      const int32_t* active, const int32_t* num_active,
                                      const int32_t* expert_slot, const void* slot_storage,
                                      int64_t slot_count, int64_t slot_stride_elems, int num_experts,
                                      int hidden_size, int intermediate_size, void* act_workspace,
                                      void* out_sorted, void* stream);

/*
 * Combine: out[t,:] = sum over the token's K routes of out_sorted[inv_pos[t*K+k],:],
 * added in ascending expert_rank[expert] (ties: ascending k) order.
 * expert_rank == NULL gives the canonical ascending-expert-id order
 * (ReductionMode.CANONICAL, qwen3_offloaded_experts.py:155-163, :200-202);
 * the rank of each expert in the execution order gives ARRIVAL_ORDER (:144-149).
 * reduce = SF_REDUCE_MODEL_DTYPE reproduces index_add_'s rounding after every
 * add; SF_REDUCE_F32 accumulates in fp32.  out may not alias out_sorted.
 */
SF_API int sf_moe_combine(const void* out_sorted, int dtype, const int32_t* inv_pos,
                   const int64_t* topk_index, const int32_t* expert_rank, int num_experts,
                   int64_t tokens, int top_k, int hidden_size, int reduce, void* out,
                   void* stream);

/*
 * Slot fill: n host->device copies dst[i] <- src[i] (bytes[i] each) on
 * `stream`, one cudaMemcpyAsync per copy, in order.  Sources should be pinned
 * for the copy to be asynchronous (gpu_expert_cache.py:556-561).
 */
SF_API int sf_slot_fill_batch(void* const* dst, const void* const* src, const size_t* bytes, int n,
                       void* stream);

/*
 * Expert-slot cache manager (host bookkeeping + fills).  Replaces the slot
 * bookkeeping of GpuExpertCache (src/specfit/runtime/gpu_expert_cache.py:
 * 196-266 acquire, 495-541 victim choice, 543-609 fills and their
 * publication, 684-718 release).  One manager per cache: `slots` device
 * slots of `slot_bytes` each at `storage`, `experts` page-locked host
 * sources (source order), fills on `copy_stream`.  Experts are addressed by
 * their index in source order; ready events are cudaEvent_t handles owned by
 * the caller (one fresh, already-created event per potential miss), recorded
 * here right behind each fill.  Use guards are events owned by the manager.
 *
 * sf_cache_acquire processes `experts[0..n)` in order, as n single acquires:
 *   SF_CACHE_ACQUIRE       LRU victim among unleased slots (the fill queues
 *                          behind the victim's readers); stops at the first
 *                          expert with no unleased slot: SF_ERR_NO_SLOT if
 *                          nothing was granted, else the grants so far;
 *   SF_CACHE_NONBLOCKING   LRU victim among slots whose fill and readers are
 *                          done, else not granted;
 *   SF_CACHE_RESIDENT_ONLY hits and joins only;
 *   SF_CACHE_PROBABILITY   as NONBLOCKING with the lowest-probability victim
 *                          below the incoming expert's (`probabilities`
 *                          indexed by expert).
 * Each grant holds a lease (touched now unless `defer_touch`).  Leases are
 * checked by (expert, slot, generation); sf_cache_wait orders `stream` after
 * the slot's fill, sf_cache_release records a use guard on every stream that
 * used the slot.  Not thread-safe across managers sharing a copy stream.
 * No counterpart in the reference's ABI (the reference is Python).
 */
#define SF_CACHE_ACQUIRE 0
#define SF_CACHE_NONBLOCKING 1
#define SF_CACHE_RESIDENT_ONLY 2
#define SF_CACHE_PROBABILITY 3
#define SF_GRANT_NONE 0
#define SF_GRANT_HIT 1
#define SF_GRANT_JOIN 2
#define SF_GRANT_MISS 3
#define SF_CACHE_RESET_COLD 0    /* empty slots, generations and counters zeroed */
#define SF_CACHE_RESET_DISCARD 1 /* empty slots, generations advanced, counters kept */
#define SF_SLOT_EXPERT 0
#define SF_SLOT_GENERATION 1
#define SF_SLOT_STAMP 2
#define SF_SLOT_READY 3
#define SF_SLOT_GUARDS 4

typedef struct {
  int32_t kind;        /* SF_GRANT_* */
  int32_t slot;
  uint32_t generation;
  int32_t victim;      /* evicted expert index, -1 none */
  int64_t submission;  /* fill submission number (miss, join), else -1 */
  uint64_t ready_event;
} SfCacheGrant;

typedef struct {
  int64_t h2d_submissions, resident_hits, inflight_joins, evictions, pending_use_guards;
  int64_t sequence, submission_sequence, state_version, outstanding_fills;
} SfCacheCounters;

typedef struct {
  int32_t expert;      /* -1 empty */
  uint32_t generation;
  int32_t leases;
  int32_t guards;          /* use guards held */
  int64_t stamp;           /* last-used sequence */
  uint64_t ready_event;
  int32_t guards_pending;  /* of which not yet complete */
  int32_t pad;
} SfCacheSlot;

typedef struct {
  int32_t expert, slot;
  uint32_t generation;
  int32_t done;
  int64_t submission;
  uint64_t ready_event;
} SfCacheFill;

SF_API int sf_cache_create(int slots, int experts, void* storage, size_t slot_bytes,
                           const void* const* sources, void* copy_stream, void** out);
SF_API void sf_cache_destroy(void* cache);
SF_API int sf_cache_set_copy_stream(void* cache, void* stream);
SF_API int sf_cache_acquire(void* cache, const int32_t* experts, int n, int mode, int defer_touch,
                            const uint64_t* fresh_events, const float* probabilities,
                            SfCacheGrant* grants, int* granted);
SF_API int sf_cache_touch(void* cache, int32_t expert, int32_t slot, uint32_t generation);
SF_API int sf_cache_check(void* cache, int32_t expert, int32_t slot, uint32_t generation);
SF_API int sf_cache_wait(void* cache, int32_t expert, int32_t slot, uint32_t generation, void* stream,
                         int touch);
SF_API int sf_cache_release(void* cache, int32_t expert, int32_t slot, uint32_t generation,
                            const uint64_t* streams, int n_streams);
/* refresh: bit 0 publishes completed fills, bit 1 drops completed use guards. */
SF_API int sf_cache_state(void* cache, int refresh, SfCacheCounters* counters, SfCacheSlot* slots,
                          int32_t* where, int32_t* home, int64_t* fill_seq);
SF_API int sf_cache_fills(void* cache, SfCacheFill* out, int capacity, int* n);
SF_API int sf_cache_quiescent(void* cache, int* quiescent);
/* table[e] = slot of expert e when every expert is resident and slots >= experts. */
SF_API int sf_cache_resident_table(void* cache, int32_t* table, int* complete);
SF_API int sf_cache_add_hits(void* cache, int64_t hits);
SF_API int sf_cache_reset(void* cache, int mode);
SF_API int sf_cache_slot_edit(void* cache, int32_t slot, int field, int64_t value);
SF_API int sf_cache_forget(void* cache, int which);
SF_API int sf_cache_set_version(void* cache, int64_t version);
SF_API int sf_cache_export(void* cache, void* image, size_t capacity, size_t* needed);
SF_API int sf_cache_import(void* cache, const void* image, size_t size);
/* Hand-over with the device-resident directory: slot experts (-1 empty),
 * generations, last-use stamps, expert->slot of resident experts, the LRU
 * clock and the counters {h2d, hits, joins, evictions}.  Export needs no
 * active lease and no fill in flight; adopt installs a state whose assigned
 * slots all hold published experts. */
SF_API int sf_cache_export_slots(void* cache, int32_t* slot_expert, int32_t* slot_gen, int64_t* slot_stamp,
                                 int32_t* expert_slot, int64_t* clock, int64_t* counters);
SF_API int sf_cache_adopt_slots(void* cache, const int32_t* slot_expert, const int32_t* slot_gen,
                                const int64_t* slot_stamp, int64_t clock, const int64_t* counters);

/*
 * Device-resident expert directory (device-managed cache mode).  The slot
 * bookkeeping of one cache in HBM: slot_expert[S], slot_gen[S],
 * slot_stamp[S] (int64), expert_slot[E], clock[1] and counters[4] (int64).
 * sf_dir_plan (one CTA) takes, for the dispatch's active experts (ascending,
 * or resident ones first), the decisions of the host wave loop: per wave up
 * to S experts are leased — a resident one keeps its slot, a missing one
 * evicts the least recently used unleased slot (new generation, a fill
 * record) — each acquisition and, after the wave, each release advancing the
 * LRU clock.  Outputs per wave w < waves: wave_table[w][E] (expert -> slot,
 * -1 outside the wave), wave_active[w][E], wave_count[w], and the fill list
 * fill_expert[w][S] / fill_slot[w][S] / fill_count[w].  status[0] is set to
 * 1 if the experts did not fit `waves` waves, 2 on an expert id outside
 * [0, E).  sf_dir_fill copies wave w's missing experts (fill_count read on
 * the device) from device-mapped page-locked host memory — expert_src[E]
 * holds each expert's device address — into storage + slot * slot_stride,
 * expert_bytes each, with `grid` CTAs of SM loads.  Both are stream-ordered
 * and allocate nothing.  sf_host_device_address gives the device address of
 * page-locked, device-mapped host memory (SF_ERR_UNSUPPORTED otherwise).
 * Replaces the host round trip of qwen3_offloaded_experts.py:112 /
 * :173-175 (reading the routed experts back before leasing).
 */
SF_API int sf_dir_plan(void* slot_expert, void* slot_gen, void* slot_stamp, void* expert_slot, void* clock,
                       void* counters, const void* active, const void* num_active, int num_experts,
                       int num_slots, int waves, int resident_first, void* wave_table, void* wave_active,
                       void* wave_count, void* fill_expert, void* fill_slot, void* fill_count, void* status,
                       void* stream);
/*
 * sf_dir_plan with a conditional handle (0: none, as sf_dir_plan) of the
 * graph the launch is captured into: the plan sets it to 1 when some wave
 * after the first has experts, else 0 (sf_capture_* below).
 */
SF_API int sf_dir_plan_ex(void* slot_expert, void* slot_gen, void* slot_stamp, void* expert_slot, void* clock,
                          void* counters, const void* active, const void* num_active, int num_experts,
                          int num_slots, int waves, int resident_first, void* wave_table, void* wave_active,
                          void* wave_count, void* fill_expert, void* fill_slot, void* fill_count, void* status,
                          uint64_t later_waves, void* stream);
SF_API int sf_dir_fill(const void* expert_src, void* storage, int64_t slot_stride_bytes, int64_t expert_bytes,
                       const void* fill_expert, const void* fill_slot, const void* fill_count, int num_slots,
                       int grid, void* stream);
SF_API int sf_host_device_address(const void* host, uint64_t* device_address);

/*
 * Conditional sections of a captured CUDA graph (no counterpart in the
 * reference, which runs the wave loop on the host): a device-managed cache's
 * waves after the first are captured into the body of an IF node, so a layer
 * whose experts fit its slots launches nothing for them.
 * sf_capture_cond_handle: a new conditional handle (reset to 0 at every graph
 * launch) of the graph `stream` is capturing into; SF_ERR_STATE when it is
 * not capturing.  sf_capture_if_begin: an IF node on `handle` behind the
 * stream's captured work, made the stream's dependency, and `body_stream`
 * (another stream) capturing into its body.  sf_capture_if_end: ends the body
 * capture and adds an empty kernel on `stream` behind the node.
 */
SF_API int sf_capture_body_stream(void** stream); /* per device, created once, kept until exit */
SF_API int sf_capture_cond_handle(void* stream, uint64_t* handle);
SF_API int sf_capture_if_begin(void* stream, void* body_stream, uint64_t handle);
SF_API int sf_capture_if_end(void* stream, void* body_stream);

/*
 * Tree attention (GQA): for query row i of head h (kv head h / (Hq/Hkv)),
 * key j is visible when j < prefix_len, or when bit (j - prefix_len) of
 * tree_bits[i * bit_words + ...] is set (little-endian uint32 words).
 * q: [Hq, Tq, D] with strides (q_head_stride, q_row_stride) in elements,
 * k/v: [Hkv, Tk, D] with (kv_head_stride, kv_row_stride), bf16.  D is 128
 * for the tensor-core kernels; any multiple of 4 up to 128 on the CUDA-core
 * kernel, which SF_ATTN_AUTO picks for D != 128.
 * out: [Tq, Hq, D] bf16, 8-byte aligned (the layout the o_proj consumes).
 * workspace: sf_tree_attention_workspace_bytes(Hq, Tq, Tk) bytes.
 * Replaces SDPA under the verification mask (transformers/...:172-186 with
 * eagle3_types.py:450-473).
 */
/* Implementation choice of sf_tree_attention_ex. */
#define SF_ATTN_AUTO 0 /* tcgen05 kernel for >= 256 packed rows (query rows x heads per KV head) over >= 2,048 keys, else the mma.sync kernel when supported (D=128, q rows 4-byte and K/V rows 16-byte aligned), else CUDA cores */
#define SF_ATTN_SIMT 1 /* CUDA-core split kernel (any D that is a multiple of 4, <= 128) */
#define SF_ATTN_MMA 2  /* warp-level tensor-core (mma.sync) split kernel; SF_ERR_INVALID_ARGUMENT if unsupported */
#define SF_ATTN_TCGEN05 3 /* tcgen05/TMEM kernel, K/V by TMA (D=128, 16-byte aligned q/k/v rows); SF_ERR_INVALID_ARGUMENT if unsupported */

SF_API size_t sf_tree_attention_workspace_bytes(int num_heads, int64_t q_len, int64_t kv_len);
SF_API int sf_tree_attention(const void* q, const void* k, const void* v, const uint32_t* tree_bits,
                      int bit_words, int64_t q_len, int64_t kv_len, int64_t prefix_len,
                      int num_heads, int num_kv_heads, int head_dim, int64_t q_head_stride,
                      int64_t q_row_stride, int64_t kv_head_stride, int64_t kv_row_stride,
                      float scale, void* out, void* workspace, size_t workspace_bytes,
                      void* stream);
SF_API int sf_tree_attention_ex(const void* q, const void* k, const void* v, const uint32_t* tree_bits,
                                int bit_words, int64_t q_len, int64_t kv_len, int64_t prefix_len,
                                int num_heads, int num_kv_heads, int head_dim, int64_t q_head_stride,
                                int64_t q_row_stride, int64_t kv_head_stride, int64_t kv_row_stride,
                                float scale, void* out, void* workspace, size_t workspace_bytes,
                                int impl, void* stream);

/*
 * Several requests' tree attention in one launch of the tcgen05 kernel (the
 * per-request calls of the verify forward over a batch, eagle3_tree.py:
 * 1243-1250 with batch > 1): request b's q, k/v, tree bits and output start
 * b * (q_batch_stride, kv_batch_stride, bits_batch_stride, out_batch_stride)
 * elements (uint32 words for the bits) after request 0's; every request has
 * the same q_len, kv_len, prefix_len and head strides.  The key range is
 * split so that the batch's CTAs fill the SMs.  Returns SF_ERR_UNSUPPORTED,
 * with no message, for layouts the tcgen05 kernel does not take (D != 128,
 * strides not multiples of 8 elements, unaligned rows): callers then make
 * one sf_tree_attention call per request.
 */
SF_API size_t sf_tree_attention_batched_workspace_bytes(int batch, int num_heads, int64_t q_len,
                                                       int64_t kv_len);
SF_API int sf_tree_attention_batched(const void* q, const void* k, const void* v, const uint32_t* tree_bits,
                                     int bit_words, int batch, int64_t q_batch_stride,
                                     int64_t kv_batch_stride, int64_t bits_batch_stride,
                                     int64_t out_batch_stride, int64_t q_len, int64_t kv_len,
                                     int64_t prefix_len, int num_heads, int num_kv_heads, int head_dim,
                                     int64_t q_head_stride, int64_t q_row_stride, int64_t kv_head_stride,
                                     int64_t kv_row_stride, float scale, void* out, void* workspace,
                                     size_t workspace_bytes, void* stream);

/*
 * SpecFit exact subtree selection (host function, runs on the calling CPU
 * thread; no GPU work).  Nodes are raw ids 1..num_nodes with parents[raw-1]
 * < raw (0 = the verification seed) and cumulative log-probabilities
 * cum_logp[raw-1].  footprints holds (num_nodes + 1) bitsets of `words`
 * uint64 words (raw 0 = the seed): bit 128*layer + expert set for every
 * routed (layer, expert) of that token.  resident (nullable, `words` words)
 * marks cache-resident pairs.  Among all ancestor-closed subsets S with
 * |S| <= max_nodes, maximises
 *   (1 + sum_{i in S} exp(cum_logp_i)) /
 *   (size_intercept_ns[|S|] + expert_ns*|F| + missing_ns*|F \ resident|)
 * with F the union of the seed's and S's footprints (resident == NULL: every
 * pair is missing), ties broken by the smallest (-reward, |F|, |S|, ids); the
 * reward is summed with compensated (Neumaier) summation in id order.
 * Writes the ids (increasing) to selected[0..*num_selected) and the score.
 * Replaces exact_specfit_selection / _score_packed_routes
 * (src/specfit/specfit_exact.py:58-94, topology of
 * src/specfit/cache_selection_diagnostic.py:20-39), without the reference's
 * restriction to pools of 2/6/10/14/18 nodes (num_nodes <= 63).
 */
SF_API int sf_specfit_select(int num_nodes, const int32_t* parents, const double* cum_logp,
                             const uint64_t* footprints, int words, const uint64_t* resident,
                             const double* size_intercept_ns, int max_nodes, double expert_ns,
                             double missing_ns, int32_t* selected, int32_t* num_selected,
                             double* best_score);

/* Packs routes int32 [tokens][layers][top_k] into footprint bitsets
 * [tokens][words] (bit layer*experts + expert); SF_ERR_INVALID_ARGUMENT on an
 * expert id outside [0, experts) or a repeated id within a (token, layer).
 * The packing of _pack_routes (src/specfit/specfit_exact.py:18-49). */
SF_API int sf_specfit_pack_routes(const int32_t* routes, int tokens, int layers, int top_k,
                                  int experts, uint64_t* footprints, int words);

/* Compensated (Neumaier) left-to-right sum of n doubles, the summation the
 * selection's reward uses (Python's builtin sum over floats). */
SF_API double sf_compensated_sum(const double* values, int n);

/*
 * Expert parallelism of the MoE block over `world` GPUs (no counterpart in
 * the reference, which refuses more than one GPU).  Rank r owns experts
 * [r*E/world, (r+1)*E/world).  A token travels at most once to each rank it
 * has routes on, as one row of sf_ep_row_bytes() bytes:
 *   [hidden (H elements of dtype) | int32 local_ids[K] | float weights[K] | pad]
 * local_ids ascending, -1 padded (weights 0 padded).  Per layer:
 *   source:      sf_ep_send_pack     -> rows grouped by destination rank, then token;
 *                send_counts[2d] = rows (pairs) and [2d+1] = routes for rank d
 *   exchange:    all-to-all of the rows (split by pairs per rank)
 *   destination: sf_ep_recv_group    -> stable grouping by local expert
 *                sf_ep_recv_gather   -> sorted hidden rows + weights
 *                sf_grouped_swiglu   (local experts)
 *                sf_ep_return_pack   -> one output row per received route, in
 *                                       (pair, slot) order
 *   exchange:    all-to-all back (split by routes per rank)
 *   source:      sf_moe_combine with inv_pos = route_row
 * With sources in rank order the per-expert groups and the combine order are
 * those of one GPU, so the result is bit-identical to the one-GPU block.
 */
/* Row size in bytes (a multiple of 16), or -1 for an unsupported dtype. */
SF_API int64_t sf_ep_row_bytes(int dtype, int hidden_size, int top_k);
/* send_rows: [tokens*world, row_bytes] capacity; send_counts: int64 [2*world];
 * route_row: int32 [tokens*top_k], the row of each route's output in the
 * returned buffer (-1 for an invalid route, which also sets *error_flag);
 * pair_token: int32 [tokens*world] workspace.  top_k <= 16, world <= 8. */
SF_API int sf_ep_send_pack(const void* hidden, int dtype, int64_t tokens, int hidden_size,
                           const int64_t* topk_index, const void* topk_weights, int weight_dtype,
                           int top_k, int num_experts, int world, void* send_rows,
                           int64_t row_bytes, int64_t* send_counts, int32_t* route_row,
                           int32_t* pair_token, int32_t* error_flag, void* stream);
/* Groups the pairs*top_k received route slots by local expert (slots with
 * id -1 are padding).  Outputs as sf_moe_dispatch over local_experts, plus
 * return_src[q] = sorted row of the q-th valid slot in (pair, slot) order. */
SF_API int sf_ep_recv_group(const void* recv_rows, int64_t row_bytes, int dtype, int64_t pairs,
                            int hidden_size, int top_k, int local_experts, int32_t* counts,
                            int32_t* offsets, int32_t* sorted_pos, int32_t* inv_pos,
                            int32_t* active, int32_t* num_active, int32_t* return_src,
                            int32_t* error_flag, void* stream);
/* hidden_sorted[i] = hidden of pair sorted_pos[i] / top_k, weights_sorted[i]
 * = its weight at slot sorted_pos[i] % top_k, for i < routes. */
SF_API int sf_ep_recv_gather(const void* recv_rows, int64_t row_bytes, int dtype, int hidden_size,
                             int top_k, const int32_t* sorted_pos, int64_t routes,
                             void* hidden_sorted, float* weights_sorted, void* stream);
/* return_rows[q] = out_sorted[return_src[q]] for q < routes. */
SF_API int sf_ep_return_pack(const void* out_sorted, int dtype, int hidden_size,
                             const int32_t* return_src, int64_t routes, void* return_rows,
                             void* stream);

/*
 * Expert parallelism over peer memory: the same exchange as above without
 * NCCL and without host synchronisation (every count is read on the
 * device), so a verify pass of all layers can be one CUDA graph.  Each rank
 * owns one region of sf_ep_peer_layout() bytes (sf_ipc_alloc), maps every
 * other rank's region with sf_ipc_open (CUDA IPC, peer access over NVLink)
 * and lists all bases, in rank order, in the device array `peers`.  Sources
 * store their rows straight into the destinations' regions; arrival counters
 * (system-scope fence + atomic add per CTA) tell the readers when a layer's
 * data is complete.  Waits give up after wait_limit_ms and record
 * status[0] = site (1 receive, 2 return) and status[1] |= bit of every rank
 * that did not arrive; the host reads `status` after a step.  Every rank must
 * run the same sequence of layers with the same `grid`.
 * Per layer: sf_ep_peer_send -> sf_ep_peer_recv -> sf_grouped_swiglu (rows =
 * world * cap_routes, offsets/active from sf_ep_peer_recv) ->
 * sf_ep_peer_return -> sf_ep_peer_finish.
 */
typedef struct sf_ep_peer {
  int world, rank, top_k, hidden_size, dtype, local_experts;
  int grid;           /* CTAs of the push/gather/return kernels, equal on every rank */
  int wait_limit_ms;  /* bounded waits (e.g. 2000) */
  int64_t cap_pairs;  /* max tokens a rank sends per layer (rows per source block) */
  int64_t cap_routes; /* max routes per source block: cap_pairs * top_k covers every case */
  int64_t row_bytes;  /* sf_ep_row_bytes(dtype, hidden_size, top_k) */
  int64_t out_row_bytes; /* hidden_size * element size */
  const uint64_t* peers; /* device [world]: region base of every rank */
  void* local;           /* this rank's region (peers[rank]) */
  uint64_t* epochs;      /* device [2], this rank only, zeroed with the regions */
  int32_t* status;       /* device [2], this rank only */
  int64_t off_recv_rows, off_ret_rows, off_recv_counts, off_recv_arrive, off_ret_arrive;
} sf_ep_peer;

/* Fills the off_* fields from world, capacities and row sizes; returns the
 * region size in bytes (-1 for a null descriptor). */
SF_API int64_t sf_ep_peer_layout(sf_ep_peer* d);
/* cudaMalloc + zero + IPC handle (64 bytes) of a region; the one allocating
 * entry point of the library, paired with sf_ipc_free. */
SF_API int sf_ipc_alloc(size_t bytes, void** ptr, void* handle);
SF_API int sf_ipc_free(void* ptr);
/* Maps another process's region into the current device's context. */
SF_API int sf_ipc_open(const void* handle, void** ptr);
SF_API int sf_ipc_close(void* ptr);
/* Plan + push of this rank's tokens (tokens <= cap_pairs).  staging_rows:
 * [tokens*world, row_bytes]; route_row: [tokens*top_k] rows of the returned
 * outputs in this rank's ret_rows ([d][cap_routes] layout). */
SF_API int sf_ep_peer_send(const sf_ep_peer* d, const void* hidden, int64_t tokens,
                           const int64_t* topk_index, const void* topk_weights, int weight_dtype,
                           int num_experts, void* staging_rows, int64_t* send_counts,
                           int32_t* route_row, int32_t* pair_token, int32_t* error_flag,
                           void* stream);
/* Wait for every source, group the received slots by local expert (outputs
 * sized as sf_ep_recv_group with pairs = world*cap_pairs) and gather them
 * into hidden_sorted [world*cap_routes, H] / weights_sorted. */
SF_API int sf_ep_peer_recv(const sf_ep_peer* d, int32_t* counts, int32_t* offsets,
                           int32_t* sorted_pos, int32_t* inv_pos, int32_t* active,
                           int32_t* num_active, int32_t* return_src, int32_t* error_flag,
                           void* hidden_sorted, float* weights_sorted, void* stream);
/* Store each weighted output row into its source's region. */
SF_API int sf_ep_peer_return(const sf_ep_peer* d, const void* out_sorted,
                             const int32_t* return_src, const int32_t* offsets, void* stream);
/*
 * The return fused into the expert GEMM (instead of sf_ep_peer_return after
 * sf_grouped_swiglu): sf_ep_peer_return_plan writes, for every sorted row,
 * the address of its row in its source's region (0 for none) into
 * dst_row[world * cap_routes]; sf_grouped_swiglu_peer runs the tcgen05
 * grouped SwiGLU over the received rows (rows = world * cap_routes, experts =
 * local_experts, act_workspace [rows, intermediate]) with phase 2 storing
 * each weighted output row straight to dst_row[r] (NVLink stores for a
 * peer), every CTA counting itself on `ticket` (a device uint32, zero before
 * the first call; each call leaves it zero) and the last one adding `grid`
 * to this rank's return counter in every region, exactly what
 * sf_ep_peer_return adds, so sf_ep_peer_finish is unchanged.  Every rank of
 * an exchange must use the same form for a layer.  bf16 only.  No
 * counterpart in the reference, which runs on one GPU (no expert parallelism).
 */
SF_API int sf_ep_peer_return_plan(const sf_ep_peer* d, const int32_t* return_src, const int32_t* offsets,
                                  uint64_t* dst_row, void* stream);
SF_API int sf_grouped_swiglu_peer(const sf_ep_peer* d, const void* hidden_sorted, const float* weights_sorted,
                                  const int32_t* offsets, const int32_t* active, const int32_t* num_active,
                                  const int32_t* expert_slot, const void* slot_storage, int64_t slot_count,
                                  int64_t slot_stride_elems, int intermediate_size, void* act_workspace,
                                  const uint64_t* dst_row, uint32_t* ticket, void* stream);
/* Wait for every destination's outputs and combine them (sf_moe_combine). */
SF_API int sf_ep_peer_finish(const sf_ep_peer* d, const int64_t* topk_index,
                             const int32_t* route_row, int64_t tokens, int num_experts,
                             int reduce, void* out, void* stream);

/*
 * Fused elementwise steps of a Qwen3-MoE decoder layer (bf16 only).
 * sf_add_rmsnorm: per row, h = residual_in + x rounded to bf16 (h = x when
 * residual_in is NULL), written to residual_out when non-NULL, and
 * out = bf16(weight * bf16(h * rsqrt(mean(h^2) + eps))).  H % 8 == 0,
 * H <= 8192, 16-byte aligned rows.
 */
SF_API int sf_add_rmsnorm(const void* x, const void* residual_in, void* residual_out,
                          const void* weight, float eps, int64_t rows, int hidden_size, void* out,
                          void* stream);
/*
 * sf_qk_norm_rope: qkv [batch*tokens, (Hq + 2*Hkv) * 128] (q heads, then k,
 * then v); q and k heads get the head RMSNorm with their weights [128] and the
 * rotary embedding x*cos + rotate_half(x)*sin with cos/sin [batch*tokens, 128]
 * (each product and the sum rounded to bf16).  q goes to q_out
 * [batch, Hq, tokens, 128]; k and v go to the cache rows row0 + t (row0 read
 * from row0_device when non-NULL) of k_cache / v_cache laid out
 * [batch][Hkv][rows][128] with the given batch and head strides (elements).
 * With both norm weights NULL the head norm is skipped (rotary only).
 */
/*
 * KV compaction of the accepted verify rows (_compact_tree_cache,
 * src/specfit/runtime/eagle3_tree.py:833-858) for all layers in two launches:
 * buffers is a device array of 2*layers base pointers (k and v of each
 * layer, batch 1) laid out [heads][rows][head_dim] with head_stride elements
 * between heads; rows base + src_rows[i] (device int32 [n]) move to base + i.
 * stage: 2 * layers * n * heads * head_dim bf16 elements of scratch.
 */
SF_API int sf_kv_compact(const uint64_t* buffers, int layers, int heads, int head_dim,
                         int64_t head_stride, int64_t base, const int32_t* src_rows, int n,
                         void* stage, void* stream);
/*
 * Visibility words for sf_tree_attention with prefix_len 0 over a whole KV
 * buffer: out [rows][words] int32, column c visible when c < *start_device
 * (the committed rows, read on the device) or when 0 <= c - start < 64 and
 * bit c - start of ancestor_sets[row] (int64) is set (a tree block of at most
 * 64 rows starting at row start).  New: serves drafting replayed from a graph.
 */
SF_API int sf_tree_mask_words(const int64_t* ancestor_sets, int rows, const int64_t* start_device,
                              int words, int32_t* out, void* stream);
/*
 * Log-softmax of scale * logits (bf16 [rows][vocab], row-major) and its k
 * largest entries per row, in one launch (a cluster of 16 CTAs per row, 8
 * where 16 cannot be co-scheduled; rows <= 65535): top_values [rows][k] fp32
 * log-probabilities, top_indices [rows][k] int64, larger first
 * and the lower index first among equal values.  1 <= k <= 8.  The
 * log-probability of logit y is (scale*y - max) - log(sum exp(scale*y - max)),
 * summed in fp32.  Each row must hold at least k finite values of scale*y.
 */
SF_API int sf_logsoftmax_topk(const void* logits, int64_t rows, int64_t vocab, float scale, int k,
                              float* top_values, int64_t* top_indices, void* stream);
/*
 * out[rows][out_features] = x[rows][in_features] . weight[out_features][in_features]^T
 * in bf16 with fp32 accumulation, rounded once (F.linear without bias), on
 * tcgen05 tensor cores with K split across a CTA cluster and the partial
 * sums added in a fixed order.  For verify-sized inputs: rows <= 128,
 * in_features % 64 == 0, x and weight contiguous and 16-byte aligned;
 * otherwise returns SF_ERR_UNSUPPORTED without a message (use a library
 * GEMM).
 */
SF_API int sf_linear_bf16(const void* x, int64_t rows, int64_t in_features, const void* weight,
                          int64_t out_features, void* out, void* stream);

/*
 * lm_head + greedy pick in one pass over the weight: out[t, n] (nullable)
 * = bf16(x[t] . weight[n]) as sf_linear_bf16 computes it, and argmax[t] =
 * the n with the largest bf16 value, the lowest n among equal ones (what
 * torch.argmax returns on those logits).  rows <= 128, in_features a multiple
 * of 64, 16-byte aligned x and weight.  workspace: at least
 * sf_linear_argmax_workspace_bytes(rows, in_features, out_features) bytes.
 * Replaces the target's lm_head F.linear and the argmax of the verify step
 * (src/specfit/runtime/eagle3_tree.py:1252).
 */
SF_API size_t sf_linear_argmax_workspace_bytes(int64_t rows, int64_t in_features, int64_t out_features);
SF_API int sf_linear_bf16_argmax(const void* x, int64_t rows, int64_t in_features, const void* weight,
                                 int64_t out_features, void* out, int64_t* argmax, void* workspace,
                                 size_t workspace_bytes, void* stream);
/*
 * One level of a drafted candidate pool (the tree builder's level step,
 * src/specfit/runtime/eagle3_tree.py:611-803): among rows x k children
 * (top_values / top_indices [rows][k]: each frontier row's k most likely next
 * tokens and their log-probabilities), the `width` best by cum[row] + value
 * (fp64), ties by lower frontier row then lower token, become the next
 * frontier: next_tokens, next_cum, next_ancestor_sets (the parent's set plus
 * bit row_base + slot), next_positions (*seed_pos + depth + 1) and
 * next_hidden (the parent rows of hidden [rows][hidden_size] bf16).  Their
 * pool rows (token, first + parent row, log-probability, cumulative,
 * depth + 1) are written to out_rows [width][5] fp64.  rows * k <= 32,
 * row_base + width <= 64.
 */
SF_API int sf_draft_level(const float* top_values, const int64_t* top_indices, int rows, int k,
                          const double* cum, const int64_t* ancestor_sets, const void* hidden,
                          int hidden_size, int width, int64_t first, int depth, int row_base,
                          const int64_t* seed_pos, int64_t* next_tokens, double* next_cum,
                          int64_t* next_ancestor_sets, int64_t* next_positions, void* next_hidden,
                          double* out_rows, void* stream);
/*
 * Rotary embedding rows at device-side positions: cos_out / sin_out
 * [rows][head_dim] bf16, column d and d + head_dim/2 = bf16(cos / sin(a)),
 * a = float(positions[r]) * inv_freq[d] in fp32.
 */
SF_API int sf_rope_rows(const int64_t* positions, int rows, const float* inv_freq, int head_dim,
                        void* cos_out, void* sin_out, void* stream);
/*
 * sf_moe_combine (bf16) fused with the decoder layer's residual add and the
 * next RMSNorm: for each token, moe = the combined row exactly as
 * sf_moe_combine writes it, then exactly sf_add_rmsnorm(moe, residual_in,
 * residual_out, norm_weight, eps, out).  hidden_size % 8 == 0, <= 8192; rows
 * 16-byte aligned.  residual_out may equal residual_in.
 */
SF_API int sf_moe_combine_add_rmsnorm(const void* out_sorted, const int32_t* inv_pos,
                                      const int64_t* topk_index, const int32_t* expert_rank,
                                      int num_experts, int64_t tokens, int top_k, int hidden_size,
                                      int reduce, const void* residual_in, void* residual_out,
                                      const void* norm_weight, float eps, void* out, void* stream);
SF_API int sf_qk_norm_rope(const void* qkv, int64_t batch, int64_t tokens, int num_heads,
                           int num_kv_heads, int head_dim, const void* q_norm_weight,
                           const void* k_norm_weight, const void* cos, const void* sin, float eps,
                           void* q_out, void* k_cache, void* v_cache, int64_t kv_batch_stride,
                           int64_t kv_head_stride, int64_t row0, const int64_t* row0_device,
                           void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPECFIT_B200_H_ */
