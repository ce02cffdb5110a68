/*
 * mtp_b200 - B200 (sm_100a) W4A16 mixture-of-experts layer and expert-prefetch
 * path: the C ABI.
 *
 * Every entry point takes plain pointers and sizes, returns an int status
 * (0 = MTP_OK, a distinct non-zero code per failure class, never an exception)
 * and, where it launches GPU work, runs asynchronously on the caller's stream
 * (`stream` is a cudaStream_t passed as void*; NULL = the legacy default
 * stream). The caller allocates every output and workspace; the prefetch
 * session alone owns device state and a side stream.
 *
 * Reference interfaces replaced (paths relative to the reference project,
 * HUSRCF/MTP "mtp-expert-prefetch"; vLLM 0.22.0 paths relative to the package):
 *   mtp_router_topk            <- vLLM torch.ops._moe_C.topk_softmax, restated by
 *                                 the reference at tracing/vllm_router_trace.py:4201-4227
 *   mtp_moe_align              <- vLLM fused_moe/moe_align_block_size.py
 *                                 moe_align_block_size(), called at
 *                                 vllm_router_trace.py:19648-19659 (replaced there
 *                                 through _prepare_expert_assignment, :20083)
 *   mtp_gptq_dequant           <- repack/gptq_unpack.py:88-131
 *                                 dequantize_gptq_projection()
 *   mtp_w4a16_repack_gptq      <- vLLM moe_wna16.py GPTQ weight conversion
 *                                 (qweight.T -> [E, N, K/2] uint8) consumed by
 *                                 tracing/vllm_wna16_group_plan.py:242-486
 *   mtp_w4a16_moe_layer        <- vLLM fused_experts_impl as restated at
 *                                 vllm_router_trace.py:19330-19840 (W1 at 19674,
 *                                 activation 19714, W2 at 19761, moe_sum 19801),
 *                                 the shared-expert gate at 3994-4031 / 4140-4152,
 *                                 and the CPU forms TopKExpertMlp.forward
 *                                 (repack/gptq_unpack.py:293-327) and
 *                                 MtpExtraRunner.moe_tokens (mtp/extra_tensors.py:544-598);
 *                                 the expert->slot indirection follows the
 *                                 expert_map reads at vllm_wna16_group_plan.py:87-95,
 *                                 1555-1567 and the premap slot plan at
 *                                 runtime/premap.py:223-294
 *   mtp_predictor_topk         <- training/hidden_residual.py:44-134 forward +
 *                                 topk as in training/predictor.py:105
 *   mtp_prefetch_session_*     <- the native producer session C ABI at
 *                                 microbench/premap_kernel_consumer/
 *                                 premap_payload_cache_inprocess_native_producer_stub.hip:505-960
 *                                 (create / destroy / update with int codes and an
 *                                 opaque u64 handle) and the counter semantics of
 *                                 runtime/cache_manager.py:193-578
 */
#ifndef MTP_B200_H_
#define MTP_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define MTP_API __attribute__((visibility("default")))
#else
#define MTP_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------- */
enum MtpStatus {
  MTP_OK = 0,
  MTP_ERR_NULL = 1,       /* a required pointer is NULL                       */
  MTP_ERR_SHAPE = 2,      /* a size is out of range or not supported         */
  MTP_ERR_ALIGN = 3,      /* a pointer is not aligned as the kernel requires  */
  MTP_ERR_WORKSPACE = 4,  /* workspace smaller than the size query returned   */
  MTP_ERR_LAUNCH = 5,     /* a kernel launch failed                           */
  MTP_ERR_CUDA = 6,       /* another CUDA runtime call failed                 */
  MTP_ERR_HANDLE = 7,     /* bad or destroyed session handle                  */
  MTP_ERR_CAPACITY = 8,   /* no free slot / ring full                         */
  MTP_ERR_ARG = 9         /* an enum or flag argument has an unknown value    */
};

MTP_API const char* mtp_status_string(int status);
MTP_API int mtp_abi_version(void);

/* Device address of pinned (page-locked, mapped) host memory, for
 * MtpMoeLayerArgs.host_blobs: cudaHostGetDevicePointer on the current device. */
MTP_API int mtp_host_device_pointer(const void* host_ptr, void** device_ptr);

/* ---- router (softmax -> top-k -> renormalise) ----------------------------- */
/* logits [M, E] fp32 -> topk_weights [M, k] fp32, topk_ids [M, k] int32
 * (descending; exact ties -> lower expert id), token_expert_indices [M, k]
 * (= j, as the reference fallback writes; may be NULL). renormalize: w/sum(w)
 * with the sum clamped to 1e-20. 1 <= k <= 32, 1 <= E <= 1024.               */
MTP_API int mtp_router_topk(const float* logits, int32_t M, int32_t E, int32_t k,
                    int32_t renormalize, float* topk_weights, int32_t* topk_ids,
                    int32_t* token_expert_indices, void* stream);

/* ---- moe_align_block_size (canonical order) ------------------------------- */
/* Buffer sizes exactly as vLLM's wrapper computes them.                      */
MTP_API int mtp_moe_align_sizes(int32_t numel, int32_t num_experts, int32_t block_size,
                        int32_t pad_sorted_ids, int32_t* sorted_capacity,
                        int32_t* max_blocks, int32_t* max_segments);
/* topk_ids [numel] int32 -> sorted_token_ids [sorted_capacity] (sentinel numel),
 * expert_ids [max_blocks] (-1 past the last used block), num_tokens_post_padded
 * [1]; within an expert the flat pair index ascends. expert_map [E] may be
 * NULL. segments (may be NULL) receives [max_segments][3] rows
 * (expert, first_block, block_count) and num_segments [1] their count.       */
MTP_API int mtp_moe_align(const int32_t* topk_ids, int32_t numel, int32_t num_experts,
                  int32_t block_size, const int32_t* expert_map,
                  int32_t ignore_invalid_experts, int32_t pad_sorted_ids,
                  int32_t* sorted_token_ids, int32_t* expert_ids,
                  int32_t* num_tokens_post_padded, int32_t* segments,
                  int32_t* num_segments, void* stream);

/* ---- GPTQ int4 weights ----------------------------------------------------- */
enum MtpZeroMode {
  MTP_ZERO_RAW = 0,   /* (q - stored zero) * scale: the reference torch oracle */
  MTP_ZERO_SYM8 = 1   /* (q - 8) * scale, stored zeros ignored: vLLM sym GPTQ */
};

/* fp32 dequantisation of one projection, GPTQ checkpoint form:
 * qweight [K/8, N] int32, qzeros [K/G, N/8] int32, scales [K/G, N] fp16 (bits),
 * g_idx [K] int32 or NULL (= k / G). out [N, K] fp32 (Linear orientation).   */
MTP_API int mtp_gptq_dequant(const int32_t* qweight, const int32_t* qzeros,
                     const uint16_t* scales, const int32_t* g_idx, int32_t K,
                     int32_t N, int32_t group_size, int32_t zero_mode,
                     float* out, void* stream);

/* Byte offsets of the sections of one expert blob in the kernel layout:
 * [w13 weights | w13 scales | w13 zeros | w2 weights | w2 scales | w2 zeros],
 * w13 = gate rows then up rows, [2I, H]; w2 = [H, I]. Every section starts on
 * a 256-byte boundary; `bytes` is the blob stride.                            */
typedef struct MtpExpertLayout {
  int64_t w13_qweight, w13_scales, w13_zeros;
  int64_t w2_qweight, w2_scales, w2_zeros;
  int64_t bytes;
} MtpExpertLayout;
MTP_API int mtp_w4a16_expert_layout(int32_t hidden, int32_t inter, int32_t group_size,
                            MtpExpertLayout* out);

/* Repack E experts from the GPTQ checkpoint form (stacked on a leading E axis:
 * w13 qweight [E, H/8, 2I], qzeros [E, H/G, 2I/8], scales [E, H/G, 2I];
 * w2 qweight [E, I/8, H], qzeros [E, I/G, H/8], scales [E, I/G, H]) into
 * out_blobs [E, layout.bytes].                                              */
MTP_API int mtp_w4a16_repack_gptq(const int32_t* w13_qweight, const int32_t* w13_qzeros,
                          const uint16_t* w13_scales, const int32_t* w2_qweight,
                          const int32_t* w2_qzeros, const uint16_t* w2_scales,
                          int32_t num_experts, int32_t hidden, int32_t inter,
                          int32_t group_size, uint8_t* out_blobs, void* stream);

/* ---- the MoE layer forward ------------------------------------------------- */
typedef struct MtpMoeLayerArgs {
  int32_t num_tokens;        /* M >= 1                                        */
  int32_t hidden;            /* H: multiple of 256, 256..2048                 */
  int32_t inter;             /* I: multiple of 128, 128..1024                 */
  int32_t num_experts;       /* E: 1..1024 (global expert count)              */
  int32_t top_k;             /* 1..32                                         */
  int32_t group_size;        /* 64 or 128                                     */
  int32_t renormalize;       /* router: renormalise the top-k weights         */
  int32_t zero_mode;         /* MtpZeroMode                                   */
  const uint16_t* hidden_states;   /* [M, H] bf16                             */
  const float* router_logits;      /* [M, E] fp32; NULL -> use topk_* below   */
  const float* topk_weights;       /* [M, k] fp32 (when router_logits NULL)   */
  const int32_t* topk_ids;         /* [M, k] int32 (when router_logits NULL)  */
  const uint8_t* expert_blobs;     /* resident experts: slot s at
                                      expert_blobs + s * expert_bytes         */
  int64_t expert_bytes;            /* mtp_w4a16_expert_layout().bytes         */
  const int32_t* slot_table;       /* [E] expert -> slot, -1 = not resident;
                                      NULL -> slot = expert                   */
  const uint8_t* host_blobs;       /* device-visible pinned host store, expert
                                      e at host_blobs + e * expert_bytes, read
                                      for slot -1 (demand fetch); may be NULL */
  const uint8_t* shared_blob;      /* shared expert blob or NULL              */
  const uint16_t* shared_gate_weight; /* [H] bf16, required with shared_blob  */
  uint16_t* out;                   /* [M, H] bf16                             */
  float* out_f32;                  /* optional [M, H] fp32 copy (may be NULL) */
  float* topk_weights_out;         /* optional [M, k] router weights          */
  int32_t* topk_ids_out;           /* optional [M, k] router ids              */
  int32_t* demand_log;             /* optional [1 + min(E, M*k)]: count, then
                                      the distinct experts demanded, ascending */
  int32_t* status;                 /* optional [4]: [0] slot misses served from
                                      host_blobs, [1] misses with no host store
                                      (expert output zeroed), [2],[3] reserved;
                                      accumulated, the caller zeroes it        */
  void* workspace;                 /* device, 256-byte aligned, at least
                                      mtp_w4a16_moe_layer_workspace_size()
                                      bytes, ZERO-FILLED before its first use:
                                      the layer keeps its per-call counters
                                      there and every call leaves them zero
                                      again, a call whose waits timed out
                                      included (see _timeouts below)         */
  int64_t workspace_bytes;
  /* Expert parallelism (ABI version 2). expert_map [global_num_experts], as
     vLLM fused_experts(expert_map=...) (consumed by the reference at
     tracing/vllm_wna16_group_plan.py:87-95): topk_ids hold global ids and
     expert_map[g] is the local expert (index into expert_blobs, below
     num_experts) or -1 when another rank owns g; such pairs contribute
     nothing. Only with given ids (router_logits NULL). NULL: ids are local. */
  const int32_t* expert_map;
  int32_t global_num_experts;
  /* Rows [shared_rows_begin, shared_rows_end) get the shared expert (the
     home rows of an expert-parallel call whose partial rows are summed over
     ranks); both 0 = every row.                                            */
  int32_t shared_rows_begin;
  int32_t shared_rows_end;
} MtpMoeLayerArgs;

MTP_API int mtp_w4a16_moe_layer_workspace_size(int32_t num_tokens, int32_t num_experts,
                                       int32_t top_k, int32_t hidden,
                                       int32_t inter, int64_t* bytes);
MTP_API int mtp_w4a16_moe_layer(const MtpMoeLayerArgs* args, void* stream);

/* Number of calls on this layer workspace whose bounded waits ran out (each
 * such call also sets bit 0 of status[2] when `status` is given, and leaves
 * a wrong output). The workspace repairs itself: the last CTA of such a call
 * clears every counter, so the next call is correct. Copies the count to the
 * host and synchronises `stream`. No counterpart in the reference (its
 * kernels have no bounded waits).                                           */
MTP_API int mtp_w4a16_moe_layer_timeouts(const void* workspace, int32_t* count, void* stream);

/* ---- the layer forward without a caller-provided workspace ------------------
 * No counterpart in the reference: an addition for callers that cannot
 * allocate device memory (an FFI host that only passes pointers to buffers it
 * was given; a serving loop whose device memory belongs to another allocator).
 * Same arguments and results as mtp_w4a16_moe_layer, except that `workspace`
 * and `workspace_bytes` are ignored: the scratch is a fixed array of
 * MTP_NOALLOC_SCRATCH_BYTES compiled into the library (held by every GPU that
 * loads it until exit), enough for M <= 48 at H = 2048, I = 512, E = 256,
 * top-8. A request needing more returns MTP_ERR_WORKSPACE without launching.
 * Allocates nothing. The first call on a device looks up the array's device
 * address (with that device current), so make it before any stream capture.
 * All calls share the array and it keeps the last call's contents; calls that
 * overlap on the GPU race and must be serialised by the caller.            */
#define MTP_NOALLOC_SCRATCH_BYTES (6u << 20)
MTP_API int mtp_w4a16_moe_layer_noalloc(const MtpMoeLayerArgs* args, void* stream);

/* ---- the layer forward for prefill-sized calls ------------------------------
 * Same layer as mtp_w4a16_moe_layer (replaces the same boundary: vLLM
 * fused_moe W1 -> silu_and_mul -> W2 (MUL_ROUTED_WEIGHT) -> moe_sum as the
 * reference launches it, tracing/vllm_router_trace.py:19648-19801, plus the
 * gated shared expert) for calls with many pairs per expert: pairs are blocked
 * 128 per expert and each block is one bf16 tensor-core tile, the int4 weights
 * unpacked once per block. Differences from mtp_w4a16_moe_layer: dequantised
 * weights are rounded to bf16 as the reference's bf16 GEMM does (the
 * decode kernel keeps them exact), the W2 output per pair is rounded to bf16
 * before the fp32 top-k sum (vLLM's intermediate_cache3); all experts must be
 * resident (slot_table == NULL, host_blobs ignored: else MTP_ERR_ARG);
 * demand_log must be NULL; E + (shared ? 1 : 0) <= 1024. The workspace needs
 * no zero fill (nothing persists between calls); its size grows with M
 * (about M * (top_k + 1) * (2 H + I) * 2 bytes plus padding).                */
MTP_API int mtp_w4a16_moe_prefill_workspace_size(int32_t num_tokens, int32_t num_experts,
                                         int32_t top_k, int32_t hidden,
                                         int32_t inter, int64_t* bytes);
MTP_API int mtp_w4a16_moe_prefill(const MtpMoeLayerArgs* args, void* stream);

/* Where a prefill call leaves its align tables in its workspace (byte offsets),
 * for inspection: the pairs extended by the shared expert (pair_expert_ids
 * [M, pairs_per_token] int32, the shared expert as id E, -1 for ids outside
 * [0, E)), and the moe_align_block_size result over them with block_size 128
 * and E (+1) experts: sorted_token_ids [capacity] (pair indices, sentinel
 * M * pairs_per_token, valid up to num_tokens_post_padded), expert_ids
 * [max_blocks] (valid for the first num_tokens_post_padded / 128 blocks),
 * num_tokens_post_padded [1]. Same contract as mtp_moe_align (vLLM
 * fused_moe/moe_align_block_size.py, called at
 * tracing/vllm_router_trace.py:19648-19659) with pad_sorted_ids.           */
typedef struct MtpPrefillTables {
  int64_t pair_expert_ids, sorted_token_ids, expert_ids, num_tokens_post_padded;
  int32_t capacity, max_blocks, pairs_per_token, block_size;
} MtpPrefillTables;
MTP_API int mtp_w4a16_moe_prefill_tables(int32_t num_tokens, int32_t num_experts, int32_t top_k,
                                         int32_t hidden, int32_t inter, int32_t has_shared,
                                         MtpPrefillTables* out);


/* ---- MTP expert-demand predictor (prefetch driver) --------------------------
 * logits = W2 . silu(W1 . h + b1) + b2 for each hidden state h [M, hidden]
 * bf16: hidden -> width -> future x experts, then the top_k experts of every
 * future layer (descending logit, exact ties to the lower expert id) into
 * ids_out [M, future, top_k] int32. The first layer's activation is rounded to
 * bf16 before the second linear. Replaces the forward of the reference's
 * predictor family (training/hidden_residual.py:44-134
 * HiddenResidualExpertPredictor; training/predictor.py:193-241) and the
 * topk(logits.float()) ranking of recall_at_m (training/predictor.py:105).
 * Weights W1 [width, hidden] and W2 [future*experts, width] (bf16, out x in)
 * are prepacked once by mtp_predictor_pack into the kernel's fragment order
 * (same byte size). b1 [width] and b2 [future*experts] bf16 may be NULL.
 * hidden, width: multiples of 128, <= 2048; experts <= 1024; top_k <= 32.   */
MTP_API int mtp_predictor_pack(const uint16_t* w, int32_t rows, int32_t cols, uint16_t* out, void* stream);
MTP_API int mtp_predictor_workspace_size(int32_t M, int32_t width, int32_t future, int32_t experts,
                                         int64_t* bytes);
MTP_API int mtp_predict_topk(const uint16_t* h, int32_t M, int32_t hidden, const uint16_t* w1_packed,
                             const uint16_t* b1, int32_t width, const uint16_t* w2_packed,
                             const uint16_t* b2, int32_t future, int32_t experts, int32_t top_k,
                             float* logits_out, int32_t* ids_out, void* workspace,
                             int64_t workspace_bytes, void* stream);

/* The reference predictor architecture, HiddenResidualExpertPredictor.forward
 * (training/hidden_residual.py:44-103): state = LayerNorm(silu(W1 . h + b1))
 * (ln_weight, ln_bias may be NULL = 1 / 0; biased variance; ln_eps), then for
 * every future delta f < future the shared classifier
 * logits[m, f] = Wc . silu(state + layer_emb[layer_ids[m]] + delta_emb[f]) + bc
 * and the top_k experts of each (m, f) into ids_out [M, future, top_k]
 * (logits_out [M, future, experts] fp32 optional). W1 [width, hidden] and
 * Wc [experts, width] bf16 are packed by mtp_predictor_pack; b1 [width],
 * ln_weight / ln_bias [width], layer_emb [num_layers, width], delta_emb
 * [future, width], bc [experts] bf16; layer_ids [M] int32 (NULL = layer 0;
 * clamped to the table). The classifier's input columns are rounded to bf16.
 * Workspace: mtp_predictor_hr_workspace_size bytes.                         */
MTP_API int mtp_predictor_hr_workspace_size(int32_t M, int32_t width, int32_t future, int32_t experts,
                                            int64_t* bytes);
MTP_API int mtp_predict_topk_hidden_residual(const uint16_t* h, const int32_t* layer_ids, int32_t M,
                                             int32_t hidden, const uint16_t* w1_packed, const uint16_t* b1,
                                             int32_t width, const uint16_t* ln_weight,
                                             const uint16_t* ln_bias, float ln_eps,
                                             const uint16_t* layer_emb, int32_t num_layers,
                                             const uint16_t* delta_emb, int32_t future,
                                             const uint16_t* wc_packed, const uint16_t* bc, int32_t experts,
                                             int32_t top_k, float* logits_out, int32_t* ids_out,
                                             void* workspace, int64_t workspace_bytes, void* stream);


/* ---- expert prefetch session (premap slot cache) ----------------------------
 * A per-layer HBM slot cache of expert blobs (slots_per_layer of num_experts
 * resident per layer) filled from a pinned host store by cudaMemcpyAsync on a
 * session-owned side stream, and the expert -> slot tables the layer reads
 * (MtpMoeLayerArgs.slot_table / expert_blobs / host_blobs of layer l:
 * slot_tables + l * num_experts, cache_base + l * slots_per_layer *
 * expert_bytes, host_store + l * num_experts * expert_bytes).
 * Replaces the reference's producer session C-ABI
 * (premap_payload_cache_inprocess_native_producer_stub.hip: session_create_v1
 * 505, destroy_v1 570, update_v1 800), which moves no bytes, with the
 * bookkeeping of its cache managers (runtime/cache_manager.py 193-578), one
 * LRU per layer. The handle is opaque; calls on one session come from one
 * host thread. simulate = 1 keeps the bookkeeping only (no CUDA calls, copies
 * complete at once; pointers may be NULL).                                  */
typedef struct MtpPrefetchConfig {
  int32_t device;
  int32_t num_layers;
  int32_t num_experts;
  int32_t slots_per_layer;
  int64_t expert_bytes;            /* mtp_w4a16_expert_layout().bytes          */
  const uint8_t* host_store;       /* pinned [num_layers][num_experts][bytes]  */
  uint8_t* cache_base;             /* device [num_layers][slots][bytes]        */
  int32_t* slot_tables;            /* device [num_layers][num_experts], set to -1 */
  int32_t simulate;
  int64_t host_layer_stride;       /* bytes between layers in host_store:
                                      0 = num_experts * expert_bytes, -1 = all
                                      layers share one [experts][bytes] block */
} MtpPrefetchConfig;

typedef struct MtpPrefetchStats {  /* CacheManagerSnapshot counters (cache_manager.py:193-205) */
  int64_t issued_fetch_count;
  int64_t used_fetch_count;
  int64_t unused_fetch_count;      /* resident, prefetched, not yet demanded    */
  int64_t demand_count;
  int64_t demand_hit_count;
  int64_t demand_miss_count;
  int64_t evicted_before_use_count;
  int64_t ready_late_miss_count;   /* demanded while its copy was in flight     */
  int64_t inflight_count;
  int64_t resident_count;
  int64_t bytes_copied;
} MtpPrefetchStats;

MTP_API int mtp_prefetch_session_create(const MtpPrefetchConfig* cfg, uint64_t* out_handle);
MTP_API int mtp_prefetch_session_destroy(uint64_t handle);
/* Predicted experts of `layer` (host array): copy the ones neither resident
 * nor in flight, evicting least recently used slots.                        */
MTP_API int mtp_prefetch_issue(uint64_t handle, int32_t layer, const int32_t* experts, int32_t count,
                               int32_t* out_issued);
/* Record that the work enqueued on compute_stream so far is the last use of
 * layer's slots: later copies into that layer wait for it.                  */
MTP_API int mtp_prefetch_layer_used(uint64_t handle, int32_t layer, void* compute_stream);
/* Demanded experts of `layer` (host array): hit / miss accounting; a hit
 * needs the copy complete now. insert_on_miss copies missing experts in.    */
MTP_API int mtp_prefetch_demand(uint64_t handle, int32_t layer, const int32_t* experts, int32_t count,
                                int32_t insert_on_miss, int32_t* out_hits);
/* Make compute_stream wait for the copies still in flight of the given
 * experts of `layer` (issued ahead or queued by demand), so the layer call
 * enqueued next reads them from the slot cache instead of fetching the same
 * bytes from the host store a second time. Non-blocking on the host.
 * Counterpart of the ready-time wait of ReadyTimeExpertCacheManager.demand
 * (runtime/cache_manager.py:399), which charges a late copy's remaining time. */
MTP_API int mtp_prefetch_wait(uint64_t handle, int32_t layer, const int32_t* experts, int32_t count,
                              void* compute_stream);
/* Non-blocking: retire completed copies and report the counters.           */
MTP_API int mtp_prefetch_poll(uint64_t handle, MtpPrefetchStats* out);
MTP_API int mtp_prefetch_sync(uint64_t handle);

#ifdef __cplusplus
}
#endif
#endif /* MTP_B200_H_ */
