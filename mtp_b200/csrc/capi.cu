// extern "C" entry points of libmtp_b200: argument checks, workspace carving,
// launch order. Every function returns an MtpStatus; nothing throws.
#include "internal.cuh"

#include <algorithm>

namespace mtp {

constexpr int kLayerBM = 8;

struct AlignSizes {
  int cap, max_blocks, max_seg;
};

static AlignSizes align_sizes(int numel, int E, int BM, int pad) {
  int64_t cap = static_cast<int64_t>(numel) + static_cast<int64_t>(E) * (BM - 1);
  if (pad) cap = round_up(cap, BM);
  if (numel < E) cap = std::min<int64_t>(static_cast<int64_t>(numel) * BM, cap);
  AlignSizes s;
  s.cap = static_cast<int>(cap);
  s.max_blocks = static_cast<int>((cap + BM - 1) / BM);
  s.max_seg = std::min(numel, E);
  return s;
}

// Workspace of the layer call, each region 256-byte aligned. The first
// regions (grid barrier, per-expert counts, per-segment counters) have fixed
// offsets and sizes, the same for every call shape, so one workspace can serve
// calls of any size: they must be zero before the first call, and every call
// leaves them zero again (after a call whose waits timed out, its last CTA
// clears them in full).
struct LayerWs {
  int64_t bar, cnt, seg_done, tw, tid, lists, gate, xq, wseg, status, gu, ybuf, total;
  int max_ws;
};

static LayerWs layer_ws(int M, int E, int k, int H, int I) {
  const int numel = M * k;
  const AlignSizes s = align_sizes(numel, E, kLayerBM, 0);
  LayerWs w;
  w.max_ws = fused_max_work_segments(M, s.max_seg, s.max_blocks);
  int64_t o = 0;
  auto take = [&](int64_t bytes) {
    const int64_t at = o;
    o = round_up(o + bytes, 256);
    return at;
  };
  w.bar = take(32);
  w.cnt = take(4LL * kMaxExpertsWs);
  w.seg_done = take(4LL * kMaxWorkSegments);
  w.tw = take(4LL * numel);
  w.tid = take(4LL * numel);
  w.lists = take(4LL * E * M);
  w.gate = take(4LL * M);
  w.xq = take(static_cast<int64_t>(M) * xq_row_bytes(H));
  w.wseg = take(4LL * kWsInts * w.max_ws);
  w.status = take(16);
  w.gu = take((numel + M) * (8LL * I + 16));
  w.ybuf = take(4LL * (numel + M) * H);
  w.total = o;
  return w;
}

}  // namespace mtp

using namespace mtp;

extern "C" {

const char* mtp_status_string(int status) {
  switch (status) {
    case MTP_OK: return "ok";
    case MTP_ERR_NULL: return "required pointer is NULL";
    case MTP_ERR_SHAPE: return "size out of range or unsupported";
    case MTP_ERR_ALIGN: return "pointer misaligned";
    case MTP_ERR_WORKSPACE: return "workspace too small";
    case MTP_ERR_LAUNCH: return "kernel launch failed";
    case MTP_ERR_CUDA: return "CUDA runtime call failed";
    case MTP_ERR_HANDLE: return "bad session handle";
    case MTP_ERR_CAPACITY: return "capacity exhausted";
    case MTP_ERR_ARG: return "unknown enum/flag value";
    default: return "unknown status";
  }
}

int mtp_abi_version(void) { return 2; }

// expert_map / shared-row fields of MtpMoeLayerArgs (ABI version 2)
static int ep_fields(const MtpMoeLayerArgs& a, int* sh_begin, int* sh_end) {
  if (a.expert_map) {
    if (a.router_logits) return MTP_ERR_ARG;
    if (a.global_num_experts < 1 || a.global_num_experts > 65536) return MTP_ERR_SHAPE;
  }
  int b = a.shared_rows_begin, e = a.shared_rows_end;
  if (b == 0 && e == 0) e = a.num_tokens;
  if (b < 0 || b > e || e > a.num_tokens) return MTP_ERR_SHAPE;
  *sh_begin = b;
  *sh_end = e;
  return MTP_OK;
}

int mtp_host_device_pointer(const void* host_ptr, void** device_ptr) {
  if (!host_ptr || !device_ptr) return MTP_ERR_NULL;
  *device_ptr = nullptr;
  void* d = nullptr;
  if (cudaHostGetDevicePointer(&d, const_cast<void*>(host_ptr), 0) != cudaSuccess) {
    cudaGetLastError();
    return MTP_ERR_CUDA;
  }
  *device_ptr = d;
  return MTP_OK;
}

int mtp_router_topk(const float* logits, int32_t M, int32_t E, int32_t k, int32_t renormalize,
                    float* topk_weights, int32_t* topk_ids, int32_t* token_expert_indices,
                    void* stream) {
  if (!logits || !topk_weights || !topk_ids) return MTP_ERR_NULL;
  if (M < 0 || E < 1 || E > 1024 || k < 1 || k > 32 || k > E) return MTP_ERR_SHAPE;
  if (M == 0) return MTP_OK;
  return launch_router_topk(logits, M, E, k, renormalize ? 1 : 0, topk_weights, topk_ids,
                            token_expert_indices, static_cast<cudaStream_t>(stream));
}

int mtp_moe_align_sizes(int32_t numel, int32_t num_experts, int32_t block_size,
                        int32_t pad_sorted_ids, int32_t* sorted_capacity, int32_t* max_blocks,
                        int32_t* max_segments) {
  if (!sorted_capacity || !max_blocks) return MTP_ERR_NULL;
  if (numel < 0 || num_experts < 1 || block_size < 1) return MTP_ERR_SHAPE;
  const AlignSizes s = align_sizes(numel, num_experts, block_size, pad_sorted_ids);
  *sorted_capacity = s.cap;
  *max_blocks = s.max_blocks;
  if (max_segments) *max_segments = s.max_seg;
  return MTP_OK;
}

int mtp_moe_align(const int32_t* topk_ids, int32_t numel, int32_t num_experts, int32_t block_size,
                  const int32_t* expert_map, int32_t ignore_invalid_experts, int32_t pad_sorted_ids,
                  int32_t* sorted_token_ids, int32_t* expert_ids, int32_t* num_tokens_post_padded,
                  int32_t* segments, int32_t* num_segments, void* stream) {
  if (numel < 0 || num_experts < 1 || num_experts > 1024 || block_size < 1 || block_size > 1024)
    return MTP_ERR_SHAPE;
  const AlignSizes s = align_sizes(numel, num_experts, block_size, pad_sorted_ids);
  if (!num_tokens_post_padded) return MTP_ERR_NULL;
  if ((s.cap > 0 && !sorted_token_ids) || (s.max_blocks > 0 && !expert_ids)) return MTP_ERR_NULL;
  if (numel > 0 && !topk_ids) return MTP_ERR_NULL;
  if ((segments == nullptr) != (num_segments == nullptr)) return MTP_ERR_NULL;
  if (segments && s.max_seg > 0 && !segments) return MTP_ERR_NULL;
  return launch_moe_align(topk_ids, numel, num_experts, block_size, expert_map,
                          ignore_invalid_experts ? 1 : 0, s.cap, s.max_blocks, s.max_seg,
                          sorted_token_ids, expert_ids, num_tokens_post_padded, segments,
                          num_segments, static_cast<cudaStream_t>(stream));
}

int mtp_gptq_dequant(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                     const int32_t* g_idx, int32_t K, int32_t N, int32_t group_size,
                     int32_t zero_mode, float* out, void* stream) {
  if (!qweight || !scales || !out) return MTP_ERR_NULL;
  if (zero_mode != MTP_ZERO_RAW && zero_mode != MTP_ZERO_SYM8) return MTP_ERR_ARG;
  if (zero_mode == MTP_ZERO_RAW && !qzeros) return MTP_ERR_NULL;
  if (K <= 0 || N <= 0 || K % 8 || N % 8 || group_size <= 0 || K % group_size) return MTP_ERR_SHAPE;
  return gptq_dequant(qweight, qzeros, scales, g_idx, K, N, group_size, zero_mode, out,
                      static_cast<cudaStream_t>(stream));
}

int mtp_w4a16_expert_layout(int32_t hidden, int32_t inter, int32_t group_size, MtpExpertLayout* out) {
  if (!out) return MTP_ERR_NULL;
  if (hidden <= 0 || inter <= 0 || hidden % 128 || inter % 64 || group_size % 64 ||
      hidden % group_size || inter % group_size)
    return MTP_ERR_SHAPE;
  return expert_layout(hidden, inter, group_size, out);
}

int mtp_w4a16_repack_gptq(const int32_t* w13_qweight, const int32_t* w13_qzeros,
                          const uint16_t* w13_scales, const int32_t* w2_qweight,
                          const int32_t* w2_qzeros, const uint16_t* w2_scales, int32_t num_experts,
                          int32_t hidden, int32_t inter, int32_t group_size, uint8_t* out_blobs,
                          void* stream) {
  if (!w13_qweight || !w13_qzeros || !w13_scales || !w2_qweight || !w2_qzeros || !w2_scales ||
      !out_blobs)
    return MTP_ERR_NULL;
  MtpExpertLayout L;
  const int r = mtp_w4a16_expert_layout(hidden, inter, group_size, &L);
  if (r != MTP_OK) return r;
  if (num_experts <= 0) return MTP_ERR_SHAPE;
  if (!aligned(out_blobs, 256)) return MTP_ERR_ALIGN;
  return repack_gptq(w13_qweight, w13_qzeros, w13_scales, w2_qweight, w2_qzeros, w2_scales,
                     num_experts, hidden, inter, group_size, out_blobs,
                     static_cast<cudaStream_t>(stream));
}

int mtp_w4a16_moe_layer_workspace_size(int32_t num_tokens, int32_t num_experts, int32_t top_k,
                                       int32_t hidden, int32_t inter, int64_t* bytes) {
  if (!bytes) return MTP_ERR_NULL;
  if (num_tokens < 1 || num_experts < 1 || top_k < 1 || hidden < 1 || inter < 1) return MTP_ERR_SHAPE;
  *bytes = layer_ws(num_tokens, num_experts, top_k, hidden, inter).total;
  return MTP_OK;
}

int mtp_w4a16_moe_layer(const MtpMoeLayerArgs* p, void* stream) {
  if (!p) return MTP_ERR_NULL;
  const MtpMoeLayerArgs& a = *p;
  const int M = a.num_tokens, H = a.hidden, I = a.inter, E = a.num_experts, k = a.top_k;
  const int G = a.group_size;
  if (M < 1 || E < 1 || E > 1024 || k < 1 || k > 32 || k > E) return MTP_ERR_SHAPE;
  if (H < 256 || H > 2048 || H % 256) return MTP_ERR_SHAPE;
  if (I < 128 || I > 1024 || I % 128) return MTP_ERR_SHAPE;
  if (G != 64 && G != 128) return MTP_ERR_SHAPE;
  if (I % G || H % G) return MTP_ERR_SHAPE;
  if (a.zero_mode != MTP_ZERO_RAW && a.zero_mode != MTP_ZERO_SYM8) return MTP_ERR_ARG;
  if (!a.hidden_states || !a.out || !a.workspace) return MTP_ERR_NULL;
  if (!a.expert_blobs && !(a.slot_table && a.host_blobs)) return MTP_ERR_NULL;
  if (!a.router_logits && (!a.topk_weights || !a.topk_ids)) return MTP_ERR_NULL;
  if (a.shared_blob && !a.shared_gate_weight) return MTP_ERR_NULL;
  MtpExpertLayout L;
  if (expert_layout(H, I, G, &L) != MTP_OK) return MTP_ERR_SHAPE;
  if (a.expert_bytes < L.bytes) return MTP_ERR_SHAPE;
  if (!aligned(a.hidden_states, 16) || !aligned(a.out, 8) || !aligned(a.workspace, 256) ||
      (a.expert_blobs && !aligned(a.expert_blobs, 256)) || (a.expert_bytes % 256) ||
      (a.host_blobs && !aligned(a.host_blobs, 256)) ||
      (a.shared_blob && !aligned(a.shared_blob, 256)) || (a.out_f32 && !aligned(a.out_f32, 16)))
    return MTP_ERR_ALIGN;
  int sh_begin = 0, sh_end = 0;
  if (const int r = ep_fields(a, &sh_begin, &sh_end)) return r;
  const LayerWs w = layer_ws(M, E, k, H, I);
  if (w.max_ws > kMaxWorkSegments) return MTP_ERR_SHAPE;
  if (a.workspace_bytes < w.total) return MTP_ERR_WORKSPACE;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned char* ws = static_cast<unsigned char*>(a.workspace);
  const int numel = M * k;
  if (!fused_supported(H, I, G)) return MTP_ERR_SHAPE;
  FusedArgs f;
  f.M = M; f.H = H; f.I = I; f.E = E; f.k = k; f.numel = numel; f.zero_mode = a.zero_mode;
  f.has_shared = a.shared_blob ? 1 : 0; f.G = G; f.renorm = a.renormalize ? 1 : 0;
  f.max_ws = w.max_ws;
  f.x = a.hidden_states;
  f.logits = a.router_logits;
  f.gate_w = a.shared_gate_weight;
  if (a.router_logits) {
    f.topk_w = a.topk_weights_out ? a.topk_weights_out : reinterpret_cast<float*>(ws + w.tw);
    f.topk_ids = a.topk_ids_out ? a.topk_ids_out : reinterpret_cast<int32_t*>(ws + w.tid);
  } else {
    f.topk_w = const_cast<float*>(a.topk_weights);
    // mapped ids go to the workspace (the combine phase reads local ids)
    f.topk_ids = a.expert_map ? reinterpret_cast<int32_t*>(ws + w.tid) : const_cast<int32_t*>(a.topk_ids);
  }
  f.topk_ids_in = a.router_logits ? f.topk_ids : a.topk_ids;
  f.emap = a.expert_map;
  f.E_map = a.expert_map ? a.global_num_experts : 0;
  f.sh_begin = sh_begin;
  f.sh_end = sh_end;
  f.wseg = reinterpret_cast<int32_t*>(ws + w.wseg);
  f.L = L;
  f.blobs = a.expert_blobs; f.expert_bytes = a.expert_bytes;
  f.slot_table = a.slot_table; f.host_blobs = a.host_blobs; f.shared_blob = a.shared_blob;
  f.gate = reinterpret_cast<float*>(ws + w.gate);
  f.xq = reinterpret_cast<uint8_t*>(ws + w.xq);
  f.bar = reinterpret_cast<int32_t*>(ws + w.bar);
  f.cnt = reinterpret_cast<int32_t*>(ws + w.cnt);
  f.seg_done = reinterpret_cast<int32_t*>(ws + w.seg_done);
  f.lists = reinterpret_cast<int32_t*>(ws + w.lists);
  f.gu = reinterpret_cast<float*>(ws + w.gu);
  f.ybuf = reinterpret_cast<float*>(ws + w.ybuf);
  f.out = a.out; f.out_f32 = a.out_f32;
  f.status = a.status ? a.status : reinterpret_cast<int32_t*>(ws + w.status);
  f.demand_log = a.demand_log;
  f.stages = 0; f.sk = 0; f.stage_bytes = 0; f.xbuf_bytes = 0;
  return launch_moe_fused(f, st);
}

int mtp_w4a16_moe_layer_timeouts(const void* workspace, int32_t* count, void* stream) {
  if (!workspace || !count) return MTP_ERR_NULL;
  if (!aligned(workspace, 256)) return MTP_ERR_ALIGN;
  // bar[4] of the fixed counter region (see finish_call in moe_fused.cu)
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t v = 0;
  if (cudaMemcpyAsync(&v, static_cast<const int32_t*>(workspace) + 4, sizeof(v), cudaMemcpyDeviceToHost, st) !=
          cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess) {
    cudaGetLastError();
    return MTP_ERR_CUDA;
  }
  *count = v;
  return MTP_OK;
}

int mtp_w4a16_moe_prefill_tables(int32_t num_tokens, int32_t num_experts, int32_t top_k, int32_t hidden,
                                 int32_t inter, int32_t has_shared, MtpPrefillTables* out) {
  if (!out) return MTP_ERR_NULL;
  if (num_tokens < 1 || num_experts < 1 || top_k < 1 || hidden < 1 || inter < 1) return MTP_ERR_SHAPE;
  const PrefillWs w = prefill_ws(num_tokens, num_experts, top_k, hidden, inter, has_shared ? 1 : 0);
  out->pair_expert_ids = w.ids_x;
  out->sorted_token_ids = w.sorted;
  out->expert_ids = w.eids;
  out->num_tokens_post_padded = w.ntpp;
  out->capacity = static_cast<int32_t>(w.cap);
  out->max_blocks = static_cast<int32_t>(w.max_blocks);
  out->pairs_per_token = top_k + (has_shared ? 1 : 0);
  out->block_size = static_cast<int32_t>(w.cap / w.max_blocks);
  return MTP_OK;
}

int mtp_w4a16_moe_prefill_workspace_size(int32_t num_tokens, int32_t num_experts, int32_t top_k,
                                         int32_t hidden, int32_t inter, int64_t* bytes) {
  if (!bytes) return MTP_ERR_NULL;
  if (num_tokens < 1 || num_experts < 1 || top_k < 1 || hidden < 1 || inter < 1) return MTP_ERR_SHAPE;
  *bytes = prefill_ws(num_tokens, num_experts, top_k, hidden, inter, 1).total;
  return MTP_OK;
}

int mtp_w4a16_moe_prefill(const MtpMoeLayerArgs* p, void* stream) {
  if (!p) return MTP_ERR_NULL;
  const MtpMoeLayerArgs& a = *p;
  const int M = a.num_tokens, H = a.hidden, I = a.inter, E = a.num_experts, k = a.top_k;
  const int G = a.group_size;
  const int has_shared = a.shared_blob ? 1 : 0;
  if (M < 1 || E < 1 || E + has_shared > 1024 || k < 1 || k > 32 || k > E) return MTP_ERR_SHAPE;
  if (H < 256 || H > 2048 || H % 256) return MTP_ERR_SHAPE;
  if (I < 128 || I > 1024 || I % 128) return MTP_ERR_SHAPE;
  if (G != 64 && G != 128) return MTP_ERR_SHAPE;
  if (static_cast<int64_t>(M) * (k + 1) > (1LL << 30)) return MTP_ERR_SHAPE;
  if (a.zero_mode != MTP_ZERO_RAW && a.zero_mode != MTP_ZERO_SYM8) return MTP_ERR_ARG;
  if (a.slot_table || a.demand_log) return MTP_ERR_ARG;
  if (!a.hidden_states || !a.out || !a.workspace || !a.expert_blobs) return MTP_ERR_NULL;
  if (!a.router_logits && (!a.topk_weights || !a.topk_ids)) return MTP_ERR_NULL;
  if (a.shared_blob && !a.shared_gate_weight) return MTP_ERR_NULL;
  MtpExpertLayout L;
  if (expert_layout(H, I, G, &L) != MTP_OK) return MTP_ERR_SHAPE;
  if (a.expert_bytes < L.bytes) return MTP_ERR_SHAPE;
  if (!aligned(a.hidden_states, 16) || !aligned(a.out, 16) || !aligned(a.workspace, 256) ||
      !aligned(a.expert_blobs, 256) || (a.expert_bytes % 256) || (a.shared_blob && !aligned(a.shared_blob, 256)) ||
      (a.shared_gate_weight && !aligned(a.shared_gate_weight, 16)) || (a.out_f32 && !aligned(a.out_f32, 16)))
    return MTP_ERR_ALIGN;
  int sh_begin = 0, sh_end = 0;
  if (const int r = ep_fields(a, &sh_begin, &sh_end)) return r;
  const PrefillWs w = prefill_ws(M, E, k, H, I, has_shared);
  if (a.workspace_bytes < w.total) return MTP_ERR_WORKSPACE;

  unsigned char* ws = static_cast<unsigned char*>(a.workspace);
  PrefillArgs f;
  f.M = M; f.H = H; f.I = I; f.E = E; f.k = k; f.kx = k + has_shared; f.numel_x = M * f.kx;
  f.G = G; f.zero_mode = a.zero_mode; f.has_shared = has_shared;
  f.cap = static_cast<int>(w.cap); f.max_blocks = static_cast<int>(w.max_blocks);
  f.x = a.hidden_states; f.gate_w = a.shared_gate_weight;
  if (a.router_logits) {
    f.topk_w = a.topk_weights_out ? a.topk_weights_out : reinterpret_cast<float*>(ws + w.tw);
    f.topk_ids = a.topk_ids_out ? a.topk_ids_out : reinterpret_cast<int32_t*>(ws + w.tid);
  } else {
    f.topk_w = a.topk_weights;
    f.topk_ids = a.topk_ids;
  }
  f.emap = a.expert_map;
  f.E_map = a.expert_map ? a.global_num_experts : 0;
  f.sh_begin = sh_begin;
  f.sh_end = sh_end;
  f.ids_x = reinterpret_cast<int32_t*>(ws + w.ids_x);
  f.w_x = reinterpret_cast<float*>(ws + w.w_x);
  f.inv = reinterpret_cast<int32_t*>(ws + w.inv);
  f.sorted = reinterpret_cast<int32_t*>(ws + w.sorted);
  f.eids = reinterpret_cast<int32_t*>(ws + w.eids);
  f.ntpp = reinterpret_cast<int32_t*>(ws + w.ntpp);
  f.pos_tok = reinterpret_cast<int32_t*>(ws + w.pos_tok);
  f.pos_w = reinterpret_cast<float*>(ws + w.pos_w);
  f.blk_n = reinterpret_cast<int32_t*>(ws + w.blk_n);
  f.hist = reinterpret_cast<int32_t*>(ws + w.hist);
  f.ebase = reinterpret_cast<int32_t*>(ws + w.ebase);
  f.xg = ws + w.xg;
  f.hg = ws + w.hg;
  f.y = reinterpret_cast<uint16_t*>(ws + w.y);
  f.L = L;
  f.blobs = a.expert_blobs; f.expert_bytes = a.expert_bytes; f.shared_blob = a.shared_blob;
  f.out = a.out; f.out_f32 = a.out_f32;
  f.status = a.status ? a.status : reinterpret_cast<int32_t*>(ws + w.status);
  return launch_moe_prefill(f, a.renormalize ? 1 : 0, a.router_logits, static_cast<cudaStream_t>(stream));
}


// ---- MTP expert-demand predictor ----------------------------------------------
int mtp_predictor_pack(const uint16_t* w, int32_t rows, int32_t cols, uint16_t* out, void* stream) {
  if (!w || !out) return MTP_ERR_NULL;
  if (rows <= 0 || cols <= 0 || rows % 16 || cols % 16) return MTP_ERR_SHAPE;
  if (!aligned(w, 4) || !aligned(out, 16)) return MTP_ERR_ALIGN;
  return predictor_pack(w, rows, cols, out, static_cast<cudaStream_t>(stream));
}

static bool predictor_shapes_ok(int M, int hidden, int width, int future, int experts, int k) {
  if (M < 1 || future < 1 || experts < 1 || experts > 1024 || k < 1 || k > 32 || k > experts) return false;
  if (hidden < 128 || hidden > 2048 || hidden % 128) return false;
  if (width < 128 || width > 2048 || width % 128) return false;
  return (static_cast<int64_t>(future) * experts) % 16 == 0;
}

int mtp_predictor_workspace_size(int32_t M, int32_t width, int32_t future, int32_t experts, int64_t* bytes) {
  if (!bytes) return MTP_ERR_NULL;
  if (M < 1 || width < 1 || future < 1 || experts < 1) return MTP_ERR_SHAPE;
  // fp32 partial sums of both linears, one slice per K-split
  *bytes = round_up(4LL * kMaxPredictorKs * M * width, 256) +
           round_up(4LL * kMaxPredictorKs * M * future * experts, 256);
  return MTP_OK;
}

int mtp_predict_topk(const uint16_t* h, int32_t M, int32_t hidden, const uint16_t* w1_packed, const uint16_t* b1,
                     int32_t width, const uint16_t* w2_packed, const uint16_t* b2, int32_t future, int32_t experts,
                     int32_t top_k, float* logits_out, int32_t* ids_out, void* workspace, int64_t workspace_bytes,
                     void* stream) {
  if (!h || !w1_packed || !w2_packed || !ids_out || !workspace) return MTP_ERR_NULL;
  if (!predictor_shapes_ok(M, hidden, width, future, experts, top_k)) return MTP_ERR_SHAPE;
  if (!aligned(h, 16) || !aligned(w1_packed, 16) || !aligned(w2_packed, 16) || !aligned(workspace, 256) ||
      (logits_out && !aligned(logits_out, 4)))
    return MTP_ERR_ALIGN;
  int64_t need = 0;
  mtp_predictor_workspace_size(M, width, future, experts, &need);
  if (workspace_bytes < need) return MTP_ERR_WORKSPACE;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  float* part1 = reinterpret_cast<float*>(ws);
  float* part2 = reinterpret_cast<float*>(ws + round_up(4LL * kMaxPredictorKs * M * width, 256));
  return predictor_run(h, M, hidden, w1_packed, b1, width, w2_packed, b2, future, experts, top_k, logits_out, ids_out,
                       part1, part2, static_cast<cudaStream_t>(stream));
}

int mtp_predictor_hr_workspace_size(int32_t M, int32_t width, int32_t future, int32_t experts, int64_t* bytes) {
  if (!bytes) return MTP_ERR_NULL;
  if (M < 1 || width < 1 || future < 1 || experts < 1) return MTP_ERR_SHAPE;
  *bytes = round_up(4LL * kMaxPredictorKs * M * width, 256) + round_up(2LL * M * future * width, 256) +
           round_up(4LL * kMaxPredictorKs * M * future * experts, 256);
  return MTP_OK;
}

int mtp_predict_topk_hidden_residual(const uint16_t* h, const int32_t* layer_ids, int32_t M, int32_t hidden,
                                     const uint16_t* w1_packed, const uint16_t* b1, int32_t width,
                                     const uint16_t* ln_weight, const uint16_t* ln_bias, float ln_eps,
                                     const uint16_t* layer_emb, int32_t num_layers, const uint16_t* delta_emb,
                                     int32_t future, const uint16_t* wc_packed, const uint16_t* bc, int32_t experts,
                                     int32_t top_k, float* logits_out, int32_t* ids_out, void* workspace,
                                     int64_t workspace_bytes, void* stream) {
  if (!h || !w1_packed || !wc_packed || !layer_emb || !delta_emb || !ids_out || !workspace) return MTP_ERR_NULL;
  if (!predictor_shapes_ok(M, hidden, width, future, experts, top_k) || experts % 16 || num_layers < 1 ||
      !(ln_eps > 0.f))
    return MTP_ERR_SHAPE;
  if (!aligned(h, 16) || !aligned(w1_packed, 16) || !aligned(wc_packed, 16) || !aligned(workspace, 256) ||
      (logits_out && !aligned(logits_out, 4)))
    return MTP_ERR_ALIGN;
  int64_t need = 0;
  mtp_predictor_hr_workspace_size(M, width, future, experts, &need);
  if (workspace_bytes < need) return MTP_ERR_WORKSPACE;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  const int64_t o1 = round_up(4LL * kMaxPredictorKs * M * width, 256);
  const int64_t o2 = o1 + round_up(2LL * M * future * width, 256);
  return predictor_hr_run(h, layer_ids, M, hidden, w1_packed, b1, width, ln_weight, ln_bias, ln_eps, layer_emb,
                          num_layers, delta_emb, future, wc_packed, bc, experts, top_k, logits_out, ids_out,
                          reinterpret_cast<float*>(ws), reinterpret_cast<uint16_t*>(ws + o1),
                          reinterpret_cast<float*>(ws + o2), static_cast<cudaStream_t>(stream));
}

}  // extern "C"
