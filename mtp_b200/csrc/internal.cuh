// Declarations shared between the .cu files of libmtp_b200 (not part of the ABI).
#pragma once

#include "common.cuh"

namespace mtp {

// Device-side arguments of one W4A16 MoE layer call (decode kernels).
struct MoeDevArgs {
  int M, H, I, E, k, zero_mode, numel, max_seg, has_shared;
  const uint16_t* x;          // [M, H] bf16
  const float* topk_w;        // [M*k]
  const int32_t* topk_ids;    // [M*k]
  const int32_t* sorted;      // sorted_token_ids (block size 8)
  const int32_t* segs;        // [max_seg][3] (expert, first block, block count)
  const int32_t* nseg;        // [1]
  const uint8_t* blobs;       // resident expert blobs (slot-indexed)
  int64_t expert_bytes;
  const int32_t* slot_table;  // [E] or NULL
  const uint8_t* host_blobs;  // device-mapped pinned host store or NULL
  const uint8_t* shared_blob; // or NULL
  MtpExpertLayout L;
  uint16_t* hbuf;             // [numel + M, I] bf16
  float* ybuf;                // [numel + M, H] fp32
  int32_t* status;            // [4] or NULL
};

int launch_router_topk(const float* logits, int M, int E, int k, int renorm, float* w,
                       int32_t* ids, int32_t* tei, cudaStream_t st);
int launch_moe_align(const int32_t* ids, int numel, int E, int BM, const int32_t* emap,
                     int ignore_invalid, int cap, int max_blocks, int max_seg, int32_t* sorted,
                     int32_t* eids, int32_t* ntpp, int32_t* segs, int32_t* nseg, cudaStream_t st);
int expert_layout(int hidden, int inter, int G, MtpExpertLayout* out);
int repack_gptq(const int32_t* w13q, const int32_t* w13z, const uint16_t* w13s, const int32_t* w2q,
                const int32_t* w2z, const uint16_t* w2s, int E, int H, int I, int G, uint8_t* out,
                cudaStream_t st);
int gptq_dequant(const int32_t* q, const int32_t* z, const uint16_t* s, const int32_t* gidx, int K,
                 int N, int G, int zero_mode, float* out, cudaStream_t st);
int launch_moe_decode(const MoeDevArgs& a, int G, const uint16_t* gate_w, uint16_t* out,
                      float* out_f32, int32_t* demand_log, cudaStream_t st);

}  // namespace mtp
