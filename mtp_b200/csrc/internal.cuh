// Declarations shared between the .cu files of libmtp_b200 (not part of the ABI).
#pragma once

#include "common.cuh"

namespace mtp {

// Work segment: kWsBlocks token block(s) of one expert (or of the shared
// expert), written by the route kernel and copied into shared memory by the
// fused kernel. 12 ints = 48 bytes (16-byte multiple). One block per segment
// lets every unit of a segment reuse the same operand rows.
constexpr int kWsBlocks = 1;
constexpr int kWsInts = 4 + 8 * kWsBlocks;
//   [0..1] expert blob address (0 = missing), [2] block count,
//   [3] flags (bit 0 shared expert, bit 1 blob in host memory),
//   [4..] pair ids (row of h / y), -1 for padding.

// One quantised x row: H high-digit bytes, H low-digit bytes, the per-group sums
// of the 16-bit values (int32, room for groups of 64), the row scale (fp32)
// and padding to 16 bytes. The meta travels with the row in one bulk copy.
__host__ __device__ constexpr uint32_t xq_row_bytes(int H) {
  return 2u * static_cast<uint32_t>(H) + static_cast<uint32_t>(H) / 16u + 16u;
}

// Device-side arguments of the fused layer kernel (moe_fused.cu).
struct FusedArgs {
  int M, H, I, E, k, numel, zero_mode, has_shared, G, renorm, max_ws;
  const uint16_t* x;
  const float* logits;       // [M, E] or NULL (topk_w / topk_ids given)
  const uint16_t* gate_w;    // [H] shared-expert gate or NULL
  float* topk_w;             // [M*k] written when logits != NULL
  int32_t* topk_ids;         // [M*k] local ids (written when logits != NULL or emap != NULL)
  const int32_t* topk_ids_in;  // [M*k] the caller's ids (global when emap != NULL)
  const int32_t* emap;       // [E_map] global -> local expert or -1; NULL: ids are local
  int E_map;
  int sh_begin, sh_end;      // rows that get the shared expert
  int32_t* wseg;             // [max_ws][kWsInts] spill area for large ranges
  MtpExpertLayout L;
  const uint8_t* blobs;
  int64_t expert_bytes;
  const int32_t* slot_table;
  const uint8_t* host_blobs;
  const uint8_t* shared_blob;
  float* gate;               // [M] sigmoid(x . w_g)
  uint8_t* xq;               // [M][xq_row_bytes(H)] quantised x rows, see xq_row_bytes
  int32_t* bar;              // [8] grid-barrier count, (unused),       \ zero before the first
                             //     CTAs done, dirty flag, timeouts seen |
  int32_t* cnt;              // [E] pairs per expert                    |  call; every call
  int32_t* seg_done;         // [max_ws] W1 units published per segment /  leaves them zero
  int32_t* lists;            // [E][M] pair ids per expert
  float* gu;                 // [numel + M][2I + 4] fp32 W1 sums per pair: gate | up, combine weight
  float* ybuf;
  uint16_t* out;
  float* out_f32;
  int32_t* status;
  int32_t* demand_log;
  int stages, sk;             // weight stages in the ring, K per stage
  uint32_t stage_bytes;
  uint32_t xbuf_bytes;
};

// Fixed counter regions of the layer workspace (see capi.cu layer_ws).
constexpr int kMaxExpertsWs = 1024;
constexpr int kMaxWorkSegments = 32768;

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

int predictor_pack(const uint16_t* w, int rows, int cols, uint16_t* out, cudaStream_t st);
// K-splits of the predictor's linears are at most this (workspace sizing).
constexpr int kMaxPredictorKs = 8;
int predictor_run(const uint16_t* h, int M, int H, const uint16_t* w1p, const uint16_t* b1, int width,
                  const uint16_t* w2p, const uint16_t* b2, int F, int E, int k, float* logits, int32_t* ids,
                  float* part1, float* part2, cudaStream_t st);
int predictor_hr_run(const uint16_t* h, const int32_t* layer_ids, int M, int H, const uint16_t* w1p,
                     const uint16_t* b1, int width, const uint16_t* ln_w, const uint16_t* ln_b, float eps,
                     const uint16_t* layer_emb, int num_layers, const uint16_t* delta_emb, int F,
                     const uint16_t* wcp, const uint16_t* bc, int E, int k, float* logits, int32_t* ids, float* part1,
                     uint16_t* ctx, float* part2, cudaStream_t st);

bool fused_supported(int H, int I, int G);
int fused_max_work_segments(int M, int max_seg, int max_blocks);
int launch_moe_fused(const FusedArgs& a, cudaStream_t st);

// Prefill path (moe_prefill.cu): pairs per expert in blocks of 128.
struct PrefillArgs {
  int M, H, I, E, k, kx, numel_x, G, zero_mode, has_shared;
  int cap, max_blocks;         // sorted capacity and blocks (align sizes for 128-pair blocks)
  const uint16_t* x;           // [M, H] bf16
  const uint16_t* gate_w;      // [H] bf16 shared-expert gate or NULL
  const float* topk_w;         // [M, k]
  const int32_t* topk_ids;     // [M, k] (global ids when emap != NULL)
  const int32_t* emap;         // [E_map] global -> local expert or -1; NULL: ids are local
  int E_map;
  int sh_begin, sh_end;        // rows that get the shared expert
  int32_t* ids_x;              // [M, kx] pairs extended by the shared expert (id E)
  float* w_x;                  // [M, kx] pair weights (sigmoid gate for the shared expert)
  int32_t* inv;                // [M, kx] sorted position of each pair, -1 if not routed
  int32_t* sorted;             // [cap] align output
  int32_t* eids;               // [max_blocks] expert per block (E = shared)
  int32_t* ntpp;               // [1] positions used
  int32_t* pos_tok;            // [cap] token of each position, -1 for padding
  float* pos_w;                // [cap] weight of each position
  int32_t* blk_n;              // [max_blocks] valid columns rounded up to 16 (MMA N)
  int32_t* hist;               // [chunks][E (+1)] align: per-chunk counts, then offsets
  int32_t* ebase;              // [E (+1)] align: first position of each expert
  uint8_t* xg;                 // [max_blocks] blocks of x rows in the B-operand layout
  uint8_t* hg;                 // [max_blocks] blocks of h rows in the B-operand layout
  uint16_t* y;                 // [cap, H] bf16 W2 output times the pair weight
  MtpExpertLayout L;
  const uint8_t* blobs;
  int64_t expert_bytes;
  const uint8_t* shared_blob;
  uint16_t* out;
  float* out_f32;
  int32_t* status;
};

struct PrefillWs {
  int64_t cap, max_blocks, nchunks;
  int64_t tw, tid, ids_x, w_x, inv, sorted, eids, ntpp, pos_tok, pos_w, blk_n, hist, ebase, status, xg, hg, y, total;
};

PrefillWs prefill_ws(int M, int E, int k, int H, int I, int has_shared);
int launch_moe_prefill(PrefillArgs& a, int renorm, const float* logits, cudaStream_t st);

}  // namespace mtp
