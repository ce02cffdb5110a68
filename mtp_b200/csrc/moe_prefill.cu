// The W4A16 MoE layer forward for prefill-sized calls (many pairs per
// expert) on sm_100a. The decode kernel (moe_fused.cu) forms MMA columns from
// blocks of 8 pairs and re-unpacks an expert's weights for every block; here
// one block holds up to 128 pairs of one expert, so each weight tile is
// unpacked once per 128 pairs and the MMA is a bf16 tile of N = 128 columns
// with fp32 accumulation over all of K in tensor memory (the vLLM fused_moe
// path the reference runs for prefill: W1, silu_and_mul, W2 with
// MUL_ROUTED_WEIGHT, moe_sum; tracing/vllm_router_trace.py:19648-19801).
//
// Launches, in stream order:
//   router   softmax / top-k / renormalise (when logits are given);
//   prep     one warp per token: the pair lists extended by the shared
//            expert as expert E (weight sigmoid(x . w_g)), inverse map reset;
//   align    moe_align_block_size with 128-pair blocks over E (+1) experts
//            in three launches (per-chunk expert counts; offsets, padding and
//            expert per block; a stable scatter per chunk): the canonical
//            order (pair index ascending inside an expert, sentinel numel);
//   gather   one CTA per block: the block's x rows (bulk-copied row by row
//            into shared memory) into the B-operand layout (below), each
//            position's token and weight, the valid column count rounded up
//            to 16 (the MMA's N for that block);
//   W1       persistent GEMM: tile = (block, row block of 64 gate + 64 up
//            rows); epilogue writes h = bf16(silu(gate) * up) in the same
//            B-operand layout for W2;
//   W2       persistent GEMM: tile = (block, row block of 128 rows of H);
//            epilogue writes y = bf16(acc * pair weight) per position;
//   combine  out[t] = bf16(sum over the token's slots in slot order, shared
//            expert last, of y in fp32).
//
// B-operand layout of a block (x for W1, h for W2; K = H or I):
//   [K/128 stages][16 column groups][16 chunks][8 columns][8 bf16]: a core
//   matrix (8 columns x 16 bytes) is 128 contiguous bytes, chunks of one
//   group are 128 bytes apart (the descriptor's K-direction offset) and
//   groups 2 KB apart (its N-direction offset); the first N columns of a
//   stage are one contiguous range of N * 256 bytes, one bulk copy.
//
// GEMM kernel (one CTA per SM, 14 warps):
//   warp 13   producer: per stage, bulk copies of the 128 x 128 int4 weight
//             tile (8 KB), its scales and zero points, and the block's
//             operand columns into a 4-deep ring;
//   warps 0-7 dequant: w = bf16((q - z) * bf16(s)) (an exact integer q - z,
//             one rounding of the product) into tensor memory, lane = weight
//             row, two k per 32-bit column: the MMA's A operand;
//   warp 12   one thread issues tcgen05.mma kind::f16 (M = 128, N = 16..128,
//             K = 16; A bf16 from tensor memory, B bf16 from shared memory,
//             D fp32 in tensor memory) for all stages of a tile into one of
//             two accumulators, and commits;
//   warps 8-11 epilogue: tcgen05.ld of the accumulator, then the W1 output
//             (gate rows handed to the up rows through shared memory) or the
//             W2 output (staged in shared memory, written 16 bytes a thread).
// Every wait is bounded by a deadline on the global timer; on expiry the
// kernel sets bit 0 of status[2] and runs to its end.
#include "internal.cuh"
#include "route.cuh"

namespace mtp {
namespace {

constexpr int kPN = 128;             // pairs per block = widest MMA N
constexpr int kPSK = 128;            // K per stage
constexpr int kPStages = 4;          // shared-memory stages = tensor-memory A tiles
constexpr int kPDq = 8;              // dequant warps 0-7
constexpr int kPMma = 12;            // MMA issue (and tensor-memory allocation)
constexpr int kPProd = 13;           // producer
constexpr int kPEpiWarp0 = 8;        // epilogue warps 8-11
constexpr int kPThreads = 14 * 32;
constexpr uint32_t kPWBytes = kPSK / 2 * 128;   // int4 weight tile of a stage
constexpr uint32_t kPXBytes = kPSK * 2 * kPN;   // operand tile of a stage (bf16)
constexpr uint32_t kPSBytes = 2 * 256;          // scales of at most two groups
constexpr uint32_t kPZBytes = 2 * 64;           // zero points of at most two groups
constexpr uint32_t kPStageBytes = kPWBytes + kPXBytes + kPSBytes + kPZBytes;
constexpr uint32_t kPCtrl = 1024;
constexpr uint32_t kPGateBytes = 64 * kPN * 4;  // W1: gate rows handed to the up rows; W2: y tile
constexpr uint32_t kPSmem = kPCtrl + kPStages * kPStageBytes + kPGateBytes;
constexpr int kPACols = kPSK / 2;               // tensor-memory columns of an A tile
constexpr int kPDCol0 = kPStages * kPACols;     // two accumulators of kPN columns follow
constexpr uint32_t kPIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (8u << 24);  // D f32, A/B bf16, M = 128
constexpr uint64_t kPTimeoutNs = 2000000000ull;
constexpr int kBarPEpi = 1;                     // named barrier: the 4 epilogue warps

static_assert(kPSmem <= 227 * 1024, "shared memory");
static_assert(kPDCol0 + 2 * kPN <= 512, "tensor memory");

struct PrefillCtrl {
  uint64_t full[kPStages];    // stage landed (bulk-copy bytes)
  uint64_t empty[kPStages];   // stage free: 8 dequant warps + the MMA commit
  uint64_t afull[kPStages];   // A tile in tensor memory (8 dequant warps)
  uint64_t aempty[kPStages];  // A tile consumed (MMA commit)
  uint64_t dfull[2];          // accumulator complete (MMA commit)
  uint64_t dempty[2];         // accumulator read (4 epilogue warps)
  uint32_t tmem;
};

__device__ __forceinline__ void umma_bf16_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d),
      "r"(a), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

__device__ __forceinline__ void record_ptimeout(const PrefillArgs& a) { atomicOr(a.status + 2, 1); }

__device__ __forceinline__ const uint8_t* tile_blob(const PrefillArgs& a, int e) {
  return e >= a.E ? a.shared_blob : a.blobs + static_cast<int64_t>(e) * a.expert_bytes;
}

// Eight int4 weights of one word (k0..k0+3 in the low nibbles, k0+4..k0+7 in
// the high nibbles) -> four bf16x2 columns (k0, k0+1), ..., (k0+6, k0+7).
// 0x43 above a nibble q is the bf16 128 + q, so subtracting 128 + z leaves the
// exact integer q - z; one rounding in the multiply by the scale.
__device__ __forceinline__ void dequant_word_bf16(uint32_t w, __nv_bfloat162 zb, __nv_bfloat162 s2,
                                                  uint32_t* o) {
  const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
  const uint32_t v[4] = {__byte_perm(lo, 0x43u, 0x4140), __byte_perm(lo, 0x43u, 0x4342),
                         __byte_perm(hi, 0x43u, 0x4140), __byte_perm(hi, 0x43u, 0x4342)};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&v[j]);
    b = __hmul2(__hsub2(b, zb), s2);
    o[j] = *reinterpret_cast<const uint32_t*>(&b);
  }
}

// ---------------------------------------------------------------------------
// prep: pair lists (global ids through the expert map when one is given)
// extended by the shared expert for the rows in [sh_begin, sh_end), inverse
// map reset
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) prefill_prep_kernel(const PrefillArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= a.M) return;
  for (int j = lane; j < a.k; j += 32) {
    const int64_t src = static_cast<int64_t>(t) * a.k + j, dst = static_cast<int64_t>(t) * a.kx + j;
    int id = a.topk_ids[src];
    if (a.emap) id = id >= 0 && id < a.E_map ? a.emap[id] : -1;
    a.ids_x[dst] = id >= 0 && id < a.E ? id : -1;
    a.w_x[dst] = a.topk_w[src];
    a.inv[dst] = -1;
  }
  if (a.has_shared && (t < a.sh_begin || t >= a.sh_end)) {
    if (lane == 0) {
      const int64_t dst = static_cast<int64_t>(t) * a.kx + a.k;
      a.ids_x[dst] = -1;
      a.w_x[dst] = 0.f;
      a.inv[dst] = -1;
    }
  } else if (a.has_shared) {
    const uint4* xr = reinterpret_cast<const uint4*>(a.x + static_cast<int64_t>(t) * a.H);
    const uint4* wg = reinterpret_cast<const uint4*>(a.gate_w);
    float part = 0.f;
    for (int c = lane; c < a.H / 8; c += 32) {
      const uint4 xv = xr[c], wv = __ldg(wg + c);
      const uint32_t* xs = reinterpret_cast<const uint32_t*>(&xv);
      const uint32_t* ws = reinterpret_cast<const uint32_t*>(&wv);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        part = fmaf(__uint_as_float(xs[q] << 16), __uint_as_float(ws[q] << 16), part);
        part = fmaf(__uint_as_float(xs[q] & 0xffff0000u), __uint_as_float(ws[q] & 0xffff0000u), part);
      }
    }
    part = warp_sum(part);
    if (lane == 0) {
      const int64_t dst = static_cast<int64_t>(t) * a.kx + a.k;
      a.ids_x[dst] = a.E;
      a.w_x[dst] = 1.f / (1.f + expf(-part));
      a.inv[dst] = -1;
    }
  }
}

// ---------------------------------------------------------------------------
// align over many CTAs: the same output as align_block (route.cuh) for
// 128-pair blocks, in three launches. Pairs are cut into chunks of kAChunk;
// `hist` [chunks][ex] holds each chunk's per-expert counts, then (after the
// offsets launch) each chunk's first position inside its expert's range.
// ---------------------------------------------------------------------------
constexpr int kAChunk = 4096;

__device__ __forceinline__ int pair_key(const PrefillArgs& a, int i, int ex) {
  const int e = a.ids_x[i];
  return e >= 0 && e < ex ? e : -1;
}

__global__ void __launch_bounds__(kAlignThreads) prefill_hist_kernel(const PrefillArgs a, int ex) {
  extern __shared__ int hs[];
  for (int e = threadIdx.x; e < ex; e += kAlignThreads) hs[e] = 0;
  __syncthreads();
  const int i0 = blockIdx.x * kAChunk, i1 = min(i0 + kAChunk, a.numel_x);
  for (int i = i0 + threadIdx.x; i < i1; i += kAlignThreads) {
    const int key = pair_key(a, i, ex);
    if (key >= 0) atomicAdd(&hs[key], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < ex; e += kAlignThreads) a.hist[static_cast<int64_t>(blockIdx.x) * ex + e] = hs[e];
}

// One CTA: expert e's count and its chunks' starting offsets, the padded
// ranges (exclusive scan over experts), the expert of every block, the
// sentinel of every padding position and the number of positions used.
__global__ void __launch_bounds__(kAlignThreads) prefill_offsets_kernel(const PrefillArgs a, int ex, int nchunks) {
  __shared__ int scan_tmp[32];
  const int e = threadIdx.x;
  int cnt = 0;
  if (e < ex)
    for (int c = 0; c < nchunks; ++c) {
      const int64_t at = static_cast<int64_t>(c) * ex + e;
      const int v = a.hist[at];
      a.hist[at] = cnt;
      cnt += v;
    }
  const int padded = (cnt + kPN - 1) / kPN * kPN;
  int total;
  const int off = block_exclusive_scan(padded, &total, scan_tmp);
  if (e < ex) {
    a.ebase[e] = off;
    for (int b = off / kPN; b < (off + padded) / kPN; ++b) a.eids[b] = e;
    for (int p = off + cnt; p < off + padded; ++p) a.sorted[p] = a.numel_x;
  }
  if (e == 0) *a.ntpp = total;
}

// Stable scatter of one chunk: pair i goes to its expert's base + the chunk's
// offset + its rank among the chunk's earlier pairs of that expert.
__global__ void __launch_bounds__(kAlignThreads) prefill_scatter_kernel(const PrefillArgs a, int ex) {
  extern __shared__ int sm[];
  int* run = sm;         // [ex] next position of each expert for this chunk
  int* wcnt = sm + ex;   // [32][ex] pairs of each expert in each warp of a round
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < ex; e += kAlignThreads)
    run[e] = a.ebase[e] + a.hist[static_cast<int64_t>(blockIdx.x) * ex + e];
  for (int x = tid; x < 32 * ex; x += kAlignThreads) wcnt[x] = 0;
  __syncthreads();
  const unsigned lt_mask = (1u << lane) - 1u;
  const int i0 = blockIdx.x * kAChunk, i1 = min(i0 + kAChunk, a.numel_x);
  for (int c0 = i0; c0 < i1; c0 += kAlignThreads) {
    const int i = c0 + tid;
    const int key = i < i1 ? pair_key(a, i, ex) : -1;
    const unsigned mask = __match_any_sync(kFullMask, key);
    const int rank = __popc(mask & lt_mask);
    const int leader = __ffs(mask) - 1;
    const int cw = __popc(mask);
    if (key >= 0 && lane == leader) wcnt[warp * ex + key] = cw;
    __syncthreads();
    int base = 0;
    if (key >= 0 && lane == leader) {
      base = run[key];
      for (int w = 0; w < warp; ++w) base += wcnt[w * ex + key];
    }
    base = __shfl_sync(kFullMask, base, leader);
    if (key >= 0) a.sorted[base + rank] = i;
    __syncthreads();
    if (key >= 0 && lane == leader) {
      atomicAdd(&run[key], cw);  // several warps may hold the same expert
      wcnt[warp * ex + key] = 0;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// gather: one CTA (256 threads) per block of 128 sorted positions. Per stage
// (128 of K) each valid row's 256 bytes arrive by one 1-D bulk copy (issued by
// the row's own thread) in a row-major shared tile padded to 272 bytes a row,
// two stages in flight; the threads then write the stage's first N columns
// in the B-operand layout with 16-byte loads (conflict-free: 8 rows of a core
// matrix fall on 8 distinct bank quads) and 16-byte coalesced stores.
// ---------------------------------------------------------------------------
constexpr int kGRow = 272;                       // padded bytes per row of the tile
constexpr uint32_t kGTile = kPN * kGRow;         // one stage
constexpr uint32_t kGSmem = 2 * kGTile;

__global__ void __launch_bounds__(256) prefill_gather_kernel(const PrefillArgs a) {
  extern __shared__ __align__(128) uint8_t gsm[];
  __shared__ uint64_t gbar[2];
  const int blk = blockIdx.x;
  if (blk * kPN >= *a.ntpp) return;
  const int tid = threadIdx.x;
  int tok = -1;
  if (tid < kPN) {
    const int64_t p = static_cast<int64_t>(blk) * kPN + tid;
    const int pair = a.sorted[p];
    if (pair < a.numel_x) tok = pair / a.kx;
    a.pos_tok[p] = tok;
    a.pos_w[p] = tok >= 0 ? a.w_x[pair] : 0.f;
    if (tok >= 0) a.inv[pair] = static_cast<int>(p);
  }
  if (tid == 0) {
    mbar_init(smem_u32(&gbar[0]), 1);
    mbar_init(smem_u32(&gbar[1]), 1);
    fence_mbar_init();
  }
  // valid positions come first in a block (an expert's padding is at its end)
  const int valid = __syncthreads_count(tid < kPN && tok >= 0);
  const int n = valid <= 16 ? 16 : (valid + 15) / 16 * 16;
  if (tid == 0) a.blk_n[blk] = n;
  const uint64_t deadline = global_timer_ns() + kPTimeoutNs;
  const int nst = a.H / kPSK;
  const uint8_t* xrow = tok >= 0 ? reinterpret_cast<const uint8_t*>(a.x) + static_cast<int64_t>(tok) * a.H * 2 : nullptr;
  uint8_t* dst = a.xg + static_cast<int64_t>(blk) * kPN * a.H * 2;
  auto issue = [&](int s) {
    const int b = s & 1;
    if (tid == 0) mbar_arrive_expect_tx(smem_u32(&gbar[b]), static_cast<uint32_t>(valid) * 256);
    __syncthreads();
    if (tok >= 0) bulk_g2s(smem_u32(gsm + b * kGTile + tid * kGRow), xrow + s * 256, 256, smem_u32(&gbar[b]));
  };
  issue(0);
  for (int s = 0; s < nst; ++s) {
    const int b = s & 1;
    if (s + 1 < nst) issue(s + 1);
    const bool landed = mbar_wait(smem_u32(&gbar[b]), static_cast<uint32_t>((s >> 1) & 1), deadline);
    if (__syncthreads_or(!landed)) {
      // Timed out: issue nothing more, and before the CTA (and its shared
      // memory) goes away give the copies still in flight into both buffers,
      // stage s and stage s + 1, one more bounded wait.
      if (tid == 0) atomicOr(a.status + 2, 1);
      const uint64_t drain = global_timer_ns() + kPTimeoutNs;
      mbar_wait(smem_u32(&gbar[b]), static_cast<uint32_t>((s >> 1) & 1), drain);
      if (s + 1 < nst) mbar_wait(smem_u32(&gbar[b ^ 1]), static_cast<uint32_t>(((s + 1) >> 1) & 1), drain);
      __syncthreads();
      return;
    }
    const uint8_t* tile = gsm + b * kGTile;
    uint8_t* out = dst + static_cast<int64_t>(s) * 32768;
    for (int idx = tid; idx < n * 16; idx += 256) {
      // piece idx: column group idx / 128, chunk (idx / 8) % 16, row idx % 8
      const int row = ((idx >> 7) << 3) | (idx & 7), c = (idx >> 3) & 15;
      *reinterpret_cast<uint4*>(out + idx * 16) = lds128(smem_u32(tile + row * kGRow + c * 16));
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// GEMM roles
// ---------------------------------------------------------------------------
template <int MODE>
__device__ __forceinline__ void tile_of(const PrefillArgs& a, int t, int& blk, int& rb) {
  const int rbs = MODE == 0 ? a.I / 64 : a.H / 128;
  blk = t / rbs;
  rb = t - blk * rbs;
}

template <int MODE>
__device__ void prefill_producer(const PrefillArgs& a, PrefillCtrl& cb, uint8_t* stages, int ntiles,
                                 uint64_t deadline) {
  const int K = MODE == 0 ? a.H : a.I;
  const int nst = K / kPSK, gps = kPSK / a.G;
  const int64_t wo = MODE == 0 ? a.L.w13_qweight : a.L.w2_qweight;
  const int64_t so = MODE == 0 ? a.L.w13_scales : a.L.w2_scales;
  const int64_t zo = MODE == 0 ? a.L.w13_zeros : a.L.w2_zeros;
  const uint8_t* ops = MODE == 0 ? a.xg : a.hg;
  int st = 0;
  uint32_t ph = 0;
  int64_t issued = 0;
  for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
    int blk, rb;
    tile_of<MODE>(a, t, blk, rb);
    const uint8_t* blob = tile_blob(a, a.eids[blk]);
    const int ngroups = a.blk_n[blk] / 8;
    const uint8_t* wsrc = blob + wo + static_cast<int64_t>(rb) * (K / 32) * 2048;
    const uint8_t* ssrc = blob + so + static_cast<int64_t>(rb) * (K / a.G) * 256;
    const uint8_t* zsrc = blob + zo + static_cast<int64_t>(rb) * (K / a.G) * 64;
    const uint8_t* xsrc = ops + static_cast<int64_t>(blk) * kPN * K * 2;
    for (int s = 0; s < nst; ++s) {
      if (!mbar_wait(smem_u32(&cb.empty[st]), ph ^ 1u, deadline)) record_ptimeout(a);
      const uint32_t sb = smem_u32(stages + st * kPStageBytes);
      const uint32_t bar = smem_u32(&cb.full[st]);
      mbar_arrive_expect_tx(bar, kPWBytes + gps * 320 + ngroups * 2048);
      bulk_g2s(sb, wsrc + static_cast<int64_t>(s) * kPWBytes, kPWBytes, bar);
      bulk_g2s(sb + kPWBytes + kPXBytes, ssrc + static_cast<int64_t>(s) * gps * 256, gps * 256, bar);
      bulk_g2s(sb + kPWBytes + kPXBytes + kPSBytes, zsrc + static_cast<int64_t>(s) * gps * 64, gps * 64, bar);
      bulk_g2s(sb + kPWBytes, xsrc + static_cast<int64_t>(s) * 32768, ngroups * 2048, bar);
      ++issued;
      if (++st == kPStages) {
        st = 0;
        ph ^= 1u;
      }
    }
  }
  // no bulk copy may still be writing shared memory when the CTA exits (the
  // consumers waited for every stage unless a wait timed out)
  const uint64_t drain = global_timer_ns() + 100000000ull;
  for (int64_t j = issued - 1; j >= 0 && j >= issued - kPStages; --j)
    if (!mbar_wait(smem_u32(&cb.full[j % kPStages]), static_cast<uint32_t>((j / kPStages) & 1), drain))
      record_ptimeout(a);
}

template <int MODE>
__device__ void prefill_dequant(const PrefillArgs& a, PrefillCtrl& cb, const uint8_t* stages, uint32_t tmem,
                                int ntiles, uint64_t deadline) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quad = warp & 3, half = warp >> 2;
  const int r = 32 * quad + lane;
  const int K = MODE == 0 ? a.H : a.I;
  const int nst = K / kPSK;
  const int gl = a.G == 64 ? half : 0;  // this thread's group inside the stage
  const uint32_t trow = tmem + (static_cast<uint32_t>(32 * quad) << 16) + 32 * half;
  int st = 0;
  uint32_t ph = 0;
  for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
    for (int s = 0; s < nst; ++s) {
      if (!mbar_wait(smem_u32(&cb.full[st]), ph, deadline) && lane == 0) record_ptimeout(a);
      const uint8_t* sb = stages + st * kPStageBytes;
      const uint4 w0 = lds128(smem_u32(sb + (2 * half) * 2048 + r * 16));
      const uint4 w1 = lds128(smem_u32(sb + (2 * half + 1) * 2048 + r * 16));
      const float sc = __half2float(reinterpret_cast<const __half*>(sb + kPWBytes + kPXBytes)[gl * 128 + r]);
      int z = 8;
      if (a.zero_mode == MTP_ZERO_RAW) z = (sb[kPWBytes + kPXBytes + kPSBytes + gl * 64 + (r >> 1)] >> (4 * (r & 1))) & 15;
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&cb.empty[st]));
      const uint32_t zbits = 0x4300u | static_cast<uint32_t>(z);
      const uint32_t zz = zbits | (zbits << 16);
      const __nv_bfloat162 zb = *reinterpret_cast<const __nv_bfloat162*>(&zz);
      const __nv_bfloat162 s2 = __float2bfloat162_rn(sc);
      uint32_t o[16];
      if (!mbar_wait(smem_u32(&cb.aempty[st]), ph ^ 1u, deadline) && lane == 0) record_ptimeout(a);
      tc_fence_after();
      dequant_word_bf16(w0.x, zb, s2, o + 0);
      dequant_word_bf16(w0.y, zb, s2, o + 4);
      dequant_word_bf16(w0.z, zb, s2, o + 8);
      dequant_word_bf16(w0.w, zb, s2, o + 12);
      tmem_st16(trow + st * kPACols, o);
      dequant_word_bf16(w1.x, zb, s2, o + 0);
      dequant_word_bf16(w1.y, zb, s2, o + 4);
      dequant_word_bf16(w1.z, zb, s2, o + 8);
      dequant_word_bf16(w1.w, zb, s2, o + 12);
      tmem_st16(trow + st * kPACols + 16, o);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&cb.afull[st]));
      if (++st == kPStages) {
        st = 0;
        ph ^= 1u;
      }
    }
  }
}

template <int MODE>
__device__ void prefill_mma(const PrefillArgs& a, PrefillCtrl& cb, const uint8_t* stages, uint32_t tmem,
                            int ntiles, uint64_t deadline) {
  const int K = MODE == 0 ? a.H : a.I;
  const int nst = K / kPSK;
  int st = 0, db = 0;
  uint32_t ph = 0, dph = 0;
  for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
    int blk, rb;
    tile_of<MODE>(a, t, blk, rb);
    const uint32_t idesc = kPIdesc | (static_cast<uint32_t>(a.blk_n[blk] >> 3) << 17);
    if (!mbar_wait(smem_u32(&cb.dempty[db]), dph ^ 1u, deadline)) record_ptimeout(a);
    tc_fence_after();
    const uint32_t d = tmem + kPDCol0 + db * kPN;
    for (int s = 0; s < nst; ++s) {
      if (!mbar_wait(smem_u32(&cb.afull[st]), ph, deadline)) record_ptimeout(a);
      tc_fence_after();
      const uint32_t at = tmem + st * kPACols;
      // B: column group g at +2048 g (SBO), chunk c of 8 k at +128 c (LBO);
      // K step j (16 k = 2 chunks) starts 256 bytes further (start field +16)
      const uint64_t desc0 = smem_desc_kmajor(smem_u32(stages + st * kPStageBytes + kPWBytes), 128, 2048);
#pragma unroll
      for (int j = 0; j < kPSK / 16; ++j) umma_bf16_ts(d, at + j * 8, desc0 + 16 * j, idesc, (s | j) != 0);
      umma_commit(smem_u32(&cb.aempty[st]));
      umma_commit(smem_u32(&cb.empty[st]));
      if (++st == kPStages) {
        st = 0;
        ph ^= 1u;
      }
    }
    umma_commit(smem_u32(&cb.dfull[db]));
    if (++db == 2) {
      db = 0;
      dph ^= 1u;
    }
  }
}

template <int MODE>
__device__ void prefill_epilogue(const PrefillArgs& a, PrefillCtrl& cb, float* gbuf, uint32_t tmem, int ntiles,
                                 uint64_t deadline) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quad = warp & 3;
  int db = 0;
  uint32_t dph = 0;
  for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
    int blk, rb;
    tile_of<MODE>(a, t, blk, rb);
    const int n = a.blk_n[blk];
    float wl = 0.f, wnext[kPN / 32];
    if (MODE == 1) {
      // the pair weights of the tile's columns, loaded before the wait
#pragma unroll
      for (int q = 0; q < kPN / 32; ++q)
        wnext[q] = 32 * q < n ? a.pos_w[static_cast<int64_t>(blk) * kPN + 32 * q + lane] : 0.f;
    }
    if (!mbar_wait(smem_u32(&cb.dfull[db]), dph, deadline) && lane == 0) record_ptimeout(a);
    tc_fence_after();
    const uint32_t dt = tmem + (static_cast<uint32_t>(32 * quad) << 16) + kPDCol0 + db * kPN;
    uint32_t v[16];
    if (MODE == 0) {
      if (quad < 2) {
        // gate rows: hand them to the up rows through shared memory ([column][row])
        for (int c = 0; c < n; c += 16) {
          tmem_ld16(dt + c, v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) gbuf[(c + j) * 64 + 32 * quad + lane] = __uint_as_float(v[j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&cb.dempty[db]));
        named_bar_sync(kBarPEpi, 128);
        named_bar_sync(kBarPEpi, 128);
      } else {
        named_bar_sync(kBarPEpi, 128);
        const int i = 32 * (quad - 2) + lane;  // column of h inside the row block
        const int ig = 64 * rb + i;
        uint8_t* hb = a.hg + static_cast<int64_t>(blk) * kPN * a.I * 2 + (ig >> 7) * 32768 + ((ig >> 3) & 15) * 128 +
                      (ig & 7) * 2;
        for (int c = 0; c < n; c += 16) {
          tmem_ld16(dt + c, v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int col = c + j;
            const float g = gbuf[col * 64 + i];
            const float h = silu_fast(g) * __uint_as_float(v[j]);
            *reinterpret_cast<__nv_bfloat16*>(hb + (col >> 3) * 2048 + (col & 7) * 16) =
                __float2bfloat16_rn(h);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&cb.dempty[db]));
        named_bar_sync(kBarPEpi, 128);
      }
    } else {
      // y rows of the block's positions: the tile (128 rows of H x n columns)
      // is staged in shared memory as [column][128 rows] bf16, then each
      // column's 256 contiguous bytes are written with 16-byte stores
      const int r = 32 * quad + lane;
      uint16_t* stg = reinterpret_cast<uint16_t*>(gbuf);
#pragma unroll
      for (int c = 0; c < kPN; c += 16) {
        if (c >= n) break;
        if ((c & 31) == 0) wl = wnext[c >> 5];
        tmem_ld16(dt + c, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float w = __shfl_sync(kFullMask, wl, (c & 16) + j);
          stg[(c + j) * 128 + r] = __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(v[j]) * w));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&cb.dempty[db]));
      named_bar_sync(kBarPEpi, 128);
      const int et = threadIdx.x - 32 * kPEpiWarp0;
      uint16_t* yb = a.y + static_cast<int64_t>(blk) * kPN * a.H + 128 * rb;
      for (int idx = et; idx < n * 16; idx += 128) {
        const int col = idx >> 4, piece = idx & 15;
        *reinterpret_cast<uint4*>(yb + static_cast<int64_t>(col) * a.H + piece * 8) =
            lds128(smem_u32(stg + col * 128 + piece * 8));
      }
      named_bar_sync(kBarPEpi, 128);
    }
    if (++db == 2) {
      db = 0;
      dph ^= 1u;
    }
  }
}

template <int MODE>
__global__ void __launch_bounds__(kPThreads, 1) prefill_gemm_kernel(const PrefillArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  PrefillCtrl& cb = *reinterpret_cast<PrefillCtrl*>(smem);
  uint8_t* stages = smem + kPCtrl;
  float* gbuf = reinterpret_cast<float*>(smem + kPCtrl + kPStages * kPStageBytes);
  const int warp = threadIdx.x >> 5;
  const uint64_t deadline = global_timer_ns() + kPTimeoutNs;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kPStages; ++i) {
      mbar_init(smem_u32(&cb.full[i]), 1);
      mbar_init(smem_u32(&cb.empty[i]), kPDq + 1);
      mbar_init(smem_u32(&cb.afull[i]), kPDq);
      mbar_init(smem_u32(&cb.aempty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&cb.dfull[i]), 1);
      mbar_init(smem_u32(&cb.dempty[i]), 4);
    }
    fence_mbar_init();
  }
  if (warp == kPMma) {
    tmem_alloc(smem_u32(&cb.tmem), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = cb.tmem;
  const int rbs = MODE == 0 ? a.I / 64 : a.H / 128;
  const int ntiles = (*a.ntpp / kPN) * rbs;
  if (warp == kPProd) {
    if ((threadIdx.x & 31) == 0) prefill_producer<MODE>(a, cb, stages, ntiles, deadline);
  } else if (warp == kPMma) {
    if ((threadIdx.x & 31) == 0) prefill_mma<MODE>(a, cb, stages, tmem, ntiles, deadline);
  } else if (warp < kPDq) {
    prefill_dequant<MODE>(a, cb, stages, tmem, ntiles, deadline);
  } else {
    prefill_epilogue<MODE>(a, cb, gbuf, tmem, ntiles, deadline);
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kPMma) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// combine: one CTA of H / 8 threads per token
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) prefill_combine_kernel(const PrefillArgs a) {
  const int t = blockIdx.x;
  const int h8 = threadIdx.x * 8;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < a.kx; ++j) {
    const int p = a.inv[static_cast<int64_t>(t) * a.kx + j];
    if (p < 0) continue;
    const uint4 v = *reinterpret_cast<const uint4*>(a.y + static_cast<int64_t>(p) * a.H + h8);
    const uint32_t* vs = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      acc[2 * q] += __uint_as_float(vs[q] << 16);
      acc[2 * q + 1] += __uint_as_float(vs[q] & 0xffff0000u);
    }
  }
  uint4 o;
  uint32_t* os = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * q], acc[2 * q + 1]);
    os[q] = *reinterpret_cast<const uint32_t*>(&b);
  }
  *reinterpret_cast<uint4*>(a.out + static_cast<int64_t>(t) * a.H + h8) = o;
  if (a.out_f32) {
    float4* of = reinterpret_cast<float4*>(a.out_f32 + static_cast<int64_t>(t) * a.H + h8);
    of[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    of[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
}

}  // namespace

PrefillWs prefill_ws(int M, int E, int k, int H, int I, int has_shared) {
  PrefillWs w;
  const int64_t kx = k + (has_shared ? 1 : 0);
  const int64_t numel_x = static_cast<int64_t>(M) * kx;
  const int64_t ex = E + (has_shared ? 1 : 0);
  w.cap = round_up(numel_x + ex * (kPN - 1), kPN);
  w.max_blocks = w.cap / kPN;
  int64_t o = 0;
  auto take = [&](int64_t bytes) {
    const int64_t at = o;
    o = round_up(o + bytes, 256);
    return at;
  };
  w.tw = take(static_cast<int64_t>(M) * k * 4);
  w.tid = take(static_cast<int64_t>(M) * k * 4);
  w.ids_x = take(numel_x * 4);
  w.w_x = take(numel_x * 4);
  w.inv = take(numel_x * 4);
  w.sorted = take(w.cap * 4);
  w.eids = take(w.max_blocks * 4);
  w.ntpp = take(16);
  w.pos_tok = take(w.cap * 4);
  w.pos_w = take(w.cap * 4);
  w.blk_n = take(w.max_blocks * 4);
  w.nchunks = (numel_x + kAChunk - 1) / kAChunk;
  w.hist = take(w.nchunks * ex * 4);
  w.ebase = take(ex * 4);
  w.status = take(16);
  w.xg = take(w.cap * H * 2);
  w.hg = take(w.cap * I * 2);
  w.y = take(w.cap * H * 2);
  w.total = o;
  return w;
}

int launch_moe_prefill(PrefillArgs& a, int renorm, const float* logits, cudaStream_t st) {
  static int configured_device = -1;
  static int num_sms = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MTP_ERR_CUDA;
  if (configured_device != dev) {
    if (cudaFuncSetAttribute(prefill_gather_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kGSmem)) != cudaSuccess ||
        cudaFuncSetAttribute(prefill_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(33 * 1024 * sizeof(int))) != cudaSuccess ||
        cudaFuncSetAttribute(prefill_gemm_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kPSmem)) != cudaSuccess ||
        cudaFuncSetAttribute(prefill_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kPSmem)) != cudaSuccess ||
        cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return MTP_ERR_CUDA;
    configured_device = dev;
  }
  if (logits) {
    const int rc = launch_router_topk(logits, a.M, a.E, a.k, renorm, const_cast<float*>(a.topk_w),
                                      const_cast<int32_t*>(a.topk_ids), nullptr, st);
    if (rc != MTP_OK) return rc;
  }
  prefill_prep_kernel<<<(a.M + 7) / 8, 256, 0, st>>>(a);
  if (cudaGetLastError() != cudaSuccess) return MTP_ERR_LAUNCH;
  const int ex = a.E + a.has_shared;
  const int nchunks = (a.numel_x + kAChunk - 1) / kAChunk;
  prefill_hist_kernel<<<nchunks, kAlignThreads, ex * sizeof(int), st>>>(a, ex);
  prefill_offsets_kernel<<<1, kAlignThreads, 0, st>>>(a, ex, nchunks);
  prefill_scatter_kernel<<<nchunks, kAlignThreads, 33 * ex * sizeof(int), st>>>(a, ex);
  prefill_gather_kernel<<<a.max_blocks, 256, kGSmem, st>>>(a);
  prefill_gemm_kernel<0><<<num_sms, kPThreads, kPSmem, st>>>(a);
  prefill_gemm_kernel<1><<<num_sms, kPThreads, kPSmem, st>>>(a);
  prefill_combine_kernel<<<a.M, a.H / 8, 0, st>>>(a);
  return launch_status();
}

}  // namespace mtp
