// The W4A16 MoE layer forward on sm_100a as one persistent kernel (one CTA
// per SM, 16 warps). It runs in three phases separated by grid-wide barriers:
//
//   routing  CTA c routes tokens c, c + G, ... (G = CTAs): router softmax /
//            top-k / renormalise (warps 0-6, one token each) and the shared
//            expert's sigmoid gate (warps 7-13); each (token, slot) pair is
//            appended to its expert's list with an atomic counter. Pair order
//            inside a list does not change any result: every pair is its own
//            MMA column.
//   table    every CTA derives the work segments (the shared expert's token
//            blocks, then each routed expert's pairs in blocks of 8, experts
//            ascending) from the per-expert counts, and fills the entries of
//            its own unit ranges into shared memory with the blob address
//            already resolved through the slot table.
//   experts  warp-specialised pipeline over the work units, with the
//            5th-generation tensor cores (tcgen05) doing the MMAs:
//     warp 13  weight producer - streams the int4 weights, fp16 scales and
//              zero nibbles of each stage (128 rows x SK of K) of each unit
//              from HBM into a ring of shared-memory stages with 1-D bulk
//              copies completing on mbarriers;
//     warp 14  operand producer - brings the 8 bf16 rows of each token block
//              (x for W1, h for W2) into a double buffer; before the first W2
//              unit of a segment it waits until every W1 unit of that segment
//              has published its h columns;
//     warps 0-7  dequant - quantise each new block of operand rows in place to
//              16-bit integers laid out as the MMA's B operand (v = 256 hi +
//              lo with both digits signed bytes: a high and a low digit
//              plane, K-major 8x16-byte core matrices, one scale per row,
//              sums of v per quantisation group),
//              and unpack each stage's int4 weights to u8 straight into tensor
//              memory (the MMA's A operand, lane = weight row);
//     warps 12, 15  MMA issuers (alternate stages) - one thread each issues
//              tcgen05.mma kind::i8 (M=128, N=16 = the 8 rows of the high
//              digit plane then the 8 of the low one, K=32; A u8 from tensor
//              memory, B s8 from shared memory) into per-group int32
//              accumulators in tensor memory, and commits each stage to
//              mbarriers;
//     warps 8-11 epilogue - read the accumulators back (tcgen05.ld), fold
//              zero point, group scale and row scale in fp32 per group:
//              acc += s_g * (256 * D_hi + D_lo - z_g * sum_g(x)), then at the
//              end of a unit write h = silu(gate) * up (W1) or y = acc * w
//              (W2).
//   Tensor memory holds two rings: A slots (the u8 tile of one stage; freed by
//   the MMA's commit) and accumulator slots (the group accumulators of one
//   stage; freed by the epilogue), so dequant, MMA and epilogue of
//   consecutive stages overlap and the dequant warps never wait for the
//   epilogue.
//
// Work units, in this order (each CTA takes a contiguous range of each list;
// a work segment is one token block, so ranges balance and consecutive units
// of a segment reuse the same operand rows):
//   W1 unit (segment, row block b): gate rows 64b..64b+63 and up rows
//      I+64b..I+64b+63 over all of K = H -> h = silu(gate) * up (bf16) for
//      every (token, slot) pair of the segment (vLLM fused_moe W1 +
//      silu_and_mul, tracing/vllm_router_trace.py:19674-19719).
//   W2 unit (segment, row block b): down rows 128b..128b+127 over K = I ->
//      y = h . W2^T times the router weight (MUL_ROUTED_WEIGHT, :19761-19782),
//      fp32 per pair.
// Then a second grid-wide barrier, after which every CTA combines a slice of
// the output and clears a slice of the per-call counters: out = sum over the
// top-k slots in slot order of y + sigmoid(x . w_g) * y_shared (moe_sum :19801
// and the shared-expert gate :3994-4031, :4140-4152), so the result is
// deterministic.
//
// Cross-CTA dependencies go through release/acquire counters. Units never
// wait on later units and the final barrier is reached by every CTA after
// its own units, so with all CTAs resident (one per SM, sized by shared
// memory) nothing deadlocks. Every wait is bounded by a deadline on the
// global timer; on expiry the kernel sets bit 0 (value 1) of status[2] and
// carries on, so it always terminates. A caller-given top-k row that repeats
// an expert sets value 4 (the repeat is dropped).
#include "internal.cuh"

namespace mtp {

constexpr int kFBM = 8;             // pairs per token block = MMA N
constexpr int kDQ = 8;              // dequant warps 0-7
constexpr int kEpi0 = 8;            // epilogue warps 8-11
constexpr int kMmaWarp = 12;        // MMA issue: even stages (and the tensor-memory allocation)
constexpr int kWProd = 13;          // weight producer warp
constexpr int kBProd = 14;          // operand producer warp
constexpr int kMmaWarp2 = 15;       // MMA issue: odd stages
constexpr int kMmaIssuers = 2;
constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kRouteWarps = 7;      // warps 0-6 route, 7-13 gate
constexpr int kMaxStages = 8;
constexpr int kMaxASlots = 4;
constexpr int kMaxDSlots = 8;
constexpr int kTmemCols = 512;
__host__ __device__ constexpr int accs_for(int sk) { return sk >= 512 ? 4 : 2; }
__host__ __device__ constexpr int aslots_for(int sk) { return sk >= 512 ? 2 : 4; }
__host__ __device__ constexpr int dslot_cols(int sk) { return accs_for(sk) * 16; }
__host__ __device__ constexpr int dslots_for(int sk) {
  return (kTmemCols - aslots_for(sk) * (sk / 4)) / dslot_cols(sk) < kMaxDSlots
             ? (kTmemCols - aslots_for(sk) * (sk / 4)) / dslot_cols(sk)
             : kMaxDSlots;
}
template <int SK>
struct StageCfg {
  static constexpr int accs = accs_for(SK);
  static constexpr int aslots = aslots_for(SK);
  static constexpr int dslots = dslots_for(SK);
  static constexpr uint32_t acols = SK / 4;
  static constexpr uint32_t dbase = aslots * acols;
  static constexpr uint32_t dstride = dslot_cols(SK);
};
constexpr int kCtrlBytes = 1024;
constexpr int kWsCache = 64;        // work segments cached in shared memory per pass
constexpr int kTableBytes = 2 * kWsCache * kWsInts * 4;
constexpr int kMaxGroups = 32;      // K / G for K <= 2048, G >= 64
constexpr int kMaxStageGroups = 4;  // SK / G: 512 / 128 or 256 / 64 at most
constexpr int kSRing = 8;           // scale ring entries: a stage's group scales and zero points
constexpr int kSRingBytes = kMaxStageGroups * (256 + 64);
constexpr uint64_t kTimeoutNs = 2000000000ull;  // 2 s per layer call
constexpr int kBarDequant = 1;      // named barrier: the 8 dequant warps
constexpr int kBarEpi = 2;          // named barrier: the 4 epilogue warps
// kind::i8 instruction descriptor: int32 D, A u8, B s8, both K-major, N=16
// (the 8 high-byte rows then the 8 low-byte rows of a token block), M=128.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 10) | (2u << 17) | (8u << 24);

// ---------------------------------------------------------------------------
// shared-memory control block and the per-pass work-segment view
// ---------------------------------------------------------------------------
struct Ctrl {
  uint64_t full[kMaxStages];    // weight stage landed (tx count)
  uint64_t empty[kMaxStages];   // weight stage consumed by the dequant warps
  uint64_t xfull[2];            // operand rows landed
  uint64_t xempty[2];           // operand buffer free (one commit per MMA issuer + 4 epilogue warps)
  uint64_t qfull[2];            // operand quantised (B operand ready)
  uint64_t afull[kMaxASlots];
  uint64_t aempty[kMaxASlots];
  uint64_t dfull[kMaxDSlots];
  uint64_t dempty[kMaxDSlots];
  uint64_t drain;               // final MMA commit
  uint64_t sempty[kSRing];      // scale entry read by the 4 epilogue warps
  int scale_valid[kSRing];      // 0: the stage's expert has no weights (its terms are zero)
  int seg_first[2];   // first work segment of the pass range
  int cached[2];      // 1 if the pass range's segments are in the table
  int ub[2], ue[2];   // this CTA's unit range per pass
  int S;              // work segments of this call
  int last;           // 1 in the CTA that finished last
  uint32_t tmem;      // tensor-memory base address
  int scan[32];       // block-scan scratch
};
static_assert(sizeof(Ctrl) <= kCtrlBytes, "control block too large");

// Per operand buffer: quantisation metadata of its 8 rows.
struct OperandMeta {
  float sx[kFBM];                // row scale: x = sx * (256 * hi + lo)
  int xsum[kMaxGroups][kFBM];    // per quantisation group and row: sum of the 16-bit values
};


// Units per work segment: W1 row blocks of 64 gate + 64 up rows, W2 row blocks
// of 128 rows.
__device__ __forceinline__ int units_per_segment(const FusedArgs& a, int pass) {
  return pass == 0 ? a.I / 64 : a.H / 128;
}

struct Pass {
  int ub, ue, per;    // unit range and units per segment
  int seg_first;
  const int* table;   // smem copy of segments [seg_first, ...] or the global table
};

__device__ __forceinline__ const int* ws_entry(const Pass& P, int seg) {
  return P.table + static_cast<size_t>(seg - P.seg_first) * kWsInts;
}

__device__ __forceinline__ const uint8_t* ws_blob(const int* e) {
  const uint64_t lo = static_cast<uint32_t>(e[0]), hi = static_cast<uint32_t>(e[1]);
  return reinterpret_cast<const uint8_t*>((hi << 32) | lo);
}

// floats per gu row: gate | up sums (2I), the combine weight, padding
__device__ __forceinline__ int64_t gu_stride(const FusedArgs& a) { return 2LL * a.I + 4; }

__device__ __forceinline__ int pair_token(const FusedArgs& a, int p) {
  return p >= a.numel ? p - a.numel : p / a.k;
}

__device__ __forceinline__ void unit_range(int total_units, int& b, int& e) {
  const uint32_t g = gridDim.x, c = blockIdx.x, t = static_cast<uint32_t>(total_units);
  if (t <= 0xffffffffu / g) {  // 32-bit products: the common case, no 64-bit division
    b = static_cast<int>(t * c / g);
    e = static_cast<int>(t * (c + 1) / g);
  } else {
    b = static_cast<int>(static_cast<uint64_t>(t) * c / g);
    e = static_cast<int>(static_cast<uint64_t>(t) * (c + 1) / g);
  }
}

__device__ __forceinline__ Pass make_pass(const FusedArgs& a, const Ctrl& cb, const int* table, int pass) {
  Pass P;
  P.per = units_per_segment(a, pass);
  P.ub = cb.ub[pass];  // set by build_table
  P.ue = cb.ue[pass];
  P.seg_first = cb.seg_first[pass];
  P.table = cb.cached[pass] ? table + pass * kWsCache * kWsInts : a.wseg + static_cast<size_t>(P.seg_first) * kWsInts;
  return P;
}


// Every role walks its unit range in order, carrying unit u as (segment seg,
// row block b) and advancing it with next_unit: no division and no table read
// per unit (each one sat on a single-thread or single-warp role's critical
// path; taking them out made the kernel 8 % faster over the decode sweep). A
// unit reuses the operand buffer of the previous unit when both belong to the
// same segment, i.e. when u != ub and b != 0; the next unit does when
// u + 1 < ue and b + 1 != units per segment.
static_assert(kWsBlocks == 1, "a work segment is one token block");
__device__ __forceinline__ void next_unit(const Pass& P, int& seg, int& b) {
  if (++b == P.per) {
    b = 0;
    ++seg;
  }
}

// A wait ran out: report it (status bit 0) and mark the workspace so that the
// CTA finishing last clears every counter region for the next call.
__device__ __forceinline__ void record_timeout(const FusedArgs& a) {
  atomicOr(a.status + 2, 1);
  atomicExch(a.bar + 3, 1);
}

// The CTA that finishes last (arrival counter bar[2]) resets the grid-barrier
// count bar[0] and checks the dirty flag bar[3]: after a call in which any
// wait ran out, counters may be left anywhere (a barrier that gave up, late
// arrivals), so it clears every counter region in full, counts the event in
// bar[4] and rearms the flag. One timed-out call therefore does not disturb
// the next.
__device__ void finish_call(const FusedArgs& a, int* last_flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    *last_flag = atom_acq_rel_gpu_add(a.bar + 2, 1) == static_cast<int>(gridDim.x) - 1;
  }
  __syncthreads();
  if (!*last_flag) return;
  if (ld_acquire_gpu(a.bar + 3) != 0) {
    for (int i = threadIdx.x; i < kMaxExpertsWs; i += blockDim.x) a.cnt[i] = 0;
    for (int i = threadIdx.x; i < kMaxWorkSegments; i += blockDim.x) a.seg_done[i] = 0;
    __syncthreads();
    if (threadIdx.x == 0) {
      a.bar[4] += 1;
      a.bar[3] = 0;
    }
  }
  if (threadIdx.x == 0) {
    // every CTA has passed both grid barriers (it arrived here after them)
    a.bar[0] = 0;
    __threadfence();
    a.bar[2] = 0;
  }
}

// Grid-wide barrier number n (1, 2) of a call over the kernel's CTAs (all
// resident: one per SM). One thread per CTA calls it. The arrival count
// a.bar[0] only grows during a call (the CTA that finishes last sets it back
// to 0, see finish_call), so barrier n is passed once it reaches n x CTAs.
// Arrivals are fire-and-forget reductions: no CTA waits for its own atomic's
// round trip behind the others'.
__device__ __forceinline__ bool grid_sync(const FusedArgs& a, int n, uint64_t deadline) {
  // the arrival releases this CTA's writes (ordered before it by the CTA
  // barrier); the acquiring load that sees the full count acquires everyone's
  red_release_gpu_add(a.bar, 1);
  const int target = n * static_cast<int>(gridDim.x);
  while (ld_acquire_gpu(a.bar) < target) {
    if (global_timer_ns() > deadline) return false;
  }
  return true;
}

// Exclusive scan over all threads of the CTA (blockDim.x <= 1024); `tmp` is
// 32 ints of shared memory. Every thread must call it.
__device__ __forceinline__ int cta_exclusive_scan(int v, int* total, int* tmp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(kFullMask, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) tmp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int t = lane < nw ? tmp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(kFullMask, t, o);
      if (lane >= o) t += y;
    }
    tmp[lane] = t;
  }
  __syncthreads();
  const int base = warp > 0 ? tmp[warp - 1] : 0;
  *total = tmp[nw - 1];
  __syncthreads();
  return base + x - v;
}

// ---------------------------------------------------------------------------
// routing, spread over the CTAs: CTA c takes tokens c, c + G, c + 2G, ...
// ---------------------------------------------------------------------------
// Router for one token by one warp, E <= 1024 logits staged in shared memory:
// softmax over all E, top-k descending with exact ties to the lower expert
// id, optional renormalisation with the sum clamped to 1e-20 (vLLM
// topk_softmax as tracing/vllm_router_trace.py:4201-4227 restates it). Lane
// j < k returns pick j.
// Router for one token by one warp with the logits in registers (E <= 256:
// eight per lane, lane l holding ids l, l + 32, ...). Same selection as
// router_warp below: softmax over all E, top-k descending, exact ties to the
// lower expert; the probability is exp(v - max) / sum, the same operations in
// the same order as the standalone router (route.cuh router_token), so both
// give the same bits.
__device__ __forceinline__ void router_warp_regs(const float* __restrict__ row, int E, int k, int renorm,
                                                 float* w_out, int* id_out) {
  const int lane = threadIdx.x & 31;
  float x[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int i = 32 * j + lane;
    x[j] = i < E ? __ldg(row + i) : -INFINITY;
  }
  float mx = x[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) mx = fmaxf(mx, x[j]);
  mx = warp_max(mx);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (32 * j + lane < E) s += expf(x[j] - mx);
  s = warp_sum(s);
  // each lane's best untaken candidate; `taken` marks the lane's picked slots
  uint32_t taken = 0;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (32 * j + lane < E && x[j] > bv) {
      bv = x[j];
      bi = 32 * j + lane;
    }
  float my_w = 0.f, wsum = 0.f;
  int my_id = 0;
  for (int r = 0; r < k; ++r) {
    float wv = bv;
    int wi = bi;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(kFullMask, wv, o);
      const int oi = __shfl_xor_sync(kFullMask, wi, o);
      if (ov > wv || (ov == wv && oi < wi)) {
        wv = ov;
        wi = oi;
      }
    }
    const float p = expf(wv - mx) / s;
    wsum += p;
    if (lane == r) {
      my_w = p;
      my_id = wi;
    }
    if (wi < E && (wi & 31) == lane) {  // the winner's lane drops it and rescans its registers
      taken |= 1u << (wi >> 5);
      bv = -INFINITY;
      bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (!((taken >> j) & 1u) && 32 * j + lane < E && x[j] > bv) {
          bv = x[j];
          bi = 32 * j + lane;
        }
    }
  }
  if (renorm) my_w = my_w / fmaxf(wsum, 1e-20f);
  *w_out = my_w;
  *id_out = my_id;
}

__device__ __forceinline__ void router_warp(const float* __restrict__ row, int E, int k, int renorm, float* v,
                                            float* w_out, int* id_out) {
  const int lane = threadIdx.x & 31;
  float mx = -INFINITY;
  for (int base = 0; base < E; base += 256) {  // eight loads per lane in flight
    float x[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = base + 32 * j + lane;
      x[j] = i < E ? row[i] : -INFINITY;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = base + 32 * j + lane;
      if (i < E) v[i] = x[j];
      mx = fmaxf(mx, x[j]);
    }
  }
  mx = warp_max(mx);
  float s = 0.f;
  for (int i = lane; i < E; i += 32) s += expf(v[i] - mx);
  s = warp_sum(s);
  // each lane's best untaken candidate (ascending id within the lane breaks ties)
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = lane; i < E; i += 32)
    if (v[i] > bv) {
      bv = v[i];
      bi = i;
    }
  float my_w = 0.f, wsum = 0.f;
  int my_id = 0;
  for (int j = 0; j < k; ++j) {
    float wv = bv;
    int wi = bi;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(kFullMask, wv, o);
      const int oi = __shfl_xor_sync(kFullMask, wi, o);
      if (ov > wv || (ov == wv && oi < wi)) {
        wv = ov;
        wi = oi;
      }
    }
    const float p = expf(wv - mx) / s;
    wsum += p;
    if (lane == j) {
      my_w = p;
      my_id = wi;
    }
    if (wi < E && (wi & 31) == lane) {  // the winner's lane takes it and rescans its column
      v[wi] = -INFINITY;
      bv = -INFINITY;
      bi = 0x7fffffff;
      for (int i = lane; i < E; i += 32)
        if (v[i] > bv) {
          bv = v[i];
          bi = i;
        }
    }
    __syncwarp();
  }
  if (renorm) my_w = my_w / fmaxf(wsum, 1e-20f);
  *w_out = my_w;
  *id_out = my_id;
}

// Largest |v| of the 16-bit activation integers: v = 256 * hi + lo with both
// digits signed bytes (lo in [-128, 127], hi = (v + 128) >> 8) needs
// v <= 127 * 256 + 127.
constexpr float kVMax = 32639.f;

// 16-bit integers v (|v| <= kVMax) -> the signed-digit bytes hi = (v + 128) >> 8
// and lo = v - 256 * hi (the low byte of v read as signed) of four values,
// packed little-endian. sum_k q v = 256 sum_k q hi + sum_k q lo with both MMAs
// signed, so no correction term is needed.
__device__ __forceinline__ void pack_hilo(int v0, int v1, int v2, int v3, uint32_t& hw, uint32_t& lw) {
  hw = __byte_perm(__byte_perm(v0 + 128, v1 + 128, 0x0051), __byte_perm(v2 + 128, v3 + 128, 0x0051), 0x5410);
  lw = __byte_perm(__byte_perm(v0, v1, 0x0040), __byte_perm(v2, v3, 0x0040), 0x5410);
}

// Quantise one token's x row (one warp, lane holding the 8-element vectors
// lane + 32 j) to 16-bit integers v = round(x / sx), sx = max|x| / kVMax, and
// store them as a high-digit row then a low-digit row (pack_hilo), followed by
// the per-group sums of v and sx (one xq_row_bytes(H) row per token).
__device__ __forceinline__ void quantize_token(const FusedArgs& a, int t, const uint4 (&xv)[8]) {
  const int lane = threadIdx.x & 31;
  const int nvec = a.H / 8;
  float mx = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (lane + 32 * j < nvec) {
      const uint32_t m = __vmaxu2(__vmaxu2(xv[j].x & 0x7fff7fffu, xv[j].y & 0x7fff7fffu),
                                  __vmaxu2(xv[j].z & 0x7fff7fffu, xv[j].w & 0x7fff7fffu));
      mx = fmaxf(mx, fmaxf(__uint_as_float(m << 16), __uint_as_float(m & 0xffff0000u)));
    }
  }
  mx = warp_max(mx);
  const float inv = mx > 0.f ? kVMax / mx : 0.f;
  uint8_t* row = a.xq + static_cast<int64_t>(t) * xq_row_bytes(a.H);
  int32_t* gsum = reinterpret_cast<int32_t*>(row + 2 * a.H);
  const int lpg = a.G / 8;  // lanes (8-element vectors) per group: 8 or 16
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    int sum = 0;
    if (lane + 32 * j < nvec) {
      const uint32_t w[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
      int v[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        v[2 * e] = __float2int_rn(__uint_as_float(w[e] << 16) * inv);
        v[2 * e + 1] = __float2int_rn(__uint_as_float(w[e] & 0xffff0000u) * inv);
      }
      uint2 hi, lo;
      pack_hilo(v[0], v[1], v[2], v[3], hi.x, lo.x);
      pack_hilo(v[4], v[5], v[6], v[7], hi.y, lo.y);
      const int vi = lane + 32 * j;
      *reinterpret_cast<uint2*>(row + 8 * vi) = hi;
      *reinterpret_cast<uint2*>(row + a.H + 8 * vi) = lo;
#pragma unroll
      for (int e = 0; e < 8; ++e) sum += v[e];
    }
    // a group is lpg consecutive lanes of one j
    for (int o = 1; o < lpg; o <<= 1) sum += __shfl_xor_sync(kFullMask, sum, o);
    if ((lane & (lpg - 1)) == 0 && lane + 32 * j < nvec) gsum[(lane + 32 * j) / lpg] = sum;
  }
  if (lane == 0) *reinterpret_cast<float*>(row + 2 * a.H + a.H / 16) = mx / kVMax;
}

// Phase 1: route this CTA's tokens, count and list the (token, slot) pairs per
// expert, and compute the shared-expert gate. Warps 0-6 route a token each;
// warps 7-13 compute the gates of the same tokens. `scratch` holds 7 x E
// floats (the stage ring, still unused).
__device__ void route_phase(const FusedArgs& a, float* scratch) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp >= 2 * kRouteWarps) return;
  const int G = gridDim.x;
  const int slot = warp % kRouteWarps;
  for (int i0 = 0; static_cast<int64_t>(blockIdx.x) + static_cast<int64_t>(G) * i0 < a.M; i0 += kRouteWarps) {
    const int64_t t64 = static_cast<int64_t>(blockIdx.x) + static_cast<int64_t>(G) * (i0 + slot);
    if (t64 >= a.M) continue;
    const int t = static_cast<int>(t64);
    if (warp < kRouteWarps) {
      int id = -1;
      float w = 0.f;
      if (a.logits) {
        if (a.E <= 256)
          router_warp_regs(a.logits + static_cast<int64_t>(t) * a.E, a.E, a.k, a.renorm, &w, &id);
        else
          router_warp(a.logits + static_cast<int64_t>(t) * a.E, a.E, a.k, a.renorm, scratch + slot * a.E, &w, &id);
        if (lane < a.k) {
          a.topk_w[t * a.k + lane] = w;
          a.topk_ids[t * a.k + lane] = id;
        }
      } else if (lane < a.k) {
        // caller-given ids; global ones go through the expert map (-1: the
        // pair belongs to another rank) and the local ids are kept for the
        // combine phase
        id = a.topk_ids_in[t * a.k + lane];
        w = a.topk_w[t * a.k + lane];
        if (a.emap) {
          id = id >= 0 && id < a.E_map ? a.emap[id] : -1;
          a.topk_ids[t * a.k + lane] = id;
        }
      }
      // the pair's combine weight travels with its gate|up row to the W2 pass
      if (lane < a.k) a.gu[static_cast<int64_t>(t * a.k + lane) * gu_stride(a) + 2 * a.I] = w;
      if (lane < a.k && id >= 0 && id < a.E) {
        // an expert holds at most one pair per token (distinct ids per token);
        // a repeated id in a caller-given row is dropped and flagged
        const int pos = atomicAdd(a.cnt + id, 1);
        if (pos < a.M) a.lists[static_cast<int64_t>(id) * a.M + pos] = t * a.k + lane;
        else atomicOr(a.status + 2, 4);
      }
    } else {
      // The token's x row, all of a lane's 16-byte loads in flight at once:
      // quantised once for every expert that uses it (see quantize_token), and
      // sigmoid(x . w_g) for the shared expert.
      const uint4* xr = reinterpret_cast<const uint4*>(a.x + static_cast<int64_t>(t) * a.H);
      const uint4* wg = reinterpret_cast<const uint4*>(a.gate_w);
      const int nvec = a.H / 8;  // <= 256: at most 8 per lane
      uint4 xv[8], wv[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (lane + 32 * j < nvec) xv[j] = xr[lane + 32 * j];
        if (a.has_shared && lane + 32 * j < nvec) wv[j] = __ldg(wg + lane + 32 * j);
      }
      quantize_token(a, t, xv);
      if (a.has_shared && t >= a.sh_begin && t < a.sh_end) {
        float part = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (lane + 32 * j < nvec) {
            const uint32_t* xs = reinterpret_cast<const uint32_t*>(&xv[j]);
            const uint32_t* ws = reinterpret_cast<const uint32_t*>(&wv[j]);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              part = fmaf(__uint_as_float(xs[q] << 16), __uint_as_float(ws[q] << 16), part);
              part = fmaf(__uint_as_float(xs[q] & 0xffff0000u), __uint_as_float(ws[q] & 0xffff0000u), part);
            }
          }
        }
        part = warp_sum(part);
        if (lane == 0) {
          a.gate[t] = 1.f / (1.f + expf(-part));
          a.gu[static_cast<int64_t>(a.numel + t) * gu_stride(a) + 2 * a.I] = 1.f;
        }
      }
    }
  }
}

// Work segment s as a table entry (see kWsInts): the shared expert's token
// blocks first, then every routed expert in ascending id, cut into blocks of
// kFBM pairs. `cnt` / `sbase` are the per-expert pair counts and exclusive
// segment offsets in shared memory.
__device__ void fill_entry(const FusedArgs& a, int s, int shared_ws, const int* cnt, const int* sbase, int* w) {
  const uint8_t* blob = nullptr;
  int flags = 0;
  if (s < shared_ws) {
    blob = a.shared_blob;
    flags = 1;
    for (int j = 0; j < kFBM; ++j) {
      const int tk = a.sh_begin + s * kFBM + j;
      w[4 + j] = tk < a.sh_end ? a.numel + tk : -1;
    }
  } else {
    const int r = s - shared_ws;
    int lo = 0, hi = a.E - 1;  // last expert with sbase <= r
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (sbase[mid] <= r) lo = mid; else hi = mid - 1;
    }
    const int ex = lo, b = r - sbase[ex];
    for (int j = 0; j < kFBM; ++j) {
      const int idx = b * kFBM + j;
      w[4 + j] = idx < cnt[ex] ? __ldcg(a.lists + static_cast<int64_t>(ex) * a.M + idx) : -1;
    }
    const int slot = a.slot_table ? a.slot_table[ex] : ex;
    if (slot >= 0) {
      blob = a.blobs + static_cast<int64_t>(slot) * a.expert_bytes;
    } else if (a.host_blobs) {
      blob = a.host_blobs + static_cast<int64_t>(ex) * a.expert_bytes;
      flags = 2;
    }
  }
  const uint64_t addr = reinterpret_cast<uint64_t>(blob);
  w[0] = static_cast<int32_t>(addr & 0xffffffffu);
  w[1] = static_cast<int32_t>(addr >> 32);
  w[2] = 1;
  w[3] = flags;
}

// Phase 2 (all threads, after the grid barrier): every CTA derives the work
// segments from the per-expert counts and fills the table entries of its own
// two unit ranges; CTA 0 also writes the demand log and the miss counts.
// `scratch` holds 2E + 1 ints (the stage ring, still unused).
__device__ void build_table(const FusedArgs& a, Ctrl& cb, int* table, int* scratch) {
  const int tid = threadIdx.x, nt = blockDim.x;
  int* cnt = scratch;           // [E]
  int* sbase = scratch + a.E;   // [E + 1]
  // thread tid owns experts [tid * per, tid * per + per)
  const int per = (a.E + nt - 1) / nt;  // <= 3 for E <= 1024
  const int e0 = tid * per;
  int c[3] = {0, 0, 0};
  int nseg = 0, nused = 0;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    if (j < per && e0 + j < a.E) {
      c[j] = min(__ldcg(a.cnt + e0 + j), a.M);
      nseg += (c[j] + kFBM - 1) / kFBM;
      nused += c[j] > 0;
    }
  }
  int total;
  int ex = cta_exclusive_scan(nseg, &total, cb.scan);
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    if (j < per && e0 + j < a.E) {
      cnt[e0 + j] = c[j];
      sbase[e0 + j] = ex;
      ex += (c[j] + kFBM - 1) / kFBM;
    }
  }
  if (tid == 0) sbase[a.E] = total;
  const int shared_ws = a.has_shared ? (a.sh_end - a.sh_begin + kFBM - 1) / kFBM : 0;
  const int S = shared_ws + total;
  if (tid == 0) cb.S = S;
  if (blockIdx.x == 0) {
    int nall;
    int rank = cta_exclusive_scan(nused, &nall, cb.scan);
    if (a.demand_log && tid == 0) a.demand_log[0] = nall;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int e = e0 + j;
      if (j < per && e < a.E && c[j] > 0) {
        if (a.demand_log) a.demand_log[1 + rank] = e;
        ++rank;
        const int slot = a.slot_table ? a.slot_table[e] : e;
        if (slot < 0) atomicAdd(a.host_blobs ? a.status + 0 : a.status + 1, 1);
      }
    }
  }
  __syncthreads();
  // the entries of both passes' ranges at once (their list reads overlap)
  int first[2], n[2];
  bool cached[2];
  for (int pass = 0; pass < 2; ++pass) {
    const int upg = units_per_segment(a, pass);
    int ub, ue;
    unit_range(S * upg, ub, ue);
    first[pass] = ub / upg;
    const int last = ue > ub ? (ue - 1) / upg : first[pass] - 1;
    n[pass] = last - first[pass] + 1;
    cached[pass] = n[pass] <= kWsCache;
    if (tid == 0) {
      cb.seg_first[pass] = first[pass];
      cb.cached[pass] = cached[pass];
      cb.ub[pass] = ub;
      cb.ue[pass] = ue;
    }
  }
  for (int i = tid; i < n[0] + n[1]; i += nt) {
    const bool p1 = i >= n[0];
    const int j = p1 ? i - n[0] : i, f = p1 ? first[1] : first[0];
    int* w = (p1 ? cached[1] : cached[0]) ? table + ((p1 ? kWsCache : 0) + j) * kWsInts
                                          : a.wseg + static_cast<size_t>(f + j) * kWsInts;
    fill_entry(a, f + j, shared_ws, cnt, sbase, w);
  }
  __syncthreads();
}

__device__ __forceinline__ uint32_t lds8(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}

// Explicit shared-memory accesses by 32-bit shared address (the role
// functions receive plain pointers; these keep their hot loads and stores on
// the shared-memory path).
__device__ __forceinline__ uint32_t lds16(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ float ldsf(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void sts16(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(static_cast<uint16_t>(v)) : "memory");
}
__device__ __forceinline__ void sts8(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u8 [%0], %1;" ::"r"(addr), "h"(static_cast<uint16_t>(v)) : "memory");
}

__device__ __forceinline__ float4 ldg_cg_f4(const float* p) {
  float4 v;
  asm volatile("ld.global.cg.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

// ---------------------------------------------------------------------------
// producers
// ---------------------------------------------------------------------------
// Stage s of unit (pass, row block b): K range [s * SK, (s + 1) * SK) of the
// block, three contiguous byte ranges of the blob (int4 words, group scales,
// zero points).
struct Piece {
  uint32_t src_off;
  uint32_t dst_off;
  uint32_t bytes;
};

// Each stage: the int4 words into the weight ring (read and released by the
// dequant warps), the group scales and zero points into the scale ring (read
// and released by the epilogue).
__device__ void weight_producer(const FusedArgs& a, Ctrl& cb, const int* table, uint8_t* stages,
                                uint8_t* sring, uint64_t deadline) {
  const int lane = threadIdx.x & 31;
  const uint64_t policy = l2_evict_first_policy();
  int st = 0, sr = 0;
  uint32_t ph = 0, sph = 0;
  for (int pass = 0; pass < 2; ++pass) {
    const Pass P = make_pass(a, cb, table, pass);
    const int nst = (pass == 0 ? a.H : a.I) / a.sk;
    // the pass's piece geometry, computed once per pass: a stage's pieces
    // then cost two multiply-adds (no division on the producer's path)
    const int Kp = pass == 0 ? a.H : a.I;
    const uint32_t q0 = static_cast<uint32_t>(pass == 0 ? a.L.w13_qweight : a.L.w2_qweight);
    const uint32_t s0 = static_cast<uint32_t>(pass == 0 ? a.L.w13_scales : a.L.w2_scales);
    const uint32_t z0 = static_cast<uint32_t>(pass == 0 ? a.L.w13_zeros : a.L.w2_zeros);
    const uint32_t kb = Kp / 32, ks = a.sk / 32, gb = Kp / a.G, gsk = a.sk / a.G;
    const uint32_t wbytes = static_cast<uint32_t>(a.sk) * 64u, sbytes = gsk * 256u, zbytes = gsk * 64u;
    for (int u = P.ub, seg = P.ub / P.per, b = P.ub % P.per; u < P.ue; ++u, next_unit(P, seg, b)) {
      const int* e = ws_entry(P, seg);
      const uint8_t* blob = ws_blob(e);
      const bool host = (e[3] & 2) != 0;
      for (int s = 0; s < nst; ++s) {
        Piece pc[3];
        const uint32_t chunk = static_cast<uint32_t>(b) * kb + static_cast<uint32_t>(s) * ks;
        const uint32_t grp = static_cast<uint32_t>(b) * gb + static_cast<uint32_t>(s) * gsk;
        pc[0] = {q0 + chunk * 2048u, 0u, wbytes};
        pc[1] = {s0 + grp * 256u, wbytes, sbytes};
        pc[2] = {z0 + grp * 64u, wbytes + sbytes, zbytes};
        if (!mbar_wait(smem_u32(&cb.empty[st]), ph ^ 1u, deadline) && lane == 0) record_timeout(a);
        if (!mbar_wait(smem_u32(&cb.sempty[sr]), sph ^ 1u, deadline) && lane == 0) record_timeout(a);
        uint8_t* dst[3];
        dst[0] = stages + static_cast<size_t>(st) * a.stage_bytes;
        dst[1] = sring + sr * kSRingBytes;
        dst[2] = dst[1] + pc[1].bytes;
        const uint32_t full = smem_u32(&cb.full[st]);
        if (lane == 0) cb.scale_valid[sr] = blob != nullptr;
        if (blob != nullptr && !host) {
          if (lane == 0) {
            // the scales and zero points complete on the weight stage's barrier:
            // the dequant warps acquire both, the epilogue through the MMA's commit
            mbar_arrive_expect_tx(full, pc[0].bytes + pc[1].bytes + pc[2].bytes);
            for (int i = 0; i < 3; ++i)
              bulk_g2s_hint(smem_u32(dst[i]), blob + pc[i].src_off, pc[i].bytes, full, policy);
          }
        } else {
          // Pinned host memory (demand fetch over the host link): a warp copy
          // with eight 16-byte loads in flight per lane.
          if (blob != nullptr) {
            for (int i = 0; i < 3; ++i) {
              const uint8_t* src = blob + pc[i].src_off;
              uint8_t* d = dst[i];
              for (uint32_t o = lane * 16u; o < pc[i].bytes; o += 32u * 16u * 8u) {
                uint4 v[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const uint32_t oo = o + j * 512u;
                  if (oo < pc[i].bytes) v[j] = ldg_stream16(src + oo);
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const uint32_t oo = o + j * 512u;
                  if (oo < pc[i].bytes) *reinterpret_cast<uint4*>(d + oo) = v[j];
                }
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(full);
        }
        if (++st == a.stages) {
          st = 0;
          ph ^= 1u;
        }
        if (++sr == kSRing) {
          sr = 0;
          sph ^= 1u;
        }
      }
    }
  }
}

__device__ void operand_producer(const FusedArgs& a, Ctrl& cb, const int* table, uint8_t* xbufs,
                                 uint64_t deadline) {
  const int lane = threadIdx.x & 31;
  // the quantised x rows were written with ordinary stores in the routing
  // phase; order them before this thread's bulk (async proxy) reads
  fence_proxy_async_global();
  int xb = 0;
  uint32_t xph = 0;
  for (int pass = 0; pass < 2; ++pass) {
    const Pass P = make_pass(a, cb, table, pass);
    // W1: quantised x rows with their meta; W2: fp32 gate|up rows with the
    // pair's combine weight (8I + 16 bytes).
    // An odd number of 16-byte pieces per row keeps the 8 rows' pieces in
    // distinct bank groups.
    const uint32_t row_bytes = pass == 0 ? xq_row_bytes(a.H) : 8u * a.I + 16u;
    const uint32_t row_stride = row_bytes | 16u;
    int waited_seg = -1;
    for (int u = P.ub, seg = P.ub / P.per, b = P.ub % P.per; u < P.ue; ++u, next_unit(P, seg, b)) {
      if (u != P.ub && b != 0) continue;  // same segment as the previous unit
      const int* e = ws_entry(P, seg);
      if (pass == 1 && seg != waited_seg) {
        // every W1 unit of this segment has published its h columns
        if (lane == 0) {
          bool ok = true;
          const int need = units_per_segment(a, 0);
          while (ld_acquire_gpu(a.seg_done + seg) < need) {
            if (global_timer_ns() > deadline) {
              ok = false;
              break;
            }
            __nanosleep(64);
          }
          if (!ok) record_timeout(a);
          fence_proxy_async_global();
        }
        __syncwarp();
        waited_seg = seg;
      }
      if (!mbar_wait(smem_u32(&cb.xempty[xb]), xph ^ 1u, deadline) && lane == 0) record_timeout(a);
      const int p = lane < kFBM ? e[4 + lane] : -1;
      const unsigned valid = __ballot_sync(kFullMask, p >= 0);
      const uint32_t xfull = smem_u32(&cb.xfull[xb]);
      if (lane == 0) mbar_arrive_expect_tx(xfull, __popc(valid) * row_bytes);
      __syncwarp();
      if (p >= 0) {
        const uint8_t* src = pass == 0
                                 ? a.xq + static_cast<int64_t>(pair_token(a, p)) * xq_row_bytes(a.H)
                                 : reinterpret_cast<const uint8_t*>(a.gu + static_cast<int64_t>(p) * gu_stride(a));
        bulk_g2s(smem_u32(xbufs + xb * a.xbuf_bytes + lane * row_stride), src, row_bytes, xfull);
      }
      if (++xb == 2) {
        xb = 0;
        xph ^= 1u;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// dequant warps (0-7): operand quantisation and the A tiles in tensor memory
// ---------------------------------------------------------------------------
// W1 operand: the 8 token rows arrive already quantised (xq rows: K high
// digits, K low digits, group sums, scale; see quantize_token); take the
// meta out, then rearrange them in place
// into the MMA's B layout, both planes K-major in 8-row x 16-byte core
// matrices ((n, k) at (k / 16) * 128 + n * 16 + k % 16, high plane at [0, 8K),
// low plane at [8K, 16K)), and fetch each row's scale and group sums. Thread
// t moves the 16-byte pieces t + 256 i (row fastest), so both the reads and
// the writes of a warp are conflict-free. All pieces are read before the
// barrier and written after it (the output overlaps the input).
template <int G>
__device__ __forceinline__ void relayout_x_rows(const FusedArgs& a, const int* pairs, uint8_t* rows,
                                                OperandMeta& meta) {
  const int t = threadIdx.x, K = a.H;
  const int pieces = 2 * (K / 16) * kFBM;  // <= 2048: at most 8 per thread
  const int stride = static_cast<int>(xq_row_bytes(K) | 16u);
  uint4 v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int pc = t + kDQ * 32 * i;
    if (pc < pieces) {
      const int n = pc & 7, cc = pc >> 3;  // cc over both planes: plane = cc / (K / 16)
      v[i] = *reinterpret_cast<const uint4*>(rows + n * stride + cc * 16);
    }
  }
  if (t < kFBM * (K / G)) {
    const int n = t / (K / G), g = t % (K / G);
    meta.xsum[g][n] = pairs[n] >= 0 ? *reinterpret_cast<const int32_t*>(rows + n * stride + 2 * K + 4 * g) : 0;
  }
  if (t < kFBM) meta.sx[t] = pairs[t] >= 0 ? *reinterpret_cast<const float*>(rows + t * stride + 2 * K + K / 16) : 0.f;
  named_bar_sync(kBarDequant, kDQ * 32);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int pc = t + kDQ * 32 * i;
    if (pc < pieces) {
      const int n = pc & 7, cc = pc >> 3;
      const int plane = cc / (K / 16), c = cc % (K / 16);
      *reinterpret_cast<uint4*>(rows + plane * 8 * K + c * 128 + n * 16) = v[i];
    }
  }
  fence_proxy_async_shared();  // the planes are read by the tensor cores
  named_bar_sync(kBarDequant, kDQ * 32);
}

// W2 operand: the 8 pair rows arrive as fp32 W1 sums (K gate values, K up
// values, the combine weight, padding); form h = bf16(silu(gate) * up) and
// quantise it in place to 16-bit integers v = 256 * hi + lo (pack_hilo), laid
// out as the B planes above, with one scale per row (times the combine
// weight) and per-group sums of v. Dequant warp n owns row n: lane l takes
// the 16-element chunks c = l + 32 i of K, so the row maximum and the group
// sums are warp shuffles. Every warp holds its row in registers before the
// barrier, after which the planes overwrite the rows in place.
static_assert(kDQ == kFBM, "one dequant warp per operand row");

template <int G>
__device__ __forceinline__ void quantize_h_rows(uint8_t* rows, OperandMeta& meta, int K) {
  const int n = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nchunks = K / 16;  // <= 64: at most two per lane
  const uint8_t* row = rows + n * (8 * K + 16);
  uint32_t hv[2][8];           // bf16 pairs of the lane's chunks
  float mx = 0.f;
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int c = lane + 32 * it;
    if (c < nchunks) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int k0 = 16 * c + 4 * q;
        const float4 g = *reinterpret_cast<const float4*>(row + 4 * k0);
        const float4 u = *reinterpret_cast<const float4*>(row + 4 * (K + k0));
        const __nv_bfloat162 h01 = __floats2bfloat162_rn(silu_fast(g.x) * u.x, silu_fast(g.y) * u.y);
        const __nv_bfloat162 h23 = __floats2bfloat162_rn(silu_fast(g.z) * u.z, silu_fast(g.w) * u.w);
        hv[it][2 * q] = *reinterpret_cast<const uint32_t*>(&h01);
        hv[it][2 * q + 1] = *reinterpret_cast<const uint32_t*>(&h23);
        const uint32_t m0 = __vmaxu2(hv[it][2 * q] & 0x7fff7fffu, hv[it][2 * q + 1] & 0x7fff7fffu);
        mx = fmaxf(mx, fmaxf(__uint_as_float(m0 << 16), __uint_as_float(m0 & 0xffff0000u)));
      }
    }
  }
  mx = warp_max(mx);
  // the pair's combine weight (top-k weight, 1 for the shared expert) rides in
  // the row tail; read before the planes overwrite it, folded into the scale
  const float cw = *reinterpret_cast<const float*>(row + 8 * K);
  named_bar_sync(kBarDequant, kDQ * 32);
  const float inv = mx > 0.f ? kVMax / mx : 0.f;
  constexpr int cpg = G / 16;  // chunks per quantisation group: 4 or 8 consecutive lanes
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int c = lane + 32 * it;
    int sum = 0;
    if (c < nchunks) {
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int v0 = __float2int_rn(__uint_as_float(hv[it][2 * q] << 16) * inv);
        const int v1 = __float2int_rn(__uint_as_float(hv[it][2 * q] & 0xffff0000u) * inv);
        const int v2 = __float2int_rn(__uint_as_float(hv[it][2 * q + 1] << 16) * inv);
        const int v3 = __float2int_rn(__uint_as_float(hv[it][2 * q + 1] & 0xffff0000u) * inv);
        pack_hilo(v0, v1, v2, v3, hw[q], lw[q]);
        sum += v0 + v1 + v2 + v3;
      }
      const int off = c * 128 + n * 16;
      *reinterpret_cast<uint4*>(rows + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4*>(rows + 8 * K + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
    // the group's chunks are cpg consecutive lanes of one pass
#pragma unroll
    for (int o = 1; o < cpg; o <<= 1) sum += __shfl_xor_sync(kFullMask, sum, o);
    if (c < nchunks && (lane & (cpg - 1)) == 0) meta.xsum[(16 * c) / G][n] = sum;
  }
  if (lane == 0) meta.sx[n] = mx / kVMax * cw;
  fence_proxy_async_shared();  // the plane stores are read by the tensor cores
  named_bar_sync(kBarDequant, kDQ * 32);
}

template <int SK, int G>
__device__ void dequant_warps(const FusedArgs& a, Ctrl& cb, const int* table, uint8_t* stages, uint8_t* xbufs,
                              OperandMeta* metas, uint64_t deadline) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quad = warp & 3, half = warp >> 2;
  const int r = 32 * quad + lane;  // weight row = tensor-memory lane
  const uint32_t lane_addr = static_cast<uint32_t>(32 * quad) << 16;
  constexpr int chunks = SK / 32, my_chunks = chunks / 2;
  using C = StageCfg<SK>;
  const uint32_t tmem = cb.tmem;
  int st = 0, ta = 0, xb = 0;
  uint32_t ph = 0, aph = 0, xph = 0;
  for (int pass = 0; pass < 2; ++pass) {
    const Pass P = make_pass(a, cb, table, pass);
    const int K = pass == 0 ? a.H : a.I;
    const int nst = K / SK;
    for (int u = P.ub, seg = P.ub / P.per, b = P.ub % P.per; u < P.ue; ++u, next_unit(P, seg, b)) {
      // the previous / next unit of the range belongs to the same segment
      const bool reuse = u != P.ub && b != 0;
      const bool keep = u + 1 < P.ue && b + 1 != P.per;
      if (!reuse) {
        if (!mbar_wait(smem_u32(&cb.xfull[xb]), xph, deadline) && threadIdx.x == 0) record_timeout(a);
        if (pass == 0)
          relayout_x_rows<G>(a, ws_entry(P, seg) + 4, xbufs + xb * a.xbuf_bytes, metas[xb]);
        else
          quantize_h_rows<G>(xbufs + xb * a.xbuf_bytes, metas[xb], K);
        if (threadIdx.x == 0) mbar_arrive(smem_u32(&cb.qfull[xb]));
      }
      for (int s = 0; s < nst; ++s) {
        if (!mbar_wait(smem_u32(&cb.full[st]), ph, deadline) && lane == 0) record_timeout(a);
        if (!mbar_wait(smem_u32(&cb.aempty[ta]), aph ^ 1u, deadline) && lane == 0) record_timeout(a);
        tc_fence_after();
        const uint32_t sbase = smem_u32(stages + static_cast<size_t>(st) * a.stage_bytes);
        const uint32_t tcol = tmem + lane_addr + ta * C::acols;
        // the stage's words of this thread's row and K half, loaded at once so
        // the shared-memory stage can go back to the producer before the
        // unpack (a stage of an expert without weights holds stale words; the
        // epilogue gives its terms a zero scale)
        uint4 wq[my_chunks];
#pragma unroll
        for (int c = 0; c < my_chunks; ++c) wq[c] = lds128(sbase + ((half * my_chunks + c) * 128 + r) * 16);
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&cb.empty[st]));
#pragma unroll
        for (int cp = 0; cp < my_chunks; cp += 2) {
          const int c0 = half * my_chunks + cp;
          uint32_t v[16];
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            const uint32_t w4[4] = {wq[cp + cc].x, wq[cp + cc].y, wq[cp + cc].z, wq[cp + cc].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              v[cc * 8 + 2 * j] = w4[j] & 0x0F0F0F0Fu;
              v[cc * 8 + 2 * j + 1] = (w4[j] >> 4) & 0x0F0F0F0Fu;
            }
          }
          tmem_st16(tcol + c0 * 8, v);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&cb.afull[ta]));
        if (++st == a.stages) {
          st = 0;
          ph ^= 1u;
        }
        if (++ta == C::aslots) {
          ta = 0;
          aph ^= 1u;
        }
      }
      if (!keep) {
        if (++xb == 2) {
          xb = 0;
          xph ^= 1u;
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// MMA issuer (warp 12, one thread)
// ---------------------------------------------------------------------------
// Two issuing threads in warps on different SM sub-partitions take alternate
// stages: a thread that waits for its next stage's A tile (an mbarrier wait)
// lets the tensor pipe run dry, so the other thread's stage keeps it busy
// meanwhile. Both walk every unit (operand waits, slot and buffer counters)
// and each commits the operand buffer after its own MMAs of a unit.
template <int SK, int G>
__device__ void mma_issuer(const FusedArgs& a, Ctrl& cb, const int* table, uint8_t* xbufs, int which,
                           uint64_t deadline) {
  constexpr int chunks = SK / 32;
  using C = StageCfg<SK>;
  constexpr int kAccs = C::accs;
  constexpr int cpg = G / 32, subs = kAccs / (SK / G);
  const uint32_t tmem = cb.tmem;
  int ta = 0, td = 0, xb = 0, g = 0;
  uint32_t aph = 0, dph = 0, xph = 0;
  for (int pass = 0; pass < 2; ++pass) {
    const Pass P = make_pass(a, cb, table, pass);
    const int K = pass == 0 ? a.H : a.I;
    const int nst = K / SK;
    for (int u = P.ub, seg = P.ub / P.per, b = P.ub % P.per; u < P.ue; ++u, next_unit(P, seg, b)) {
      const bool reuse = u != P.ub && b != 0;
      const bool keep = u + 1 < P.ue && b + 1 != P.per;
      if (!reuse && !mbar_wait(smem_u32(&cb.qfull[xb]), xph, deadline)) record_timeout(a);
      const uint32_t xbase = smem_u32(xbufs + xb * a.xbuf_bytes);
      for (int s = 0; s < nst; ++s, ++g) {
        const int ta_s = ta, td_s = td;
        const uint32_t aph_s = aph, dph_s = dph;
        if (++ta == C::aslots) {
          ta = 0;
          aph ^= 1u;
        }
        if (++td == C::dslots) {
          td = 0;
          dph ^= 1u;
        }
        if ((g & 1) != which) continue;
        // the accumulator slot's previous stage has been read by the epilogue
        if (!mbar_wait(smem_u32(&cb.dempty[td_s]), dph_s ^ 1u, deadline)) record_timeout(a);
        if (!mbar_wait(smem_u32(&cb.afull[ta_s]), aph_s, deadline)) record_timeout(a);
        tc_fence_after();
        const uint32_t a_t = tmem + ta_s * C::acols;
        const uint32_t d_t = tmem + C::dbase + td_s * C::dstride;
        // B: 16 rows = the high plane's 8 rows, then (SBO = 8K bytes on) the low
        // plane's; chunk c of 32 k starts 256 bytes further (start field +16).
        // kAccs independent accumulators per stage, issued round robin, so an
        // MMA's latency hides behind the next one: accumulator d holds the
        // chunks c of group d / subs with c % cpg = d % subs (mod subs).
        const uint64_t desc0 = smem_desc_kmajor(xbase + s * chunks * 256, 128, 8 * K);
#pragma unroll
        for (int t = 0; t < cpg / subs; ++t) {
#pragma unroll
          for (int d = 0; d < kAccs; ++d) {
            const int c = (d / subs) * cpg + t * subs + (d % subs);
            umma_i8_ts(d_t + d * 16, a_t + c * 8, desc0 + 16 * c, kIdesc, t != 0);
          }
        }
        umma_commit(smem_u32(&cb.aempty[ta_s]));
        umma_commit(smem_u32(&cb.dfull[td_s]));
      }
      if (!keep) {
        umma_commit(smem_u32(&cb.xempty[xb]));
        if (++xb == 2) {
          xb = 0;
          xph ^= 1u;
        }
      }
    }
  }
  umma_commit(smem_u32(&cb.drain));
  if (!mbar_wait(smem_u32(&cb.drain), 0, deadline)) record_timeout(a);
}

// ---------------------------------------------------------------------------
// epilogue warps (8-11)
// ---------------------------------------------------------------------------
template <int SK, int G>
__device__ void epilogue_warps(const FusedArgs& a, Ctrl& cb, const int* table, const OperandMeta* metas,
                               const uint8_t* sring, uint64_t deadline) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quad = warp & 3;
  const int r = 32 * quad + lane;  // accumulator row = tensor-memory lane
  const uint32_t lane_addr = static_cast<uint32_t>(32 * quad) << 16;
  using C = StageCfg<SK>;
  constexpr int kAccs = C::accs;
  constexpr int gps = SK / G, subs = kAccs / gps;
  const uint32_t tmem = cb.tmem;
  int td = 0, xb = 0, sr = 0;
  uint32_t dph = 0;
  int published = 0;
  for (int pass = 0; pass < 2; ++pass) {
    const Pass P = make_pass(a, cb, table, pass);
    const int K = pass == 0 ? a.H : a.I;
    const int nst = K / SK;
    for (int u = P.ub, seg = P.ub / P.per, b = P.ub % P.per; u < P.ue; ++u, next_unit(P, seg, b)) {
      const int* e = ws_entry(P, seg);
      const bool keep = u + 1 < P.ue && b + 1 != P.per;
      const OperandMeta& meta = metas[xb];
      float acc[kFBM];
#pragma unroll
      for (int n = 0; n < kFBM; ++n) acc[n] = 0.f;
      for (int s = 0; s < nst; ++s) {
        // dfull also orders the stage's scales and zero points (they land with
        // the weight stage, which the dequant warps acquired before the MMA)
        // and the int4 sums the dequant warps put next to the accumulators
        if (!mbar_wait(smem_u32(&cb.dfull[td]), dph, deadline) && lane == 0) record_timeout(a);
        tc_fence_after();
        const uint32_t dt = tmem + lane_addr + C::dbase + td * C::dstride;
        const uint32_t xs = smem_u32(&meta.xsum[0][0]);
        const uint32_t se = smem_u32(sring + sr * kSRingBytes);
        const bool valid = cb.scale_valid[sr] != 0;
        float scs[gps];
        int zs[gps];
#pragma unroll
        for (int g = 0; g < gps; ++g) {
          scs[g] = valid ? __half2float(__ushort_as_half(static_cast<uint16_t>(lds16(se + (g * 128 + r) * 2)))) : 0.f;
          zs[g] = a.zero_mode == MTP_ZERO_RAW ? static_cast<int>((lds8(se + gps * 256 + g * 64 + (r >> 1)) >> (4 * (r & 1))) & 0xF) : 8;
        }
        // the scale entry is no longer needed: back to the producer
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&cb.sempty[sr]));
        if (++sr == kSRing) sr = 0;
        // every accumulator of the stage in flight at once, one wait (a
        // wait per accumulator costs a tensor-memory round trip each)
        uint32_t d[kAccs][16];
#pragma unroll
        for (int j = 0; j < kAccs; ++j) tmem_ld16(dt + j * 16, d[j]);
        tmem_wait_ld();
#pragma unroll
        for (int g = 0; g < gps; ++g) {
          // 256 * D_hi + D_lo summed over the group's accumulators
          int tsum[kFBM];
#pragma unroll
          for (int n = 0; n < kFBM; ++n) tsum[n] = 0;
#pragma unroll
          for (int j = 0; j < subs; ++j) {
#pragma unroll
            for (int n = 0; n < kFBM; ++n)
              tsum[n] += 256 * static_cast<int>(d[g * subs + j][n]) + static_cast<int>(d[g * subs + j][8 + n]);
          }
          const float sc = scs[g];
          const int z = zs[g];
          const int gg = s * gps + g;
          const uint4 xa = lds128(xs + gg * kFBM * 4), xb4 = lds128(xs + gg * kFBM * 4 + 16);
          const int xsv[kFBM] = {static_cast<int>(xa.x), static_cast<int>(xa.y), static_cast<int>(xa.z), static_cast<int>(xa.w),
                                 static_cast<int>(xb4.x), static_cast<int>(xb4.y), static_cast<int>(xb4.z), static_cast<int>(xb4.w)};
#pragma unroll
          for (int n = 0; n < kFBM; ++n) {
            // sum_k (q - z) v = 256 D_hi + D_lo - z sum v
            const int v = tsum[n] - z * xsv[n];
            acc[n] = fmaf(static_cast<float>(v), sc, acc[n]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&cb.dempty[td]));
        if (++td == C::dslots) {
          td = 0;
          dph ^= 1u;
        }
      }
      // the pair columns and row scales loaded together (16-byte loads) before
      // the stores, so the loads do not wait behind each store
      const int4 cq0 = *reinterpret_cast<const int4*>(e + 4), cq1 = *reinterpret_cast<const int4*>(e + 8);
      const float4 sq0 = *reinterpret_cast<const float4*>(&meta.sx[0]), sq1 = *reinterpret_cast<const float4*>(&meta.sx[4]);
      const int cols[kFBM] = {cq0.x, cq0.y, cq0.z, cq0.w, cq1.x, cq1.y, cq1.z, cq1.w};
      const float sxv[kFBM] = {sq0.x, sq0.y, sq0.z, sq0.w, sq1.x, sq1.y, sq1.z, sq1.w};
      if (pass == 0) {
        // gate rows 0-63 and up rows 64-127 of block b: fp32 sums per pair;
        // silu(gate) * up is formed when the W2 operand is loaded
        const int row = r < 64 ? 64 * b + r : a.I + 64 * b + (r - 64);
#pragma unroll
        for (int n = 0; n < kFBM; ++n) {
          const int p = cols[n];
          if (p >= 0) a.gu[static_cast<int64_t>(p) * gu_stride(a) + row] = acc[n] * sxv[n];
        }
        ++published;
        if (u + 1 == P.ue || b + 1 == P.per) {
          // every epilogue thread's stores of this segment before the release
          named_bar_sync(kBarEpi, 128);
          if (threadIdx.x == kEpi0 * 32) red_release_gpu_add(a.seg_done + seg, published);
          published = 0;
        }
      } else {
#pragma unroll
        for (int n = 0; n < kFBM; ++n) {
          const int p = cols[n];
          if (p >= 0) {
            a.ybuf[static_cast<int64_t>(p) * a.H + 128 * b + r] = acc[n] * sxv[n];
          }
        }
      }
      if (!keep) {
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&cb.xempty[xb]));
        xb ^= 1;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int SK, int G>
__global__ void __launch_bounds__(kThreads, 1) moe_fused_kernel(FusedArgs a) {
  using C = StageCfg<SK>;
  constexpr int kAccs = C::accs;
  static_assert(SK / G >= 1 && SK / G <= kAccs && kAccs % (SK / G) == 0, "a stage's groups share the accumulators");
  static_assert(SK / G <= kMaxStageGroups && C::aslots <= kMaxASlots && C::dslots <= kMaxDSlots && C::dslots >= 2, "slots");
  static_assert(C::dbase + C::dslots * C::dstride <= kTmemCols, "rings fit");
  extern __shared__ __align__(128) uint8_t smem[];
  Ctrl& cb = *reinterpret_cast<Ctrl*>(smem);
  int* table = reinterpret_cast<int*>(smem + kCtrlBytes);
  uint8_t* stages = smem + kCtrlBytes + kTableBytes;
  uint8_t* xbufs = stages + static_cast<size_t>(a.stages) * a.stage_bytes;
  OperandMeta* metas = reinterpret_cast<OperandMeta*>(xbufs + 2 * a.xbuf_bytes);
  uint8_t* sring = reinterpret_cast<uint8_t*>(metas + 2);
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int i = 0; i < a.stages; ++i) {
      mbar_init(smem_u32(&cb.full[i]), 1);
      mbar_init(smem_u32(&cb.empty[i]), kDQ);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&cb.xfull[i]), 1);
      mbar_init(smem_u32(&cb.xempty[i]), kMmaIssuers + 4);
      mbar_init(smem_u32(&cb.qfull[i]), 1);
    }
    for (int i = 0; i < C::aslots; ++i) {
      mbar_init(smem_u32(&cb.afull[i]), kDQ);
      mbar_init(smem_u32(&cb.aempty[i]), 1);
    }
    for (int i = 0; i < C::dslots; ++i) {
      mbar_init(smem_u32(&cb.dfull[i]), 1);
      mbar_init(smem_u32(&cb.dempty[i]), 4);
    }
    for (int i = 0; i < kSRing; ++i) mbar_init(smem_u32(&cb.sempty[i]), 4);
    mbar_init(smem_u32(&cb.drain), kMmaIssuers);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(&cb.tmem), kTmemCols);
    tmem_relinquish();
  }
  const uint64_t deadline = global_timer_ns() + kTimeoutNs;
  // Launched with programmatic stream serialisation: the next kernel in the
  // stream may be scheduled onto an SM as soon as this CTA leaves it (its
  // prologue above overlaps this call's tail), and this call reads nothing in
  // global memory before the previous kernel has finished.
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();
  // Phase 1: route this CTA's tokens (the stage ring is free scratch).
  route_phase(a, reinterpret_cast<float*>(stages));
  __syncthreads();
  if (threadIdx.x == 0 && !grid_sync(a, 1, deadline)) record_timeout(a);
  __syncthreads();
  // Phase 2: the work-segment table of this CTA's unit ranges.
  build_table(a, cb, table, reinterpret_cast<int*>(stages));
  // Phase 3: the expert pipeline.
  if (warp < kDQ) {
    dequant_warps<SK, G>(a, cb, table, stages, xbufs, metas, deadline);
  } else if (warp < kEpi0 + 4) {
    epilogue_warps<SK, G>(a, cb, table, metas, sring, deadline);
  } else if (warp == kMmaWarp || warp == kMmaWarp2) {
    if ((threadIdx.x & 31) == 0) mma_issuer<SK, G>(a, cb, table, xbufs, warp == kMmaWarp2 ? 1 : 0, deadline);
    __syncwarp();
  } else if (warp == kWProd) {
    weight_producer(a, cb, table, stages, sring, deadline);
  } else if (warp == kBProd) {
    operand_producer(a, cb, table, xbufs, deadline);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(cb.tmem, kTmemCols);
  }
  // ------------------------- grid barrier + combine -------------------------
  if (threadIdx.x == 0 && !grid_sync(a, 2, deadline)) record_timeout(a);
  __syncthreads();
  // The per-call counters are no longer read by anyone: zero them for the
  // next call, a slice per CTA.
  {
    const int nc = gridDim.x, c = blockIdx.x;
    for (int i = a.E * c / nc + threadIdx.x; i < a.E * (c + 1) / nc; i += kThreads) a.cnt[i] = 0;
    for (int i = cb.S * c / nc + threadIdx.x; i < cb.S * (c + 1) / nc; i += kThreads) a.seg_done[i] = 0;
  }
  const int quads = a.H / 4;
  const int64_t total = static_cast<int64_t>(a.M) * quads;
  int64_t b, e;  // this CTA's slice; 32-bit arithmetic unless the output is huge
  if (total <= 0x7fffffff) {
    int b32, e32;
    unit_range(static_cast<int>(total), b32, e32);
    b = b32;
    e = e32;
  } else {
    b = total * blockIdx.x / gridDim.x;
    e = total * (blockIdx.x + 1) / gridDim.x;
  }
  // (token, quad) of element i carried along, one division per thread
  const int64_t i0 = b + threadIdx.x;
  int ctok, cq;
  if (i0 <= 0x7fffffff) {
    ctok = static_cast<int>(i0) / quads;
    cq = static_cast<int>(i0) % quads;
  } else {
    ctok = static_cast<int>(i0 / quads);
    cq = static_cast<int>(i0 % quads);
  }
  const int dtok = kThreads / quads, dq = kThreads % quads;
  for (int64_t i = b + threadIdx.x; i < e; i += kThreads, ctok += dtok, cq += dq, ctok += cq >= quads, cq -= cq >= quads ? quads : 0) {
    const int tok = ctok;
    const int n = cq * 4;
    // every slot's id and y (rows of unrouted slots hold stale values and are
    // not added) and the shared expert's, loaded together; then the sum in
    // slot order
    const bool with_shared = a.has_shared && tok >= a.sh_begin && tok < a.sh_end;
    float gt = 0.f;
    float4 ys = make_float4(0.f, 0.f, 0.f, 0.f);
    if (with_shared) {
      gt = __ldcg(a.gate + tok);
      ys = ldg_cg_f4(a.ybuf + static_cast<int64_t>(a.numel + tok) * a.H + n);
    }
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j0 = 0; j0 < a.k; j0 += 8) {
      int ex[8];
      float4 y[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int pp = tok * a.k + j0 + j;
        ex[j] = j0 + j < a.k ? __ldcg(a.topk_ids + pp) : -1;
        if (j0 + j < a.k) y[j] = ldg_cg_f4(a.ybuf + static_cast<int64_t>(pp) * a.H + n);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (ex[j] >= 0 && ex[j] < a.E) {
          sum.x += y[j].x;
          sum.y += y[j].y;
          sum.z += y[j].z;
          sum.w += y[j].w;
        }
      }
    }
    if (with_shared) {
      sum.x = fmaf(gt, ys.x, sum.x);
      sum.y = fmaf(gt, ys.y, sum.y);
      sum.z = fmaf(gt, ys.z, sum.z);
      sum.w = fmaf(gt, ys.w, sum.w);
    }
    const int64_t o = static_cast<int64_t>(tok) * a.H + n;
    const __nv_bfloat162 lo = __floats2bfloat162_rn(sum.x, sum.y);
    const __nv_bfloat162 hi = __floats2bfloat162_rn(sum.z, sum.w);
    uint2 packed;
    packed.x = *reinterpret_cast<const uint32_t*>(&lo);
    packed.y = *reinterpret_cast<const uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(a.out + o) = packed;
    if (a.out_f32) *reinterpret_cast<float4*>(a.out_f32 + o) = sum;
  }
  finish_call(a, &cb.last);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct FusedGeometry {
  int stages, sk;
  uint32_t stage_bytes, xbuf_bytes;
  size_t smem;
};

static uint32_t round128(uint64_t v) { return static_cast<uint32_t>((v + 127) / 128 * 128); }

constexpr int kMinStages = 4;  // weight stages in flight at least

static FusedGeometry geometry_for(int H, int I, int sk) {
  FusedGeometry f;
  f.sk = sk;
  f.stage_bytes = round128(static_cast<uint64_t>(sk) * 64);
  static_assert(kSRingBytes % 16 == 0, "scale ring entries are bulk-copy destinations");
  // operand rows: quantised x with its meta, or fp32 gate|up with the combine weight
  const uint64_t xrow = xq_row_bytes(H) | 16u, hrow = (8ull * I + 16u) | 16u;
  f.xbuf_bytes = round128(static_cast<uint64_t>(kFBM) * (xrow > hrow ? xrow : hrow));
  const size_t fixed = kCtrlBytes + kTableBytes + 2ull * f.xbuf_bytes + 2 * sizeof(OperandMeta) +
                       kSRing * kSRingBytes;
  const size_t budget = 227 * 1024;
  int s = fixed < budget ? static_cast<int>((budget - fixed) / f.stage_bytes) : 0;
  if (s > kMaxStages) s = kMaxStages;
  f.stages = s;
  f.smem = fixed + static_cast<size_t>(s) * f.stage_bytes;
  return f;
}

// K per stage: the largest of 512, 256, 128 that divides both H and I, whose
// quantisation groups fit the stage's accumulators and that leaves room for
// kMinStages stages in shared memory (the operand buffers grow with H and I).
static FusedGeometry fused_geometry(int H, int I, int G) {
  for (int sk = 512; sk > 128; sk /= 2) {
    if (H % sk || I % sk || sk % G || sk / G > accs_for(sk)) continue;
    const FusedGeometry f = geometry_for(H, I, sk);
    if (f.stages >= kMinStages) return f;
  }
  return geometry_for(H, I, 128);
}

static int device_sms() {
  static int cached_dev = -1, cached_sms = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (dev != cached_dev) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    cached_dev = dev;
    cached_sms = n;
  }
  return cached_sms;
}


bool fused_supported(int H, int I, int G) {
  if (G != 64 && G != 128) return false;
  if (H % 256 || I % 128 || H > 2048 || I > 1024 || H % G || I % G) return false;
  const FusedGeometry f = fused_geometry(H, I, G);
  if (f.sk % G) return false;
  // tensor memory: slots x (A tile + accumulators) <= 512 columns; every
  // group of a stage gets a whole number of the stage's accumulators
  const int acc = accs_for(f.sk);
  if (aslots_for(f.sk) * (f.sk / 4) + dslots_for(f.sk) * dslot_cols(f.sk) > kTmemCols || dslots_for(f.sk) < 2)
    return false;
  if (f.sk / G > acc || acc % (f.sk / G) || (G / 32) % (acc / (f.sk / G))) return false;
  return f.stages >= kMinStages;
}

int fused_max_work_segments(int M, int max_seg, int max_blocks) {
  const int shared_blocks = (M + kFBM - 1) / kFBM;
  return max_seg + max_blocks / kWsBlocks + (shared_blocks + kWsBlocks - 1) / kWsBlocks + 2;
}

template <int SK, int G>
static int launch_fused_t(const FusedArgs& a, const FusedGeometry& f, cudaStream_t st) {
  static int configured = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MTP_ERR_CUDA;
  if (configured != dev) {
    if (cudaFuncSetAttribute(moe_fused_kernel<SK, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) !=
        cudaSuccess)
      return MTP_ERR_CUDA;
    configured = dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(device_sms()));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = f.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (cudaLaunchKernelEx(&cfg, moe_fused_kernel<SK, G>, a) != cudaSuccess) {
    cudaGetLastError();
    return MTP_ERR_LAUNCH;
  }
  return MTP_OK;
}

int launch_moe_fused(const FusedArgs& a_in, cudaStream_t st) {
  FusedArgs a = a_in;
  const FusedGeometry f = fused_geometry(a.H, a.I, a.G);
  a.stages = f.stages;
  a.stage_bytes = f.stage_bytes;
  a.xbuf_bytes = f.xbuf_bytes;
  a.sk = f.sk;
  if (f.sk == 512 && a.G == 128) return launch_fused_t<512, 128>(a, f, st);
  if (f.sk == 256 && a.G == 128) return launch_fused_t<256, 128>(a, f, st);
  if (f.sk == 128 && a.G == 128) return launch_fused_t<128, 128>(a, f, st);
  if (f.sk == 128 && a.G == 64) return launch_fused_t<128, 64>(a, f, st);
  return MTP_ERR_SHAPE;
}

}  // namespace mtp
