// The W4A16 MoE layer forward on sm_100a as one persistent kernel (one CTA
// per SM, 18 warps). It runs in three phases separated by grid-wide barriers:
//
//   routing  CTA c routes tokens c, c + G, ... (G = CTAs): router softmax /
//            top-k / renormalise (warps 0-7, one token each), the shared
//            expert's sigmoid gate (warps 8-15); each (token, slot) pair is
//            appended to its expert's list with an atomic counter. Pair order
//            inside a list does not change any result: every pair is its own
//            MMA column.
//   table    every CTA derives the work segments (the shared expert's token
//            blocks, then each routed expert's pairs in blocks of 8, experts
//            ascending) from the per-expert counts, and fills the entries of
//            its own unit ranges into shared memory with the blob address
//            already resolved through the slot table.
//   experts  warp-specialised over the work units:
//          warp 16  weight producer - streams each work unit's packed int4
//                   strips, fp16 scales and zero nibbles from HBM into a ring
//                   of shared-memory stages with 1-D bulk copies
//                   (cp.async.bulk completing on an mbarrier), running ahead
//                   of the consumers by the ring depth;
//          warp 17  operand producer - brings the B operand of every token
//                   block (8 x rows for W1, 8 h rows for W2) into a double
//                   buffer; before the first W2 unit of a segment it waits
//                   until all W1 units of that segment have published h;
//          warps 0-15 consumers - quantise each new block of operand rows
//                   in shared memory to 16-bit integers (a signed high-byte
//                   row, an unsigned low-byte row, one scale per row), unpack
//                   the int4 weights to u8, run exact int32 m16n8k32 MMAs
//                   (u8 x s8 and u8 x u8) per quantisation group, fold the
//                   zero point and the scales in fp32, reduce across warps,
//                   then the epilogue.
//
// Work units, in this order (each CTA takes a contiguous range of each list;
// a work segment is one token block, so ranges balance and every unit of a
// segment reuses the same operand rows):
//   W1 unit (segment, strip pair i): gate rows 16i..16i+15 and up rows
//      I+16i..I+16i+15 over all of K = H -> h = silu(gate) * up (bf16) for
//      every (token, slot) pair of the segment (vLLM fused_moe W1 +
//      silu_and_mul, tracing/vllm_router_trace.py:19674-19719).
//   W2 unit (segment, row octet r): down rows 128r..128r+127 over K = I ->
//      y = h . W2^T times the router weight (MUL_ROUTED_WEIGHT, :19761-19782),
//      fp32 per pair.
// Then a second grid-wide barrier, after which every CTA combines a slice of
// the output and clears a slice of the per-call counters: out = sum over the top-k slots in slot order of y +
// sigmoid(x . w_g) * y_shared (moe_sum :19801 and the shared-expert gate
// :3994-4031, :4140-4152), so the result is deterministic.
//
// Consecutive units of the same single-block segment reuse the operand buffer
// (the same x or h rows) without a new copy.
//
// Cross-CTA dependencies go through release/acquire counters. Units never
// wait on later units and the final barrier is reached by every CTA after
// its own units, so with all CTAs resident (one per SM, sized by shared
// memory) nothing deadlocks. Every wait is bounded by a deadline on the
// global timer; on expiry the kernel sets bit 0 (value 1) of status[2] and
// carries on, so it always terminates. A caller-given top-k row that repeats
// an expert sets value 4 (the repeat is dropped).
#include "internal.cuh"
#include "route.cuh"

namespace mtp {

constexpr int kFBM = 8;            // tokens (pairs) per block = MMA N
constexpr int kCW = 16;            // consumer warps
constexpr int kCT = kCW * 32;      // consumer threads
constexpr int kFusedThreads = kCT + 64;
constexpr int kWProd = kCW;        // weight producer warp
constexpr int kBProd = kCW + 1;    // operand producer warp
constexpr int kMaxStages = 4;
constexpr int kCtrlBytes = 512;
constexpr int kWsCache = 64;       // work segments cached in shared memory per pass
constexpr int kTableBytes = 2 * kWsCache * kWsInts * 4;
constexpr int kRedBytes = kCW * 2 * 4 * 32 * 4 + 2 * 4 * 32 * 4;
constexpr uint64_t kTimeoutNs = 2000000000ull;  // 2 s per layer call
constexpr int kBarConsumers = 1;   // named barrier id for the consumer warps
constexpr int kMaxChunks = 32;     // K / 64 for K <= 2048

// ---------------------------------------------------------------------------
// shared-memory control block and the per-pass work-segment view
// ---------------------------------------------------------------------------
struct Ctrl {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t xfull[2];
  uint64_t xempty[2];
  int stage_valid[kMaxStages];
  int seg_first[2];   // first work segment of the pass range
  int cached[2];      // 1 if the pass range's segments are in the table
  int S;              // work segments of this call
  int gen0;           // grid-barrier generation when the kernel started
  int scan[32];       // block-scan scratch
};
static_assert(sizeof(Ctrl) <= kCtrlBytes, "control block too large");

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

__device__ __forceinline__ int pair_token(const FusedArgs& a, int p) {
  return p >= a.numel ? p - a.numel : p / a.k;
}

__device__ __forceinline__ void unit_range(int total_units, int& b, int& e) {
  const int64_t g = gridDim.x, c = blockIdx.x;
  b = static_cast<int>(total_units * c / g);
  e = static_cast<int>(total_units * (c + 1) / g);
}

__device__ __forceinline__ Pass make_pass(const FusedArgs& a, const Ctrl& cb, const int* table, int pass) {
  Pass P;
  const int S = cb.S;
  P.per = pass == 0 ? a.I / 16 : a.H / 128;
  unit_range(S * P.per, P.ub, P.ue);
  P.seg_first = cb.seg_first[pass];
  P.table = cb.cached[pass] ? table + pass * kWsCache * kWsInts : a.wseg + static_cast<size_t>(P.seg_first) * kWsInts;
  return P;
}

// A unit reuses the operand buffer of the previous unit when both belong to
// the same single-block segment (same rows).
__device__ __forceinline__ bool reuses_operand(const Pass& P, int u) {
  if (u == P.ub) return false;
  const int s = u / P.per;
  return s == (u - 1) / P.per && ws_entry(P, s)[2] == 1;
}

__device__ __forceinline__ void record_timeout(const FusedArgs& a) { atomicOr(a.status + 2, 1); }

// Grid-wide barrier over the kernel's CTAs (all resident: one per SM). One
// thread per CTA calls it; the generation word a.bar[1] counts completed
// barriers, so the kernel waits for `target` = its start value + n. The last
// arriver clears the arrival count before it publishes the new generation, so
// the count is zero again for the next barrier and the next call.
__device__ __forceinline__ bool grid_sync(const FusedArgs& a, int target, uint64_t deadline) {
  __threadfence();
  const int old = atomicAdd(a.bar, 1);
  if (old == static_cast<int>(gridDim.x) - 1) {
    atomicExch(a.bar, 0);
    __threadfence();
    red_release_gpu_add(a.bar + 1, 1);
    return true;
  }
  while (static_cast<int>(static_cast<uint32_t>(ld_acquire_gpu(a.bar + 1)) - static_cast<uint32_t>(target)) < 0) {
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

// Phase 1 (consumer warps): route this CTA's tokens, count and list the
// (token, slot) pairs per expert, and compute the shared-expert gate. Warps
// 0-7 route a token each; warps 8-15 compute the gates of the same tokens.
// `scratch` holds 8 x E floats (the stage ring, still unused).
__device__ void route_phase(const FusedArgs& a, int ctid, float* scratch) {
  const int warp = ctid >> 5, lane = ctid & 31;
  const int G = gridDim.x;
  for (int i0 = 0; static_cast<int64_t>(blockIdx.x) + static_cast<int64_t>(G) * i0 < a.M; i0 += 8) {
    const int64_t t64 = static_cast<int64_t>(blockIdx.x) + static_cast<int64_t>(G) * (i0 + (warp & 7));
    if (t64 >= a.M) continue;
    const int t = static_cast<int>(t64);
    if (warp < 8) {
      int id = -1;
      if (a.logits) {
        float w;
        router_warp(a.logits + static_cast<int64_t>(t) * a.E, a.E, a.k, a.renorm, scratch + warp * a.E, &w, &id);
        if (lane < a.k) {
          a.topk_w[t * a.k + lane] = w;
          a.topk_ids[t * a.k + lane] = id;
        }
      } else if (lane < a.k) {
        id = a.topk_ids[t * a.k + lane];
      }
      if (lane < a.k && id >= 0 && id < a.E) {
        // an expert holds at most one pair per token (distinct ids per token);
        // a repeated id in a caller-given row is dropped and flagged
        const int pos = atomicAdd(a.cnt + id, 1);
        if (pos < a.M) a.lists[static_cast<int64_t>(id) * a.M + pos] = t * a.k + lane;
        else atomicOr(a.status + 2, 4);
      }
    } else if (a.has_shared) {
      // sigmoid(x . w_g): all of a lane's 16-byte loads in flight at once
      const uint4* xr = reinterpret_cast<const uint4*>(a.x + static_cast<int64_t>(t) * a.H);
      const uint4* wg = reinterpret_cast<const uint4*>(a.gate_w);
      const int nvec = a.H / 8;  // <= 256: at most 8 per lane
      uint4 xv[8], wv[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int vi = lane + 32 * j;
        if (vi < nvec) {
          xv[j] = xr[vi];
          wv[j] = wg[vi];
        }
      }
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
      if (lane == 0) a.gate[t] = 1.f / (1.f + expf(-part));
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
      const int tk = s * kFBM + j;
      w[4 + j] = tk < a.M ? a.numel + tk : -1;
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
// `scratch` holds 2E + 1 ints (the operand buffers, still unused).
__device__ void build_table(const FusedArgs& a, Ctrl& cb, int* table, int* scratch) {
  const int tid = threadIdx.x, nt = blockDim.x;
  int* cnt = scratch;           // [E]
  int* sbase = scratch + a.E;   // [E + 1]
  // each thread owns experts [2 tid, 2 tid + 2) (E <= 1024 < 2 * 576)
  int c0 = 0, c1 = 0;
  if (2 * tid < a.E) c0 = min(__ldcg(a.cnt + 2 * tid), a.M);
  if (2 * tid + 1 < a.E) c1 = min(__ldcg(a.cnt + 2 * tid + 1), a.M);
  const int n0 = (c0 + kFBM - 1) / kFBM, n1 = (c1 + kFBM - 1) / kFBM;
  int total;
  const int ex = cta_exclusive_scan(n0 + n1, &total, cb.scan);
  if (2 * tid < a.E) {
    cnt[2 * tid] = c0;
    sbase[2 * tid] = ex;
  }
  if (2 * tid + 1 < a.E) {
    cnt[2 * tid + 1] = c1;
    sbase[2 * tid + 1] = ex + n0;
  }
  if (tid == 0) sbase[a.E] = total;
  const int shared_ws = a.has_shared ? (a.M + kFBM - 1) / kFBM : 0;
  const int S = shared_ws + total;
  if (tid == 0) cb.S = S;
  if (blockIdx.x == 0) {
    const int u0 = c0 > 0, u1 = c1 > 0;
    int nused;
    const int rank = cta_exclusive_scan(u0 + u1, &nused, cb.scan);
    if (a.demand_log) {
      if (tid == 0) a.demand_log[0] = nused;
      if (u0) a.demand_log[1 + rank] = 2 * tid;
      if (u1) a.demand_log[1 + rank + u0] = 2 * tid + 1;
    }
    for (int j = 0; j < 2; ++j) {
      const int e = 2 * tid + j;
      if (e < a.E && (j == 0 ? u0 : u1)) {
        const int slot = a.slot_table ? a.slot_table[e] : e;
        if (slot < 0) atomicAdd(a.host_blobs ? a.status + 0 : a.status + 1, 1);
      }
    }
  }
  __syncthreads();
  for (int pass = 0; pass < 2; ++pass) {
    const int per = pass == 0 ? a.I / 16 : a.H / 128;
    int ub, ue;
    unit_range(S * per, ub, ue);
    const int first = ub / per;
    const int last = ue > ub ? (ue - 1) / per : first - 1;
    const int n = last - first + 1;
    const bool cached = n <= kWsCache;
    if (tid == 0) {
      cb.seg_first[pass] = first;
      cb.cached[pass] = cached;
    }
    for (int i = tid; i < n; i += nt) {
      int* w = cached ? table + (pass * kWsCache + i) * kWsInts : a.wseg + static_cast<size_t>(first + i) * kWsInts;
      fill_entry(a, first + i, shared_ws, cnt, sbase, w);
    }
  }
  __syncthreads();
}

__device__ __forceinline__ uint32_t lds8(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ float4 ldg_cg_f4(const float* p) {
  float4 v;
  asm volatile("ld.global.cg.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

// Byte ranges of a unit inside the expert blob and inside the stage.
struct Piece {
  uint32_t src_off;
  uint32_t dst_off;
  uint32_t bytes;
};

__device__ __forceinline__ int w1_pieces(const FusedArgs& a, int strip, Piece* p) {
  const uint32_t sb = 8u * a.H;  // one 16-row strip over K = H
  const uint32_t scb = static_cast<uint32_t>(a.H / a.G) * 32u;
  const uint32_t zpb = static_cast<uint32_t>(a.H / a.G) * 8u;
  const uint32_t up = a.I / 16 + strip;
  const uint32_t L13 = static_cast<uint32_t>(a.L.w13_qweight), S13 = static_cast<uint32_t>(a.L.w13_scales),
                 Z13 = static_cast<uint32_t>(a.L.w13_zeros);
  p[0] = {L13 + strip * sb, 0, sb};
  p[1] = {L13 + up * sb, sb, sb};
  p[2] = {S13 + strip * scb, 2 * sb, scb};
  p[3] = {S13 + up * scb, 2 * sb + scb, scb};
  p[4] = {Z13 + strip * zpb, 2 * sb + 2 * scb, zpb};
  p[5] = {Z13 + up * zpb, 2 * sb + 2 * scb + zpb, zpb};
  return 6;
}

__device__ __forceinline__ int w2_pieces(const FusedArgs& a, int octet, Piece* p) {
  const uint32_t ob = 64u * a.I;  // 8 strips of 16 rows over K = I
  const uint32_t scb = 8u * static_cast<uint32_t>(a.I / a.G) * 32u;
  const uint32_t zpb = 8u * static_cast<uint32_t>(a.I / a.G) * 8u;
  const uint32_t L2 = static_cast<uint32_t>(a.L.w2_qweight), S2 = static_cast<uint32_t>(a.L.w2_scales),
                 Z2 = static_cast<uint32_t>(a.L.w2_zeros);
  p[0] = {L2 + octet * ob, 0, ob};
  p[1] = {S2 + octet * scb, ob, scb};
  p[2] = {Z2 + octet * zpb, ob + scb, zpb};
  return 3;
}

// ---------------------------------------------------------------------------
// producers
// ---------------------------------------------------------------------------
__device__ void weight_producer(const FusedArgs& a, Ctrl& cb, const int* table, uint8_t* stages,
                                uint64_t deadline) {
  const int lane = threadIdx.x & 31;
  int st = 0;
  uint32_t ph = 0;
  for (int pass = 0; pass < 2; ++pass) {
    const Pass P = make_pass(a, cb, table, pass);
    for (int u = P.ub; u < P.ue; ++u) {
      const int seg = u / P.per, idx = u % P.per;
      const int* e = ws_entry(P, seg);
      const uint8_t* blob = ws_blob(e);
      const bool host = (e[3] & 2) != 0;
      Piece pc[6];
      const int n = pass == 0 ? w1_pieces(a, idx, pc) : w2_pieces(a, idx, pc);
      if (!mbar_wait(smem_u32(&cb.empty[st]), ph ^ 1u, deadline) && lane == 0) record_timeout(a);
      uint8_t* dst = stages + static_cast<size_t>(st) * a.stage_bytes;
      const uint32_t full = smem_u32(&cb.full[st]);
      if (lane == 0) cb.stage_valid[st] = blob != nullptr;
      if (blob != nullptr && !host) {
        if (lane == 0) {
          uint32_t total = 0;
          for (int i = 0; i < n; ++i) total += pc[i].bytes;
          mbar_arrive_expect_tx(full, total);
          for (int i = 0; i < n; ++i) bulk_g2s(smem_u32(dst + pc[i].dst_off), blob + pc[i].src_off, pc[i].bytes, full);
        }
      } else {
        // Pinned host memory (demand fetch over the host link): a warp copy
        // with eight 16-byte loads in flight per lane.
        if (blob != nullptr) {
          for (int i = 0; i < n; ++i) {
            const uint8_t* src = blob + pc[i].src_off;
            uint8_t* d = dst + pc[i].dst_off;
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
    }
  }
}

__device__ void operand_producer(const FusedArgs& a, Ctrl& cb, const int* table, uint8_t* xbufs,
                                 uint64_t deadline) {
  const int lane = threadIdx.x & 31;
  int xb = 0;
  uint32_t xph = 0;
  for (int pass = 0; pass < 2; ++pass) {
    const Pass P = make_pass(a, cb, table, pass);
    const uint32_t row_bytes = pass == 0 ? 2u * a.H : 2u * a.I;
    const uint32_t row_stride = row_bytes + 16u;
    int waited_seg = -1;
    for (int u = P.ub; u < P.ue; ++u) {
      const int seg = u / P.per;
      if (reuses_operand(P, u)) continue;
      const int* e = ws_entry(P, seg);
      const int nb = e[2];
      if (pass == 1 && seg != waited_seg) {
        // every W1 unit of this segment has published its h columns
        if (lane == 0) {
          bool ok = true;
          while (ld_acquire_gpu(a.seg_done + seg) < a.I / 16) {
            if (global_timer_ns() > deadline) {
              ok = false;
              break;
            }
          }
          if (!ok) record_timeout(a);
          fence_proxy_async_global();
        }
        __syncwarp();
        waited_seg = seg;
      }
      for (int blk = 0; blk < nb; ++blk) {
        if (!mbar_wait(smem_u32(&cb.xempty[xb]), xph ^ 1u, deadline) && lane == 0) record_timeout(a);
        const int p = lane < kFBM ? e[4 + blk * kFBM + lane] : -1;
        const unsigned valid = __ballot_sync(kFullMask, p >= 0);
        const uint32_t xfull = smem_u32(&cb.xfull[xb]);
        if (lane == 0) mbar_arrive_expect_tx(xfull, __popc(valid) * row_bytes);
        __syncwarp();
        if (p >= 0) {
          const uint8_t* src = pass == 0
                                   ? reinterpret_cast<const uint8_t*>(a.x + static_cast<int64_t>(pair_token(a, p)) * a.H)
                                   : reinterpret_cast<const uint8_t*>(a.hbuf + static_cast<int64_t>(p) * a.I);
          bulk_g2s(smem_u32(xbufs + xb * a.xbuf_bytes + lane * row_stride), src, row_bytes, xfull);
        }
        if (++xb == 2) {
          xb = 0;
          xph ^= 1u;
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// consumers
// ---------------------------------------------------------------------------
// Per operand buffer: quantisation metadata of its 8 rows.
struct OperandMeta {
  float sx[kFBM];              // row scale: x = sx * (256 * hi + lo)
  float amax[kFBM][2];         // per-half row maxima (scratch)
  int xsum[kFBM][kMaxChunks];  // per 64-wide chunk: sum of the 16-bit row values
};

__device__ __forceinline__ uint32_t pick(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Quantise the 8 bf16 rows of an operand buffer in place into 16-bit
// integers split into a signed high byte row and an unsigned low byte row
// (row n: hi at [0, K), lo at [K, 2K) of its 2K + 16 byte slot), with a
// per-row scale and per-64-element-chunk sums. 512 consumer threads, 64 per
// row; thread tr owns the 4-element groups j = tr + 64 i, so every shared-
// memory access of a warp is contiguous. All values are read before the first
// barrier and written after it (the output overlaps the input).
__device__ __forceinline__ void quantize_rows(uint8_t* rows, OperandMeta& meta, int K, int ctid) {
  const int n = ctid >> 6, tr = ctid & 63;
  const int ng = K / 4;  // 16..512 groups per row
  uint8_t* row = rows + n * (2u * K + 16u);
  uint2 raw[8];  // bf16 pairs, kept packed until the scale is known
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int j = tr + 64 * i;
    raw[i] = make_uint2(0u, 0u);
    if (j < ng) {
      raw[i] = *reinterpret_cast<const uint2*>(row + 8 * j);
      const uint32_t m0 = __vmaxu2(raw[i].x & 0x7fff7fffu, raw[i].y & 0x7fff7fffu);
      mx = fmaxf(mx, fmaxf(__uint_as_float(m0 << 16), __uint_as_float(m0 & 0xffff0000u)));
    }
  }
  mx = warp_max(mx);
  if ((ctid & 31) == 0) meta.amax[n][(ctid >> 5) & 1] = mx;
  named_bar_sync(kBarConsumers, kCT);
  const float amax = fmaxf(meta.amax[n][0], meta.amax[n][1]);
  const float inv = amax > 0.f ? 32767.f / amax : 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (64 * i < ng) {  // warp-uniform: ng is a multiple of 16, the shuffles stay converged
      const int j = tr + 64 * i;
      int sum = 0;
      if (j < ng) {
        uint32_t hw = 0u, lw = 0u;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const uint32_t h = (b < 2 ? raw[i].x : raw[i].y) >> (16 * (b & 1));
          const int q = max(-32767, min(32767, __float2int_rn(__uint_as_float(h << 16) * inv)));
          sum += q;
          hw |= (static_cast<uint32_t>(q >> 8) & 0xffu) << (8 * b);
          lw |= (static_cast<uint32_t>(q) & 0xffu) << (8 * b);
        }
        *reinterpret_cast<uint32_t*>(row + 4 * j) = hw;
        *reinterpret_cast<uint32_t*>(row + K + 4 * j) = lw;
      }
      // a 64-element chunk is the 16 groups of 16 consecutive lanes
      sum += __shfl_xor_sync(kFullMask, sum, 1);
      sum += __shfl_xor_sync(kFullMask, sum, 2);
      sum += __shfl_xor_sync(kFullMask, sum, 4);
      sum += __shfl_xor_sync(kFullMask, sum, 8);
      if ((tr & 15) == 0 && j < ng) meta.xsum[n][j >> 4] = sum;
    }
  }
  if (tr == 0) meta.sx[n] = amax / 32767.f;
  named_bar_sync(kBarConsumers, kCT);
}

// B operands (high and low byte rows) of one k32 step for this lane's
// ldmatrix row: matrices hi[k0..], hi[k0+16..], lo[k0..], lo[k0+16..].
__device__ __forceinline__ void load_b(uint32_t xbase, uint32_t rs, int K, int row, int mat, int k0,
                                       uint32_t (&b)[4]) {
  const uint32_t addr = xbase + row * rs + (mat >= 2 ? K : 0) + k0 + 16 * (mat & 1);
  ldsm_x4(addr, b[0], b[1], b[2], b[3]);
}

__device__ __forceinline__ void zero_rows_of(uint32_t zb, int zero_mode, int& z0, int& z1) {
  if (zero_mode == MTP_ZERO_SYM8) {
    z0 = z1 = 8;
  } else {
    z0 = zb & 0xF;
    z1 = zb >> 4;
  }
}

// acc += s_row * (256 * hi + lo - z_row * xsum_col) for the 4 accumulator
// elements of this lane (rows g, g+8; columns 2t, 2t+1).
__device__ __forceinline__ void fold_int(float (&acc)[4], const int (&dh)[4], const int (&dl)[4], uint32_t scw,
                                         int z0, int z1, int xs0, int xs1) {
  const float2 s = half2_bits_to_float2(scw);
  acc[0] = fmaf(static_cast<float>(256 * dh[0] + dl[0] - z0 * xs0), s.x, acc[0]);
  acc[1] = fmaf(static_cast<float>(256 * dh[1] + dl[1] - z0 * xs1), s.x, acc[1]);
  acc[2] = fmaf(static_cast<float>(256 * dh[2] + dl[2] - z1 * xs0), s.y, acc[2]);
  acc[3] = fmaf(static_cast<float>(256 * dh[3] + dl[3] - z1 * xs1), s.y, acc[3]);
}

template <int W1C, int W2C>
__device__ void consumers(const FusedArgs& a, Ctrl& cb, const int* table, uint8_t* stages, uint8_t* xbufs,
                          OperandMeta* metas, float* red, uint64_t deadline) {
  const int ctid = threadIdx.x;  // 0..511
  const int warp = ctid >> 5, lane = ctid & 31, g = lane >> 2, t = lane & 3;
  const int nkw = a.H / 64 / W1C;  // warps along K in W1 (<= 16)
  const int cpg = a.G / 64;        // 64-wide chunks per quantisation group
  int st = 0, xb = 0;
  uint32_t ph = 0, xph = 0;
  const int ld_row = lane & 7, ld_mat = lane >> 3;  // ldmatrix row address of this lane
  int published = 0;  // W1 units of the current segment not yet published

  for (int pass = 0; pass < 2; ++pass) {
    const Pass P = make_pass(a, cb, table, pass);
    const int K = pass == 0 ? a.H : a.I;
    const uint32_t rs = 2u * K + 16u;
    for (int u = P.ub; u < P.ue; ++u) {
      const int seg = u / P.per, idx = u % P.per;
      const int* e = ws_entry(P, seg);
      const int nb = e[2];
      const bool reuse = reuses_operand(P, u);
      const bool keep = u + 1 < P.ue && reuses_operand(P, u + 1);
      if (!mbar_wait(smem_u32(&cb.full[st]), ph, deadline) && ctid == 0) record_timeout(a);
      const bool wvalid = cb.stage_valid[st] != 0;
      const uint32_t sbase = smem_u32(stages + static_cast<size_t>(st) * a.stage_bytes);
      for (int blk = 0; blk < nb; ++blk) {
        OperandMeta& meta = metas[xb];
        uint8_t* xrows = xbufs + xb * a.xbuf_bytes;
        if (!reuse) {
          if (!mbar_wait(smem_u32(&cb.xfull[xb]), xph, deadline) && ctid == 0) record_timeout(a);
          quantize_rows(xrows, meta, K, ctid);
        }
        const uint32_t xbase = smem_u32(xrows);
        const int* cols = e + 4 + blk * kFBM;
        if (pass == 0) {
          // ------------------------------ W1 ------------------------------
          float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
          if (wvalid && warp < nkw) {
            const uint32_t sb = 8u * a.H, scb = (a.H / a.G) * 32u, zpb = (a.H / a.G) * 8u;
            int dh[2][4], dl[2][4];
            int xs0 = 0, xs1 = 0;
#pragma unroll
            for (int j = 0; j < W1C; ++j) {
              const int c = warp * W1C + j;
              uint4 w[2];
              w[0] = lds128(sbase + (c * 32 + lane) * 16);
              w[1] = lds128(sbase + sb + (c * 32 + lane) * 16);
#pragma unroll
              for (int s2 = 0; s2 < 2; ++s2) {
                uint32_t b[4];
                load_b(xbase, rs, K, ld_row, ld_mat, 64 * c + 32 * s2, b);
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                  uint32_t A[4];
                  unpack_u8(pick(w[q], 2 * s2), pick(w[q], 2 * s2 + 1), A);
                  if (s2 == 0 && (j == 0 || c % cpg == 0)) {
                    imma_u8s8_zc(dh[q], A, b[0], b[1]);
                    imma_u8u8_zc(dl[q], A, b[2], b[3]);
                  } else {
                    imma_u8s8(dh[q], A, b[0], b[1]);
                    imma_u8u8(dl[q], A, b[2], b[3]);
                  }
                }
              }
              xs0 += meta.xsum[2 * t][c];
              xs1 += meta.xsum[2 * t + 1][c];
              if ((c + 1) % cpg == 0 || j == W1C - 1) {
                const int grp = c / cpg;
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                  const uint32_t scw = lds32(sbase + 2 * sb + q * scb + (grp * 8 + g) * 4);
                  const uint32_t zb =
                      a.zero_mode == MTP_ZERO_RAW ? lds8(sbase + 2 * sb + 2 * scb + q * zpb + grp * 8 + g) : 0x88u;
                  int z0, z1;
                  zero_rows_of(zb, a.zero_mode, z0, z1);
                  fold_int(acc[q], dh[q], dl[q], scw, z0, z1, xs0, xs1);
                }
                xs0 = xs1 = 0;
              }
            }
          }
          if (!keep) {
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&cb.xempty[xb]));
          }
          if (warp < nkw) {
#pragma unroll
            for (int q = 0; q < 2; ++q)
#pragma unroll
              for (int r = 0; r < 4; ++r) red[((warp * 2 + q) * 4 + r) * 32 + lane] = acc[q][r];
          }
          named_bar_sync(kBarConsumers, kCT);
          {
            // thread 4m+s: position m = (r, l) of the 16x8 tile, s = (strip,
            // half of the K warps); halves summed, then gate/up met by shuffle
            const int m = ctid >> 2, sub = ctid & 3, q = sub >> 1, half = sub & 1;
            float v = 0.f;
            for (int w = half; w < nkw; w += 2) v += red[w * 256 + q * 128 + m];
            v += __shfl_xor_sync(kFullMask, v, 1);
            const float up = __shfl_xor_sync(kFullMask, v, 2);
            if (sub == 0) {
              const int r = m >> 5, l = m & 31;
              const int col = 2 * (l & 3) + (r & 1);
              const int p = cols[col];
              if (p >= 0) {
                const int row = (l >> 2) + 8 * (r >> 1);
                const float sx = meta.sx[col];
                a.hbuf[static_cast<int64_t>(p) * a.I + 16 * idx + row] =
                    __bfloat16_as_ushort(__float2bfloat16(silu(v * sx) * (up * sx)));
              }
            }
          }
          // protects red from the next unit and orders the h stores before the
          // release below
          named_bar_sync(kBarConsumers, kCT);
          // publish this CTA's h columns of the segment once, when it leaves
          // the segment (or its range)
          ++published;
          if (blk == nb - 1 && (u + 1 == P.ue || (u + 1) / P.per != seg)) {
            if (ctid == 0) red_release_gpu_add(a.seg_done + seg, published);
            published = 0;
          }
        } else {
          // ------------------------------ W2 ------------------------------
          const int sidx = warp >> 1, hk = warp & 1;
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
          if (wvalid) {
            const uint32_t sb = 8u * a.I;  // one strip over K = I
            const uint32_t scb_all = 8u * (a.I / a.G) * 32u;
            const int gper = a.I / a.G;
            int dh[2][4], dl[2][4];  // two independent chains: chunk parity
            int xs0 = 0, xs1 = 0;
            bool fresh[2] = {true, true};
#pragma unroll
            for (int j = 0; j < W2C; ++j) {
              const int c = hk * W2C + j;
              const int par = j & 1;
              const uint4 w = lds128(sbase + sidx * sb + (c * 32 + lane) * 16);
#pragma unroll
              for (int s2 = 0; s2 < 2; ++s2) {
                uint32_t b[4];
                load_b(xbase, rs, K, ld_row, ld_mat, 64 * c + 32 * s2, b);
                uint32_t A[4];
                unpack_u8(pick(w, 2 * s2), pick(w, 2 * s2 + 1), A);
                if (s2 == 0 && fresh[par]) {
                  imma_u8s8_zc(dh[par], A, b[0], b[1]);
                  imma_u8u8_zc(dl[par], A, b[2], b[3]);
                } else {
                  imma_u8s8(dh[par], A, b[0], b[1]);
                  imma_u8u8(dl[par], A, b[2], b[3]);
                }
              }
              fresh[par] = false;
              xs0 += meta.xsum[2 * t][c];
              xs1 += meta.xsum[2 * t + 1][c];
              if ((c + 1) % cpg == 0 || j == W2C - 1) {
                const int grp = c / cpg;
                const uint32_t scw = lds32(sbase + 8 * sb + ((sidx * gper + grp) * 8 + g) * 4);
                const uint32_t zb =
                    a.zero_mode == MTP_ZERO_RAW ? lds8(sbase + 8 * sb + scb_all + (sidx * gper + grp) * 8 + g) : 0x88u;
                int z0, z1;
                zero_rows_of(zb, a.zero_mode, z0, z1);
                int sh[4], sl[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                  sh[r] = (fresh[0] ? 0 : dh[0][r]) + (fresh[1] ? 0 : dh[1][r]);
                  sl[r] = (fresh[0] ? 0 : dl[0][r]) + (fresh[1] ? 0 : dl[1][r]);
                }
                fold_int(acc, sh, sl, scw, z0, z1, xs0, xs1);
                xs0 = xs1 = 0;
                fresh[0] = fresh[1] = true;
              }
            }
          }
          if (!keep) {
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&cb.xempty[xb]));
          }
          if (hk == 1) {
#pragma unroll
            for (int r = 0; r < 4; ++r) red[(sidx * 4 + r) * 32 + lane] = acc[r];
          }
          named_bar_sync(kBarConsumers, kCT);
          if (hk == 0) {
            const int p0 = cols[2 * t], p1 = cols[2 * t + 1];
            const float w0 = ((p0 >= 0 && p0 < a.numel) ? __ldcg(a.topk_w + p0) : 1.f) * meta.sx[2 * t];
            const float w1 = ((p1 >= 0 && p1 < a.numel) ? __ldcg(a.topk_w + p1) : 1.f) * meta.sx[2 * t + 1];
            const int nbase = 128 * idx + 16 * sidx;
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              const int p = (r & 1) ? p1 : p0;
              if (p >= 0) {
                const float y = (acc[r] + red[(sidx * 4 + r) * 32 + lane]) * ((r & 1) ? w1 : w0);
                a.ybuf[static_cast<int64_t>(p) * a.H + nbase + g + 8 * (r >> 1)] = y;
              }
            }
          }
          named_bar_sync(kBarConsumers, kCT);
        }
        if (!keep) {
          if (++xb == 2) {
            xb = 0;
            xph ^= 1u;
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&cb.empty[st]));
      if (++st == a.stages) {
        st = 0;
        ph ^= 1u;
      }
    }
  }

  // ------------------------- grid arrival + combine -------------------------
  named_bar_sync(kBarConsumers, kCT);
  if (ctid == 0 && !grid_sync(a, cb.gen0 + 2, deadline)) record_timeout(a);
  named_bar_sync(kBarConsumers, kCT);
  // The per-call counters are no longer read by anyone: zero them for the
  // next call, a slice per CTA.
  {
    const int G = gridDim.x, c = blockIdx.x;
    for (int i = a.E * c / G + ctid; i < a.E * (c + 1) / G; i += kCT) a.cnt[i] = 0;
    for (int i = cb.S * c / G + ctid; i < cb.S * (c + 1) / G; i += kCT) a.seg_done[i] = 0;
  }
  const int quads = a.H / 4;
  const int64_t total = static_cast<int64_t>(a.M) * quads;
  const int64_t b = total * blockIdx.x / gridDim.x, e = total * (blockIdx.x + 1) / gridDim.x;
  for (int64_t i = b + ctid; i < e; i += kCT) {
    const int tok = static_cast<int>(i / quads);
    const int n = static_cast<int>(i % quads) * 4;
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < a.k; ++j) {
      const int pp = tok * a.k + j;
      const int ex = __ldcg(a.topk_ids + pp);
      if (ex >= 0 && ex < a.E) {
        const float4 y = ldg_cg_f4(a.ybuf + static_cast<int64_t>(pp) * a.H + n);
        sum.x += y.x;
        sum.y += y.y;
        sum.z += y.z;
        sum.w += y.w;
      }
    }
    if (a.has_shared) {
      const float gt = __ldcg(a.gate + tok);
      const float4 y = ldg_cg_f4(a.ybuf + static_cast<int64_t>(a.numel + tok) * a.H + n);
      sum.x = fmaf(gt, y.x, sum.x);
      sum.y = fmaf(gt, y.y, sum.y);
      sum.z = fmaf(gt, y.z, sum.z);
      sum.w = fmaf(gt, y.w, sum.w);
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
}

template <int W1C, int W2C>
__global__ void __launch_bounds__(kFusedThreads, 1) moe_fused_kernel(FusedArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  Ctrl& cb = *reinterpret_cast<Ctrl*>(smem);
  int* table = reinterpret_cast<int*>(smem + kCtrlBytes);
  uint8_t* stages = smem + kCtrlBytes + kTableBytes;
  uint8_t* xbufs = stages + static_cast<size_t>(a.stages) * a.stage_bytes;
  OperandMeta* metas = reinterpret_cast<OperandMeta*>(xbufs + 2 * a.xbuf_bytes);
  float* red = reinterpret_cast<float*>(metas + 2);
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int i = 0; i < a.stages; ++i) {
      mbar_init(smem_u32(&cb.full[i]), 1);
      mbar_init(smem_u32(&cb.empty[i]), kCW);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&cb.xfull[i]), 1);
      mbar_init(smem_u32(&cb.xempty[i]), kCW);
    }
    fence_mbar_init();
  }
  if (threadIdx.x == 0) cb.gen0 = ld_acquire_gpu(a.bar + 1);
  const uint64_t deadline = global_timer_ns() + kTimeoutNs;
  __syncthreads();
  // Phase 1: route this CTA's tokens (the stage ring is free scratch).
  if (warp < kCW) route_phase(a, threadIdx.x, reinterpret_cast<float*>(stages));
  __syncthreads();
  if (threadIdx.x == 0 && !grid_sync(a, cb.gen0 + 1, deadline)) record_timeout(a);
  __syncthreads();
  // Phase 2: the work-segment table of this CTA's unit ranges.
  build_table(a, cb, table, reinterpret_cast<int*>(stages));
  __syncthreads();
  if (warp == kWProd) {
    weight_producer(a, cb, table, stages, deadline);
  } else if (warp == kBProd) {
    operand_producer(a, cb, table, xbufs, deadline);
  } else {
    consumers<W1C, W2C>(a, cb, table, stages, xbufs, metas, red, deadline);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct FusedGeometry {
  int stages;
  uint32_t stage_bytes, xbuf_bytes;
  size_t smem;
};

static uint32_t round128(uint64_t v) { return static_cast<uint32_t>((v + 127) / 128 * 128); }

static FusedGeometry fused_geometry(int H, int I, int G) {
  FusedGeometry f;
  const uint64_t w1 = 16ull * H + 2ull * (H / G) * 32 + 2ull * (H / G) * 8;
  const uint64_t w2 = 64ull * I + 8ull * (I / G) * 32 + 8ull * (I / G) * 8;
  f.stage_bytes = round128(w1 > w2 ? w1 : w2);
  const int maxrow = H > I ? H : I;
  f.xbuf_bytes = round128(static_cast<uint64_t>(kFBM) * (2ull * maxrow + 16));
  const size_t fixed = kCtrlBytes + kTableBytes + 2ull * f.xbuf_bytes + 2ull * sizeof(OperandMeta) + kRedBytes;
  const size_t budget = 227 * 1024;
  int s = fixed < budget ? static_cast<int>((budget - fixed) / f.stage_bytes) : 0;
  if (s > kMaxStages) s = kMaxStages;
  f.stages = s;
  f.smem = fixed + static_cast<size_t>(s) * f.stage_bytes;
  return f;
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

template <int W1C, int W2C>
static int launch_fused_t(const FusedArgs& a, const FusedGeometry& f, cudaStream_t st) {
  static int configured = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured != dev) {
    if (cudaFuncSetAttribute(moe_fused_kernel<W1C, W2C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             227 * 1024) != cudaSuccess)
      return MTP_ERR_CUDA;
    configured = dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(device_sms());
  cfg.blockDim = dim3(kFusedThreads);
  cfg.dynamicSmemBytes = f.smem;
  cfg.stream = st;
  cfg.attrs = nullptr;
  cfg.numAttrs = 0;
  if (cudaLaunchKernelEx(&cfg, moe_fused_kernel<W1C, W2C>, a) != cudaSuccess) return MTP_ERR_LAUNCH;
  return MTP_OK;
}

// W1C: 64-wide K chunks per W1 warp (H/64 chunks over at most 16 warps);
// W2C: chunks per W2 warp (two warps per strip split K = I).
static bool fused_template(int H, int I, int* w1c, int* w2c) {
  *w1c = H > 1024 ? 2 : 1;
  *w2c = I / 128;
  return (H / 64) % *w1c == 0 && H / 64 / *w1c <= kCW && *w2c >= 1 && *w2c <= 8;
}

bool fused_supported(int H, int I, int G) {
  if (G != 64 && G != 128) return false;
  if (H % 128 || I % 128 || H % G || I % G) return false;
  int w1c, w2c;
  if (!fused_template(H, I, &w1c, &w2c)) return false;
  return fused_geometry(H, I, G).stages >= 2;
}

int fused_max_work_segments(int M, int max_seg, int max_blocks) {
  const int shared_blocks = (M + kFBM - 1) / kFBM;
  return max_seg + max_blocks / kWsBlocks + (shared_blocks + kWsBlocks - 1) / kWsBlocks + 2;
}

int launch_moe_fused(const FusedArgs& a_in, cudaStream_t st) {
  FusedArgs a = a_in;
  const FusedGeometry f = fused_geometry(a.H, a.I, a.G);
  a.stages = f.stages;
  a.stage_bytes = f.stage_bytes;
  a.xbuf_bytes = f.xbuf_bytes;
  int w1c, w2c;
  fused_template(a.H, a.I, &w1c, &w2c);
#define MTP_FUSED_CASE(A, B) \
  if (w1c == A && w2c == B) return launch_fused_t<A, B>(a, f, st);
  MTP_FUSED_CASE(1, 1)
  MTP_FUSED_CASE(1, 2)
  MTP_FUSED_CASE(1, 3)
  MTP_FUSED_CASE(1, 4)
  MTP_FUSED_CASE(1, 5)
  MTP_FUSED_CASE(1, 6)
  MTP_FUSED_CASE(1, 7)
  MTP_FUSED_CASE(1, 8)
  MTP_FUSED_CASE(2, 1)
  MTP_FUSED_CASE(2, 2)
  MTP_FUSED_CASE(2, 3)
  MTP_FUSED_CASE(2, 4)
  MTP_FUSED_CASE(2, 5)
  MTP_FUSED_CASE(2, 6)
  MTP_FUSED_CASE(2, 7)
  MTP_FUSED_CASE(2, 8)
#undef MTP_FUSED_CASE
  return MTP_ERR_SHAPE;
}

}  // namespace mtp
