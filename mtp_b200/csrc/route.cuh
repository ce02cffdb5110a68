// Router (one warp per token) and moe_align_block_size (one 1024-thread
// block) as device functions, shared by the standalone kernels
// (router_align.cu) and the fused layer's route kernel (moe_fused.cu).
//
// Router: the E logits of a token are spread over the 32 lanes (E/32 values
// per lane, in registers); softmax statistics and the k argmax rounds are warp
// shuffles. Semantics: vLLM topk_softmax as the reference restates it
// (tracing/vllm_router_trace.py:4201-4227): softmax over all E, top-k
// descending (exact ties -> lower expert id), optional renormalisation with the
// sum clamped to 1e-20.
//
// Align: counting by shared-memory histogram, a block scan for the padded
// per-expert offsets, then a scatter in canonical order (experts ascending,
// flat pair index ascending inside an expert): each 1024-pair chunk is ranked
// with __match_any_sync inside a warp plus per-warp per-expert counts for the
// warps before it, so the result does not depend on scheduling. Semantics:
// vLLM moe_align_block_size (fused_moe/moe_align_block_size.py).
#pragma once

#include "common.cuh"

#include <math.h>

namespace mtp {

// One warp computes token `row`'s top-k. Lane j < k returns result j.
template <int VPT>
__device__ __forceinline__ void router_token(const float* __restrict__ row, int E, int k, int renorm,
                                             float* w_out, int* id_out) {
  const int lane = threadIdx.x & 31;
  float v[VPT];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = lane + 32 * i;
    v[i] = idx < E ? row[idx] : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
  mx = warp_max(mx);
  float ex[VPT];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int idx = lane + 32 * i;
    ex[i] = idx < E ? expf(v[i] - mx) : 0.f;
    s += ex[i];
  }
  s = warp_sum(s);

  uint32_t taken = 0;
  float my_w = 0.f;
  int my_id = 0;
  float wsum = 0.f;
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int idx = lane + 32 * i;
      if (idx < E && !((taken >> i) & 1u)) {
        if (v[i] > bv || (v[i] == bv && idx < bi)) {
          bv = v[i];
          bi = idx;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(kFullMask, bv, o);
      const int oi = __shfl_xor_sync(kFullMask, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    const int owner = bi & 31;
    const int slot = bi >> 5;
    float p = 0.f;
    if (lane == owner) {
      taken |= 1u << slot;
#pragma unroll
      for (int i = 0; i < VPT; ++i)
        if (i == slot) p = ex[i] / s;
    }
    p = __shfl_sync(kFullMask, p, owner);
    wsum += p;
    if (lane == j) {
      my_w = p;
      my_id = bi;
    }
  }
  if (renorm) my_w = my_w / fmaxf(wsum, 1e-20f);
  *w_out = my_w;
  *id_out = my_id;
}

constexpr int kAlignThreads = 1024;

inline size_t align_smem_bytes(int E) { return static_cast<size_t>(35) * E * sizeof(int); }

__device__ __forceinline__ int block_exclusive_scan(int v, int* total, int* tmp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(kFullMask, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) tmp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int t = tmp[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(kFullMask, t, o);
      if (lane >= o) t += y;
    }
    tmp[lane] = t;  // inclusive over warps
  }
  __syncthreads();
  const int warp_base = warp > 0 ? tmp[warp - 1] : 0;
  *total = tmp[31];
  __syncthreads();
  return warp_base + x - v;
}

__device__ __forceinline__ int align_key(const int32_t* ids, int i, int E, const int32_t* emap,
                                         int ignore_invalid) {
  const int e = ids[i];
  if (e < 0 || e >= E) return -1;
  if (emap != nullptr && ignore_invalid && emap[e] < 0) return -1;
  return e;
}

// Whole-block moe_align_block_size. Requires blockDim.x == kAlignThreads and
// `sm` = align_smem_bytes(E) bytes of shared memory; E <= 1024.
static __device__ void align_block(const int32_t* __restrict__ ids, int numel, int E, int BM,
                            const int32_t* __restrict__ emap, int ignore_invalid, int cap,
                            int max_blocks, int max_seg, int32_t* __restrict__ sorted,
                            int32_t* __restrict__ eids, int32_t* __restrict__ ntpp,
                            int32_t* __restrict__ segs, int32_t* __restrict__ nseg, int* sm,
                            int* scan_tmp) {
  int* cnt = sm;            // [E]
  int* off = cnt + E;       // [E]
  int* run = off + E;       // [E]
  int* wcnt = run + E;      // [32][E]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < E; e += kAlignThreads) {
    cnt[e] = 0;
    run[e] = 0;
  }
  for (int x = tid; x < 32 * E; x += kAlignThreads) wcnt[x] = 0;
  __syncthreads();
  for (int i = tid; i < numel; i += kAlignThreads) {
    const int key = align_key(ids, i, E, emap, ignore_invalid);
    if (key >= 0) atomicAdd(&cnt[key], 1);
  }
  __syncthreads();

  const int c = tid < E ? cnt[tid] : 0;
  const int padded = (c + BM - 1) / BM * BM;
  int total_padded, total_has;
  const int ex_pad = block_exclusive_scan(padded, &total_padded, scan_tmp);
  const int ex_has = block_exclusive_scan(c > 0 ? 1 : 0, &total_has, scan_tmp);
  if (tid < E) off[tid] = ex_pad;
  if (tid == 0) {
    *ntpp = total_padded;
    if (nseg) *nseg = total_has;
  }
  if (tid < E && c > 0) {
    const int b0 = ex_pad / BM, nb = padded / BM;
    const int tag = emap ? emap[tid] : tid;
    for (int b = 0; b < nb; ++b) eids[b0 + b] = tag;
    for (int p = ex_pad + c; p < ex_pad + padded; ++p) sorted[p] = numel;
    if (segs) {
      segs[3 * ex_has + 0] = tid;
      segs[3 * ex_has + 1] = b0;
      segs[3 * ex_has + 2] = nb;
    }
  }
  for (int p = total_padded + tid; p < cap; p += kAlignThreads) sorted[p] = numel;
  for (int b = total_padded / BM + tid; b < max_blocks; b += kAlignThreads) eids[b] = -1;
  if (segs)
    for (int s = total_has + tid; s < max_seg; s += kAlignThreads) {
      segs[3 * s + 0] = -1;
      segs[3 * s + 1] = 0;
      segs[3 * s + 2] = 0;
    }
  __syncthreads();

  const unsigned lt_mask = (1u << lane) - 1u;
  for (int c0 = 0; c0 < numel; c0 += kAlignThreads) {
    const int i = c0 + tid;
    const int key = i < numel ? align_key(ids, i, E, emap, ignore_invalid) : -1;
    const unsigned mask = __match_any_sync(kFullMask, key);
    const int rank = __popc(mask & lt_mask);
    const int leader = __ffs(mask) - 1;
    const int cw = __popc(mask);
    if (key >= 0 && lane == leader) wcnt[warp * E + key] = cw;
    __syncthreads();
    int base = 0;
    if (key >= 0 && lane == leader) {
      base = run[key];
      for (int w = 0; w < warp; ++w) base += wcnt[w * E + key];
    }
    base = __shfl_sync(kFullMask, base, leader);
    if (key >= 0) sorted[off[key] + base + rank] = i;
    __syncthreads();
    if (key >= 0 && lane == leader) {
      atomicAdd(&run[key], cw);
      wcnt[warp * E + key] = 0;
    }
    __syncthreads();
  }
}

}  // namespace mtp
