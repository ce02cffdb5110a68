// W4A16 MoE layer forward for decode-sized batches on sm_100a.
//
// Work unit = (expert, weight strip group). The expert's packed int4 weights
// are streamed once from HBM with 16-byte no-L1-allocate loads, issued before
// anything else in the CTA so the whole working set is in flight at once;
// they stay in registers while every token block (8 routed (token, slot)
// pairs) of that expert is processed, so each weight byte is read once per
// layer call whatever the number of tokens routed to the expert.
//
// Arithmetic per 16x16 weight tile: one packed word per thread is turned into
// the four A-fragment registers of an m16n8k16 bf16 MMA by exponent-bias
// dequantisation (q - z exact in bf16, see common.cuh); the tile is multiplied
// with the 8 tokens of the block (B operand from shared memory) into a per
// group fp32 partial, which is scaled by the fp16 group scale in fp32 and
// added to the accumulator. So the weights enter the products unrounded:
// sum_k x_k (q_k - z) s_g = s_g * sum_k x_k (q_k - z).
//
// Kernels (one layer call):
//   W1   grid (I/16, units): gate strip i and up strip i of one expert, K = H
//        split over H/256 warps, cross-warp reduction in shared memory, then
//        h = silu(gate) * up stored as bf16 [pairs, I]
//        (fused_moe W1 + silu_and_mul, vllm_router_trace.py:19674-19719).
//   W2   grid (H/128, units): 8 strips of 16 output rows, K = I per warp;
//        routed pairs are multiplied by their router weight
//        (MUL_ROUTED_WEIGHT, vllm_router_trace.py:19761-19782) and stored fp32.
//   combine grid (M, H/1024): out = sum_j y[t,j] + sigmoid(x.w_g) * shared(x)
//        (moe_sum :19801 and the shared-expert gate :3994-4031, :4140-4152).
//
// A unit is either the shared expert (all M tokens, when present; unit 0) or
// one segment of the align output (expert, first block, block count). The
// expert's blob is found through the slot table: slot >= 0 reads the resident
// cache, slot -1 reads the pinned host store through its device mapping
// (demand fetch over the host link), and with no host store the expert's
// contribution is zero and counted in status[1].
#include "internal.cuh"

namespace mtp {

constexpr int kBM = 8;  // token (pair) block = MMA N


struct Unit {
  const uint8_t* blob;
  int b0, nb, shared, valid, miss_host, miss_none;
};

__device__ __forceinline__ Unit resolve_unit(const MoeDevArgs& a, int u) {
  Unit U{nullptr, 0, 0, 0, 0, 0, 0};
  if (a.has_shared) {
    if (u == 0) {
      U.blob = a.shared_blob;
      U.nb = (a.M + kBM - 1) / kBM;
      U.shared = 1;
      U.valid = 1;
      return U;
    }
    --u;
  }
  if (u >= *a.nseg) return U;
  const int e = a.segs[3 * u];
  U.b0 = a.segs[3 * u + 1];
  U.nb = a.segs[3 * u + 2];
  U.valid = 1;
  const int slot = a.slot_table ? a.slot_table[e] : e;
  if (slot >= 0) {
    U.blob = a.blobs + static_cast<int64_t>(slot) * a.expert_bytes;
  } else if (a.host_blobs) {
    U.blob = a.host_blobs + static_cast<int64_t>(e) * a.expert_bytes;
    U.miss_host = 1;
  } else {
    U.miss_none = 1;
  }
  return U;
}

// Column c of token block blk: returns the pair row (h / y row) or -1, and the
// x row through *xrow.
__device__ __forceinline__ int block_pair(const MoeDevArgs& a, const Unit& U, int blk, int c,
                                          int* xrow) {
  if (U.shared) {
    const int t = blk * kBM + c;
    if (t >= a.M) return -1;
    *xrow = t;
    return a.numel + t;
  }
  const int p = a.sorted[(U.b0 + blk) * kBM + c];
  if (p < 0 || p >= a.numel) return -1;
  *xrow = p / a.k;
  return p;
}

__device__ __forceinline__ uint32_t pick(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

__device__ __forceinline__ void zero_biases(uint32_t zbyte, int zero_mode, uint32_t* lo,
                                            uint32_t* hi) {
  if (zero_mode == MTP_ZERO_SYM8) {
    *lo = *hi = zero_bias_pair(8);
  } else {
    *lo = zero_bias_pair(zbyte & 0xF);
    *hi = zero_bias_pair(zbyte >> 4);
  }
}

// Stage the 8 rows of a token block into shared memory, [8][cols + 16] bf16.
// Inside every 16-element k group the elements are permuted so that lane
// t's B fragment (k = 2t, 2t+1, 2t+8, 2t+9) is 8 contiguous bytes at 4t:
// element e < 8 goes to 4(e/2) + e%2, element e >= 8 to 4((e-8)/2) + 2 + e%2.
// The 16-element row pad makes the 8-byte fragment loads bank-conflict free.
constexpr int kRowPad = 16;

__device__ __forceinline__ void stage_rows_permuted(uint16_t* dst, int cols,
                                                    const uint16_t* const* rows) {
  const int grp = cols / 16;  // 16-element groups per row
  for (int idx = threadIdx.x; idx < kBM * grp; idx += blockDim.x) {
    const int r = idx / grp, q = idx % grp;
    const uint16_t* src = rows[r];
    uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
    if (src) {
      lo = *reinterpret_cast<const uint4*>(src + q * 16);
      hi = *reinterpret_cast<const uint4*>(src + q * 16 + 8);
    }
    uint4* d = reinterpret_cast<uint4*>(dst + r * (cols + kRowPad) + q * 16);
    d[0] = make_uint4(lo.x, hi.x, lo.y, hi.y);
    d[1] = make_uint4(lo.z, hi.z, lo.w, hi.w);
  }
}

// Resolve the 8 columns of token block blk once per block: pair row (or -1)
// and the source row pointer for staging (x rows for W1, h rows for W2).
__device__ __forceinline__ void resolve_block(const MoeDevArgs& a, const Unit& U, int blk,
                                              bool w1, int* pair_s, const uint16_t** src_s) {
  if (threadIdx.x < kBM) {
    const int c = threadIdx.x;
    int xr = 0;
    const int p = block_pair(a, U, blk, c, &xr);
    pair_s[c] = p;
    const uint16_t* src = nullptr;
    if (p >= 0 && U.blob)
      src = w1 ? a.x + static_cast<int64_t>(xr) * a.H : a.hbuf + static_cast<int64_t>(p) * a.I;
    src_s[c] = src;
  }
}

// ---------------------------------------------------------------------------
// W1: gate_up + SiLU * up
// ---------------------------------------------------------------------------
template <int G>
__global__ void __launch_bounds__(256) moe_w1_kernel(MoeDevArgs a) {
  constexpr int GPW = 256 / G;  // groups per warp (each warp covers 256 of K)
  constexpr int CPG = G / 64;   // 64-wide chunks per group
  const Unit U = resolve_unit(a, blockIdx.y);
  if (!U.valid) return;
  const int strip = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int nw = blockDim.x >> 5;
  const int H = a.H, C = H / 64, Gn = H / G;
  const int sidx[2] = {strip, a.I / 16 + strip};

  if (!U.shared && threadIdx.x == 0 && blockIdx.x == 0 && a.status) {
    if (U.miss_host) atomicAdd(a.status + 0, 1);
    if (U.miss_none) atomicAdd(a.status + 1, 1);
  }

  // 1. Issue this thread's weight loads first: 2 strips x 4 chunks x 16 B.
  uint4 wv[2][4];
  uint32_t scw[2][GPW], zlo[2][GPW], zhi[2][GPW];
  if (U.blob) {
    const uint8_t* qw = U.blob + a.L.w13_qweight;
#pragma unroll
    for (int st = 0; st < 2; ++st)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        wv[st][j] = ldg_stream16(qw + ((static_cast<int64_t>(sidx[st]) * C + 4 * warp + j) * 32 + lane) * 16);
    const uint8_t* sc = U.blob + a.L.w13_scales;
    const uint8_t* zp = U.blob + a.L.w13_zeros;
#pragma unroll
    for (int st = 0; st < 2; ++st)
#pragma unroll
      for (int q = 0; q < GPW; ++q) {
        const int64_t sg = static_cast<int64_t>(sidx[st]) * Gn + warp * GPW + q;
        scw[st][q] = ldg_u32(sc + (sg * 8 + g) * 4);
        const uint32_t zb = a.zero_mode == MTP_ZERO_RAW ? ldg_u8(zp + sg * 8 + g) : 0x88u;
        zero_biases(zb, a.zero_mode, &zlo[st][q], &zhi[st][q]);
      }
  }

  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem_raw);
  float* red = reinterpret_cast<float*>(smem_raw + kBM * (H + kRowPad) * 2);  // [nw][2][4][32]
  float* red2 = red + nw * 256;                                              // [2][4][32]
  const int XS = H + kRowPad;

  __shared__ int pair_s[kBM];
  __shared__ const uint16_t* src_s[kBM];
  for (int blk = 0; blk < U.nb; ++blk) {
    __syncthreads();
    resolve_block(a, U, blk, true, pair_s, src_s);
    __syncthreads();
    stage_rows_permuted(xs, H, src_s);
    __syncthreads();

    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    if (U.blob) {
#pragma unroll
      for (int q = 0; q < GPW; ++q) {
        float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int cc = 0; cc < CPG; ++cc) {
          const int j = q * CPG + cc;
          const int c = 4 * warp + j;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            uint32_t b0, b1;
            lds_bfrag(xs + g * XS + 64 * c + 16 * kk + 4 * t, &b0, &b1);
#pragma unroll
            for (int st = 0; st < 2; ++st) {
              uint32_t A[4];
              dequant_word(pick(wv[st][j], kk), zlo[st][q], zhi[st][q], A);
              mma_bf16_16816(d[st], A, b0, b1);
            }
          }
        }
#pragma unroll
        for (int st = 0; st < 2; ++st) {
          const float2 s = half2_bits_to_float2(scw[st][q]);
          acc[st][0] = fmaf(s.x, d[st][0], acc[st][0]);
          acc[st][1] = fmaf(s.x, d[st][1], acc[st][1]);
          acc[st][2] = fmaf(s.y, d[st][2], acc[st][2]);
          acc[st][3] = fmaf(s.y, d[st][3], acc[st][3]);
        }
      }
    }
#pragma unroll
    for (int st = 0; st < 2; ++st)
#pragma unroll
      for (int r = 0; r < 4; ++r) red[((warp * 2 + st) * 4 + r) * 32 + lane] = acc[st][r];
    __syncthreads();
    for (int idx = threadIdx.x; idx < 256; idx += blockDim.x) {
      float s = 0.f;
      for (int w = 0; w < nw; ++w) s += red[w * 256 + idx];
      red2[idx] = s;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < 128; idx += blockDim.x) {
      const int r = idx >> 5, l = idx & 31;
      const int row = (l >> 2) + 8 * (r >> 1);
      const int col = 2 * (l & 3) + (r & 1);
      const int p = pair_s[col];
      if (p >= 0) {
        const float gate = red2[idx], up = red2[128 + idx];
        const float h = silu(gate) * up;
        a.hbuf[static_cast<int64_t>(p) * a.I + 16 * strip + row] =
            __bfloat16_as_ushort(__float2bfloat16(h));
      }
    }
  }
}

// ---------------------------------------------------------------------------
// W2: down projection (+ routed weight)
// ---------------------------------------------------------------------------
template <int G, int MAXC>
__global__ void __launch_bounds__(256) moe_w2_kernel(MoeDevArgs a) {
  constexpr int CPG = G / 64;
  constexpr int MAXG = MAXC / CPG;
  const Unit U = resolve_unit(a, blockIdx.y);
  if (!U.valid) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int s = blockIdx.x * 8 + warp;  // strip of 16 output rows
  const int H = a.H, I = a.I, C = I / 64, Gn = I / G;

  uint4 wv[MAXC];
  uint32_t scw[MAXG], zlo[MAXG], zhi[MAXG];
  if (U.blob) {
    const uint8_t* qw = U.blob + a.L.w2_qweight;
#pragma unroll
    for (int j = 0; j < MAXC; ++j)
      if (j < C) wv[j] = ldg_stream16(qw + ((static_cast<int64_t>(s) * C + j) * 32 + lane) * 16);
    const uint8_t* sc = U.blob + a.L.w2_scales;
    const uint8_t* zp = U.blob + a.L.w2_zeros;
#pragma unroll
    for (int q = 0; q < MAXG; ++q)
      if (q < Gn) {
        const int64_t sg = static_cast<int64_t>(s) * Gn + q;
        scw[q] = ldg_u32(sc + (sg * 8 + g) * 4);
        const uint32_t zb = a.zero_mode == MTP_ZERO_RAW ? ldg_u8(zp + sg * 8 + g) : 0x88u;
        zero_biases(zb, a.zero_mode, &zlo[q], &zhi[q]);
      }
  }

  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint16_t* hs = reinterpret_cast<uint16_t*>(smem_raw);
  const int HS = I + kRowPad;

  __shared__ int pair_s[kBM];
  __shared__ const uint16_t* src_s[kBM];
  for (int blk = 0; blk < U.nb; ++blk) {
    __syncthreads();
    resolve_block(a, U, blk, false, pair_s, src_s);
    __syncthreads();
    stage_rows_permuted(hs, I, src_s);
    __syncthreads();

    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    if (U.blob) {
#pragma unroll
      for (int q = 0; q < MAXG; ++q) {
        if (q < Gn) {
          float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int cc = 0; cc < CPG; ++cc) {
            const int j = q * CPG + cc;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              uint32_t b0, b1;
              lds_bfrag(hs + g * HS + 64 * j + 16 * kk + 4 * t, &b0, &b1);
              uint32_t A[4];
              dequant_word(pick(wv[j], kk), zlo[q], zhi[q], A);
              mma_bf16_16816(d, A, b0, b1);
            }
          }
          const float2 sv = half2_bits_to_float2(scw[q]);
          acc[0] = fmaf(sv.x, d[0], acc[0]);
          acc[1] = fmaf(sv.x, d[1], acc[1]);
          acc[2] = fmaf(sv.y, d[2], acc[2]);
          acc[3] = fmaf(sv.y, d[3], acc[3]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int row = g + 8 * (r >> 1);
      const int col = 2 * t + (r & 1);
      const int p = pair_s[col];
      if (p >= 0) {
        const float w = U.shared ? 1.f : a.topk_w[p];
        a.ybuf[static_cast<int64_t>(p) * H + 16 * s + row] = acc[r] * w;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// combine: top-k sum + sigmoid-gated shared expert
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) moe_combine_kernel(MoeDevArgs a, const uint16_t* gate_w,
                                                          uint16_t* out, float* out_f32) {
  const int tkn = blockIdx.x;
  const int H = a.H;
  __shared__ float red[8];
  float gate = 0.f;
  if (a.has_shared) {
    float part = 0.f;
    const uint16_t* xr = a.x + static_cast<int64_t>(tkn) * H;
    for (int h = threadIdx.x; h < H; h += blockDim.x)
      part += bf16_bits_to_float(xr[h]) * bf16_bits_to_float(gate_w[h]);
    part = warp_sum(part);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = part;
    __syncthreads();
    float dot = 0.f;
    for (int w = 0; w < (blockDim.x >> 5); ++w) dot += red[w];
    gate = 1.f / (1.f + __expf(-dot));
  }
  const int n0 = (blockIdx.y * blockDim.x + threadIdx.x) * 4;
  if (n0 >= H) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j = 0; j < a.k; ++j) {
    const int p = tkn * a.k + j;
    const int e = a.topk_ids[p];
    if (e < 0 || e >= a.E) continue;
    const float4 y = *reinterpret_cast<const float4*>(a.ybuf + static_cast<int64_t>(p) * H + n0);
    acc.x += y.x; acc.y += y.y; acc.z += y.z; acc.w += y.w;
  }
  if (a.has_shared) {
    const float4 y = *reinterpret_cast<const float4*>(a.ybuf + static_cast<int64_t>(a.numel + tkn) * H + n0);
    acc.x = fmaf(gate, y.x, acc.x);
    acc.y = fmaf(gate, y.y, acc.y);
    acc.z = fmaf(gate, y.z, acc.z);
    acc.w = fmaf(gate, y.w, acc.w);
  }
  const int64_t o = static_cast<int64_t>(tkn) * H + n0;
  __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y);
  __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z, acc.w);
  uint2 packed;
  packed.x = *reinterpret_cast<uint32_t*>(&lo);
  packed.y = *reinterpret_cast<uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(out + o) = packed;
  if (out_f32) *reinterpret_cast<float4*>(out_f32 + o) = acc;
}

__global__ void demand_log_kernel(const int32_t* segs, const int32_t* nseg, int32_t* log) {
  const int n = *nseg;
  if (threadIdx.x == 0) log[0] = n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) log[1 + i] = segs[3 * i];
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------
static size_t w1_smem(int H) { return static_cast<size_t>(kBM) * (H + kRowPad) * 2 + (H / 256) * 1024 + 1024; }
static size_t w2_smem(int I) { return static_cast<size_t>(kBM) * (I + kRowPad) * 2; }

template <typename K>
static int ensure_smem(K kernel, size_t bytes) {
  if (bytes <= 48 * 1024) return MTP_OK;
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(bytes)) == cudaSuccess
             ? MTP_OK
             : MTP_ERR_CUDA;
}

int launch_moe_decode(const MoeDevArgs& a, int G, const uint16_t* gate_w, uint16_t* out,
                      float* out_f32, int32_t* demand_log, cudaStream_t st) {
  const int units = a.max_seg + a.has_shared;
  if (demand_log) demand_log_kernel<<<1, 256, 0, st>>>(a.segs, a.nseg, demand_log);
  {
    const dim3 grid(a.I / 16, units);
    const int threads = a.H / 8;
    const size_t smem = w1_smem(a.H);
    int r;
    if (G == 128) {
      if ((r = ensure_smem(moe_w1_kernel<128>, smem)) != MTP_OK) return r;
      moe_w1_kernel<128><<<grid, threads, smem, st>>>(a);
    } else {
      if ((r = ensure_smem(moe_w1_kernel<64>, smem)) != MTP_OK) return r;
      moe_w1_kernel<64><<<grid, threads, smem, st>>>(a);
    }
    if ((r = launch_status()) != MTP_OK) return r;
  }
  {
    const dim3 grid(a.H / 128, units);
    const size_t smem = w2_smem(a.I);
    const int C = a.I / 64;
    if (G == 128) {
      if (C <= 8) moe_w2_kernel<128, 8><<<grid, 256, smem, st>>>(a);
      else moe_w2_kernel<128, 16><<<grid, 256, smem, st>>>(a);
    } else {
      if (C <= 8) moe_w2_kernel<64, 8><<<grid, 256, smem, st>>>(a);
      else moe_w2_kernel<64, 16><<<grid, 256, smem, st>>>(a);
    }
    const int r = launch_status();
    if (r != MTP_OK) return r;
  }
  {
    const dim3 grid(a.M, (a.H + 1023) / 1024);
    moe_combine_kernel<<<grid, 256, 0, st>>>(a, gate_w, out, out_f32);
  }
  return launch_status();
}

}  // namespace mtp
