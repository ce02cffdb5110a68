// MTP expert-demand predictor: logits = W2 . silu(W1 . h + b1) + b2 for each
// hidden state h (H -> width -> F x E), then the top-k experts of every
// future layer f (descending logit, exact ties to the lower expert id). The
// reference family is HiddenResidualExpertPredictor
// (training/hidden_residual.py:44-134: Linear -> SiLU -> Linear classifier per
// future delta) and its ranking is topk(logits.float()) (recall_at_m,
// training/predictor.py:105).
//
// Both linears are bf16 GEMVs with M <= 64 columns at decode: HBM-bound on the
// weight bytes. Weights are prepacked once (mtp_predictor_pack) into the
// m16n8k16 A-fragment order so that every lane streams its fragments with one
// 16-byte load per k16 step (a warp reads 512 contiguous bytes). One CTA owns
// 16 output rows over one of KS slices of K (KS chosen so that about 200 or
// more CTAs stream, two per SM); its 8 warps split the slice, and the token
// columns are processed in chunks of 16 staged in shared memory while the
// weight fragments stay in registers. The cross-warp sums are reduced in
// shared memory in a fixed order and written as fp32 partial slices; the next
// kernel of the chain adds the slices in slice order, then the bias, and
// either applies SiLU and rounds to bf16 (the first linear's output, finished
// while staging) or ranks the fp32 logits (top-k).
#include "internal.cuh"

namespace mtp {

namespace {

constexpr int kPWarps = 8;
constexpr int kPThreads = kPWarps * 32;
constexpr int kTokChunk = 16;  // token columns per staged chunk (two n8 tiles)
constexpr int kMaxKPerWarp = 128;  // 8 weight fragments per lane: two CTAs fit an SM's registers

// mma.sync m16n8k16 bf16 x bf16 -> fp32 (the predictor's weights are plain
// bf16: no dequantisation, so the register-operand MMA is the direct fit).
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint4& a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

// Prepack W [rows, cols] bf16 (row-major, out x in) into
// [rows/16][cols/16][32 lanes][4 words]: lane (g = l/4, t = l%4) of (strip s,
// k-step c) holds a0 = W[16s+g][16c+2t..], a1 = W[16s+g+8][16c+2t..],
// a2 = W[16s+g][16c+8+2t..], a3 = W[16s+g+8][16c+8+2t..].
__global__ void pack_kernel(const uint32_t* __restrict__ w, int rows, int cols, uint32_t* __restrict__ out) {
  const int64_t words = static_cast<int64_t>(rows) * cols / 2;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= words) return;
  const int j = static_cast<int>(i & 3), l = static_cast<int>((i >> 2) & 31);
  const int64_t sc = i >> 7;
  const int ksteps = cols / 16;
  const int c = static_cast<int>(sc % ksteps), s = static_cast<int>(sc / ksteps);
  const int g = l >> 2, t = l & 3;
  const int row = 16 * s + g + 8 * (j & 1);
  const int k = 16 * c + 2 * t + 8 * (j >> 1);
  out[i] = w[(static_cast<int64_t>(row) * cols + k) / 2];
}

// One linear layer's share: CTA (strip, ks) takes the 16 output rows of its
// strip over K range ks of KS (all M token columns) and writes fp32 partial
// sums part[ks][m][row] (no bias): KS > 1 spreads the weight stream over more
// SMs, and the consumer adds the KS slices in a fixed order, so the result
// does not depend on scheduling. The input is either bf16 rows x [M][K], or
// (x == NULL) the previous linear's fp32 partials xin[KSin][M][K], finished
// on load: bf16(silu(sum + xbias)).
__global__ void __launch_bounds__(kPThreads, 2) gemv_kernel(const uint16_t* __restrict__ x,
                                                         const float* __restrict__ xin, int KSin,
                                                         const uint16_t* __restrict__ xbias, int M, int K,
                                                         const uint4* __restrict__ wp, int R, int KS,
                                                         float* __restrict__ part) {
  extern __shared__ __align__(16) uint8_t psm[];
  // the staged bf16 row holds this CTA's K range only (+ 16 bytes: conflict-free B fragments)
  const int row_stride = 2 * (K / KS) + 16;
  uint8_t* hs = psm;                                                            // [16][row_stride]
  float* red = reinterpret_cast<float*>(psm + kTokChunk * row_stride);          // [8 warps][16 rows][16 tok]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int strip = blockIdx.x / KS, ks = blockIdx.x % KS;
  const int kpw = K / KS / kPWarps;  // K per warp (<= 128): kpw / 16 k-steps
  const int ks0 = (ks * (K / KS)) / 16 + warp * (kpw / 16);
  // Let the next kernel of the chain start streaming its own weights now.
  pdl_launch_dependents();
  // this warp's weight fragments, loaded once (16-byte loads, streaming);
  // they do not depend on the previous kernel, so they are issued before
  // waiting for it
  uint4 a[kMaxKPerWarp / 16];
  const uint4* src = wp + (static_cast<int64_t>(strip) * (K / 16) + ks0) * 32 + lane;
#pragma unroll
  for (int i = 0; i < kMaxKPerWarp / 16; ++i)
    if (i < kpw / 16) a[i] = ldg_stream16(src + i * 32);
  pdl_wait();  // x is the previous kernel's output
  const int kb = ks * (K / KS), kn = K / KS;  // this CTA's K range (staged columns)
  for (int c0 = 0; c0 < M; c0 += kTokChunk) {
    // stage the K range of token rows c0..c0+15 (zero rows past M)
    const int vecs = kn / 8;
    for (int i = threadIdx.x; i < kTokChunk * vecs; i += kPThreads) {
      const int n = i / vecs, v = i % vecs;
      uint4 val = make_uint4(0u, 0u, 0u, 0u);
      if (c0 + n < M) {
        const int64_t off = static_cast<int64_t>(c0 + n) * K + kb + 8 * v;
        if (x) {
          val = *reinterpret_cast<const uint4*>(x + off);
        } else {
          // every slice's loads issued together (one L2 round trip), then
          // summed in slice order
          float4 p0[kMaxPredictorKs], p1[kMaxPredictorKs];
#pragma unroll
          for (int q = 0; q < kMaxPredictorKs; ++q) {
            if (q < KSin) {
              p0[q] = __ldcg(reinterpret_cast<const float4*>(xin + q * static_cast<int64_t>(M) * K + off));
              p1[q] = __ldcg(reinterpret_cast<const float4*>(xin + q * static_cast<int64_t>(M) * K + off + 4));
            }
          }
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = 0.f;
#pragma unroll
          for (int q = 0; q < kMaxPredictorKs; ++q) {
            if (q < KSin) {
              f[0] += p0[q].x; f[1] += p0[q].y; f[2] += p0[q].z; f[3] += p0[q].w;
              f[4] += p1[q].x; f[5] += p1[q].y; f[6] += p1[q].z; f[7] += p1[q].w;
            }
          }
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float u0 = f[2 * e], u1 = f[2 * e + 1];
            if (xbias) {
              u0 += __bfloat162float(__ushort_as_bfloat16(xbias[kb + 8 * v + 2 * e]));
              u1 += __bfloat162float(__ushort_as_bfloat16(xbias[kb + 8 * v + 2 * e + 1]));
            }
            const __nv_bfloat162 h = __floats2bfloat162_rn(u0 / (1.f + expf(-u0)), u1 / (1.f + expf(-u1)));
            w[e] = *reinterpret_cast<const uint32_t*>(&h);
          }
          val = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      *reinterpret_cast<uint4*>(hs + n * row_stride + v * 16) = val;
    }
    __syncthreads();
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int i = 0; i < kMaxKPerWarp / 16; ++i) {
      if (i < kpw / 16) {
        const int k = warp * kpw + i * 16 + 2 * t;  // within the staged range
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const uint8_t* hrow = hs + (nt * 8 + g) * row_stride;
          const uint32_t b0 = *reinterpret_cast<const uint32_t*>(hrow + 2 * k);
          const uint32_t b1 = *reinterpret_cast<const uint32_t*>(hrow + 2 * (k + 8));
          mma_bf16(acc[nt], a[i], b0, b1);
        }
      }
    }
    // D fragment: (row g, cols 2t, 2t+1) = acc[0..1], (row g+8, ...) = acc[2..3]
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int row = g + 8 * (r >> 1), col = nt * 8 + 2 * t + (r & 1);
        red[(warp * 16 + row) * kTokChunk + col] = acc[nt][r];
      }
    __syncthreads();
    {
      const int row = threadIdx.x / kTokChunk, col = threadIdx.x % kTokChunk;  // 256 = 16 x 16
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kPWarps; ++w) v += red[(w * 16 + row) * kTokChunk + col];
      const int orow = strip * 16 + row, m = c0 + col;
      if (m < M) part[(static_cast<int64_t>(ks) * M + m) * R + orow] = v;
    }
    __syncthreads();
  }
}

// HiddenResidualExpertPredictor's middle (training/hidden_residual.py:86-103),
// one warp per token m: a = silu(sum of the first linear's KS partial slices
// + b1), state = LayerNorm(a) (biased variance, eps, weight, bias), then for
// every future delta f the classifier's input column m * F + f =
// bf16(silu(state + layer_emb[layer_ids[m]] + delta_emb[f])). Width <= 2048.
__global__ void hr_context_kernel(const float* __restrict__ part, int KS, const uint16_t* __restrict__ b1,
                                  int M, int W, const uint16_t* __restrict__ ln_w, const uint16_t* __restrict__ ln_b,
                                  float eps, const uint16_t* __restrict__ layer_emb, int num_layers,
                                  const int32_t* __restrict__ layer_ids, const uint16_t* __restrict__ delta_emb,
                                  int F, uint16_t* __restrict__ ctx) {
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m = blockIdx.x * (blockDim.x >> 5) + warp;
  if (m >= M) return;
  constexpr int kPer = 2048 / 32;
  float a[kPer];
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int c = lane + 32 * j;
    a[j] = c < W && b1 ? __bfloat162float(__ushort_as_bfloat16(b1[c])) : 0.f;
  }
  // slice by slice, all columns' loads of a slice in flight together
#pragma unroll
  for (int q = 0; q < kMaxPredictorKs; ++q) {
    if (q < KS) {
      const float* src = part + (static_cast<int64_t>(q) * M + m) * W;
#pragma unroll
      for (int j = 0; j < kPer; ++j)
        if (lane + 32 * j < W) a[j] += __ldcg(src + lane + 32 * j);
    }
  }
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    if (lane + 32 * j < W) {
      a[j] = a[j] / (1.f + expf(-a[j]));
      sum += a[j];
    }
  }
  const float mean = warp_sum(sum) / W;
  float var = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j)
    if (lane + 32 * j < W) var += (a[j] - mean) * (a[j] - mean);
  const float rstd = rsqrtf(warp_sum(var) / W + eps);
  int lid = layer_ids ? layer_ids[m] : 0;
  lid = lid < 0 ? 0 : (lid >= num_layers ? num_layers - 1 : lid);
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int c = lane + 32 * j;
    if (c >= W) continue;
    float st = (a[j] - mean) * rstd;
    if (ln_w) st *= __bfloat162float(__ushort_as_bfloat16(ln_w[c]));
    if (ln_b) st += __bfloat162float(__ushort_as_bfloat16(ln_b[c]));
    st += __bfloat162float(__ushort_as_bfloat16(layer_emb[static_cast<int64_t>(lid) * W + c]));
    for (int f = 0; f < F; ++f) {
      const float u = st + __bfloat162float(__ushort_as_bfloat16(delta_emb[static_cast<int64_t>(f) * W + c]));
      ctx[(static_cast<int64_t>(m) * F + f) * W + c] = __bfloat16_as_ushort(__float2bfloat16(u / (1.f + expf(-u))));
    }
  }
}

// Top-k of each row of E logits (one warp per row; E <= 1024, k <= 32):
// descending, exact ties to the lower index. The logits are finished here
// from the second linear's KS partial slices part[ks][m][f * E + i] plus the
// bias (bias first, then the slices in order), and written out when `logits`
// is given. Lane l holds the values l + 32 j (VPL per lane) as order-
// preserving unsigned keys; each round takes the warp maximum key
// (redux.sync), the lowest index holding it, and the owning lane recomputes
// its head.
__device__ __forceinline__ uint32_t order_key(float x) {
  const uint32_t u = __float_as_uint(x + 0.f);  // -0 -> +0: equal values, equal keys
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <int VPL>
__global__ void __launch_bounds__(128) topk_rows_kernel(const float* __restrict__ part, int KS,
                                                        const uint16_t* __restrict__ bias, int bias_f_stride, int M,
                                                        int F, int E, int k, float* __restrict__ logits,
                                                        int32_t* __restrict__ ids) {
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + warp;
  if (row >= M * F) return;
  const int m = row / F, f = row % F;
  const int64_t slice = static_cast<int64_t>(M) * F * E;
  const float* src = part + static_cast<int64_t>(m) * F * E + static_cast<int64_t>(f) * E;
  float x[VPL];
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int i = lane + 32 * j;
    x[j] = bias && i < E ? __bfloat162float(__ushort_as_bfloat16(bias[f * bias_f_stride + i])) : 0.f;
  }
#pragma unroll
  for (int q = 0; q < kMaxPredictorKs; ++q) {
    if (q < KS) {
#pragma unroll
      for (int j = 0; j < VPL; ++j)
        if (lane + 32 * j < E) x[j] += __ldcg(src + q * slice + lane + 32 * j);
    }
  }
  uint32_t key[VPL];  // 0: no value (past E, or taken)
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int i = lane + 32 * j;
    key[j] = i < E ? order_key(x[j]) : 0u;
    if (logits && i < E) logits[static_cast<int64_t>(row) * E + i] = x[j];
  }
  uint32_t hk = 0u;
  int hj = -1;
#pragma unroll
  for (int j = 0; j < VPL; ++j)
    if (key[j] > hk) {
      hk = key[j];
      hj = j;
    }
  int my_id = -1;
  for (int r = 0; r < k; ++r) {
    const uint32_t mk = __reduce_max_sync(kFullMask, hk);
    const uint32_t cand = hj >= 0 && hk == mk ? static_cast<uint32_t>(lane + 32 * hj) : 0xFFFFFFFFu;
    const uint32_t wi = __reduce_min_sync(kFullMask, cand);
    if (lane == r) my_id = mk == 0u ? -1 : static_cast<int>(wi);
    if (hj >= 0 && static_cast<uint32_t>(lane + 32 * hj) == wi) {
#pragma unroll
      for (int j = 0; j < VPL; ++j)
        if (j == hj) key[j] = 0u;
      hk = 0u;
      hj = -1;
#pragma unroll
      for (int j = 0; j < VPL; ++j)
        if (key[j] > hk) {
          hk = key[j];
          hj = j;
        }
    }
  }
  if (lane < k) ids[static_cast<int64_t>(row) * k + lane] = my_id;
}

int launch_topk_rows(cudaLaunchConfig_t cfg, const float* part, int KS, const uint16_t* bias, int bias_f_stride,
                     int M, int F, int E, int k, float* logits, int32_t* ids) {
  const int rows = M * F, wpb = 4;
  cfg.blockDim = dim3(wpb * 32);
  cfg.gridDim = dim3((rows + wpb - 1) / wpb);
  cfg.dynamicSmemBytes = 0;
  const int vpl = (E + 31) / 32;
  cudaError_t e;
  if (vpl <= 1)
    e = cudaLaunchKernelEx(&cfg, topk_rows_kernel<1>, part, KS, bias, bias_f_stride, M, F, E, k, logits, ids);
  else if (vpl <= 2)
    e = cudaLaunchKernelEx(&cfg, topk_rows_kernel<2>, part, KS, bias, bias_f_stride, M, F, E, k, logits, ids);
  else if (vpl <= 4)
    e = cudaLaunchKernelEx(&cfg, topk_rows_kernel<4>, part, KS, bias, bias_f_stride, M, F, E, k, logits, ids);
  else if (vpl <= 8)
    e = cudaLaunchKernelEx(&cfg, topk_rows_kernel<8>, part, KS, bias, bias_f_stride, M, F, E, k, logits, ids);
  else if (vpl <= 16)
    e = cudaLaunchKernelEx(&cfg, topk_rows_kernel<16>, part, KS, bias, bias_f_stride, M, F, E, k, logits, ids);
  else
    e = cudaLaunchKernelEx(&cfg, topk_rows_kernel<32>, part, KS, bias, bias_f_stride, M, F, E, k, logits, ids);
  return e == cudaSuccess ? MTP_OK : MTP_ERR_LAUNCH;
}

size_t gemv_smem(int K) { return static_cast<size_t>(kTokChunk) * (2 * K + 16) + kPWarps * 16 * kTokChunk * 4; }

}  // namespace

int predictor_pack(const uint16_t* w, int rows, int cols, uint16_t* out, cudaStream_t st) {
  const int64_t words = static_cast<int64_t>(rows) * cols / 2;
  pack_kernel<<<static_cast<unsigned>((words + 255) / 256), 256, 0, st>>>(reinterpret_cast<const uint32_t*>(w), rows,
                                                                          cols, reinterpret_cast<uint32_t*>(out));
  return launch_status();
}

// K-splits of one linear (rows R, inner K): enough CTAs to cover the 148 SMs
// (at least ~200 CTAs), each warp keeping a multiple of 16 of K (at most 128).
int predictor_ks(int R, int K) {
  int ks = 1;
  while (ks < kMaxPredictorKs && (R / 16) * ks < 200 && (K / (2 * ks)) % (16 * kPWarps) == 0) ks *= 2;
  while (K / ks / kPWarps > kMaxKPerWarp) ks *= 2;
  return ks;
}

int predictor_run(const uint16_t* h, int M, int H, const uint16_t* w1p, const uint16_t* b1, int width,
                  const uint16_t* w2p, const uint16_t* b2, int F, int E, int k, float* logits, int32_t* ids,
                  float* part1, float* part2, cudaStream_t st) {
  static int configured_dev = -1;
  static size_t configured_smem = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MTP_ERR_CUDA;
  const size_t smem = gemv_smem(H > width ? H : width);
  if (configured_dev != dev || configured_smem < smem) {
    if (cudaFuncSetAttribute(gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return MTP_ERR_CUDA;
    configured_dev = dev;
    configured_smem = smem;
  }
  // Programmatic dependent launches: each kernel may start (and stream its
  // weights) while the previous one finishes; it waits for it before reading
  // that kernel's output.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kPThreads);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int ks1 = predictor_ks(width, H), R2 = F * E, ks2 = predictor_ks(R2, width);
  cfg.gridDim = dim3((width / 16) * ks1);
  cfg.dynamicSmemBytes = gemv_smem(H / ks1);
  if (cudaLaunchKernelEx(&cfg, gemv_kernel, h, static_cast<const float*>(nullptr), 0,
                         static_cast<const uint16_t*>(nullptr), M, H, reinterpret_cast<const uint4*>(w1p), width, ks1,
                         part1) != cudaSuccess)
    return MTP_ERR_LAUNCH;
  cfg.gridDim = dim3((R2 / 16) * ks2);
  cfg.dynamicSmemBytes = gemv_smem(width / ks2);
  if (cudaLaunchKernelEx(&cfg, gemv_kernel, static_cast<const uint16_t*>(nullptr), static_cast<const float*>(part1),
                         ks1, b1, M, width, reinterpret_cast<const uint4*>(w2p), R2, ks2, part2) != cudaSuccess)
    return MTP_ERR_LAUNCH;
  if (launch_topk_rows(cfg, part2, ks2, b2, E, M, F, E, k, logits, ids) != MTP_OK) return MTP_ERR_LAUNCH;
  return launch_status();
}

int predictor_hr_run(const uint16_t* h, const int32_t* layer_ids, int M, int H, const uint16_t* w1p,
                     const uint16_t* b1, int width, const uint16_t* ln_w, const uint16_t* ln_b, float eps,
                     const uint16_t* layer_emb, int num_layers, const uint16_t* delta_emb, int F,
                     const uint16_t* wcp, const uint16_t* bc, int E, int k, float* logits, int32_t* ids, float* part1,
                     uint16_t* ctx, float* part2, cudaStream_t st) {
  static int configured_dev = -1;
  static size_t configured_smem = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MTP_ERR_CUDA;
  const size_t smem = gemv_smem(H > width ? H : width);
  if (configured_dev != dev || configured_smem < smem) {
    if (cudaFuncSetAttribute(gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return MTP_ERR_CUDA;
    configured_dev = dev;
    configured_smem = smem;
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kPThreads);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // encoder linear (W1 [width, H]) -> fp32 partials
  const int ks1 = predictor_ks(width, H);
  cfg.gridDim = dim3((width / 16) * ks1);
  cfg.dynamicSmemBytes = gemv_smem(H / ks1);
  if (cudaLaunchKernelEx(&cfg, gemv_kernel, h, static_cast<const float*>(nullptr), 0,
                         static_cast<const uint16_t*>(nullptr), M, H, reinterpret_cast<const uint4*>(w1p), width, ks1,
                         part1) != cudaSuccess)
    return MTP_ERR_LAUNCH;
  // SiLU, LayerNorm, layer and delta embeddings, SiLU -> bf16 columns
  const int wpb = 4;
  cfg.blockDim = dim3(wpb * 32);
  cfg.gridDim = dim3((M + wpb - 1) / wpb);
  cfg.dynamicSmemBytes = 0;
  if (cudaLaunchKernelEx(&cfg, hr_context_kernel, static_cast<const float*>(part1), ks1, b1, M, width, ln_w, ln_b,
                         eps, layer_emb, num_layers, layer_ids, delta_emb, F, ctx) != cudaSuccess)
    return MTP_ERR_LAUNCH;
  // classifier (Wc [E, width]) over the M x F columns
  const int ks2 = predictor_ks(E, width);
  cfg.blockDim = dim3(kPThreads);
  cfg.gridDim = dim3((E / 16) * ks2);
  cfg.dynamicSmemBytes = gemv_smem(width / ks2);
  if (cudaLaunchKernelEx(&cfg, gemv_kernel, static_cast<const uint16_t*>(ctx), static_cast<const float*>(nullptr), 0,
                         static_cast<const uint16_t*>(nullptr), M * F, width, reinterpret_cast<const uint4*>(wcp), E,
                         ks2, part2) != cudaSuccess)
    return MTP_ERR_LAUNCH;
  if (launch_topk_rows(cfg, part2, ks2, bc, 0, M, F, E, k, logits, ids) != MTP_OK) return MTP_ERR_LAUNCH;
  return launch_status();
}

}  // namespace mtp
