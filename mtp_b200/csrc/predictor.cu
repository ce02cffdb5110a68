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
// 16 output rows over all of K; its 8 warps split K, and the token columns are
// processed in chunks of 16 staged in shared memory while the weight
// fragments stay in registers. The cross-warp sums are reduced in shared
// memory in a fixed order, then the epilogue adds the bias and either applies
// SiLU and rounds to bf16 (first linear) or writes fp32 logits (second).
#include "internal.cuh"

namespace mtp {

namespace {

constexpr int kPWarps = 8;
constexpr int kPThreads = kPWarps * 32;
constexpr int kTokChunk = 16;  // token columns per staged chunk (two n8 tiles)
constexpr int kMaxKPerWarp = 256;

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

// One linear layer: out[m][row] for the CTA's 16 rows, all M columns.
// mode 0: out_bf16 = bf16(silu(acc + bias)); mode 1: out_f32 = acc + bias.
__global__ void __launch_bounds__(kPThreads) gemv_kernel(const uint16_t* __restrict__ x, int M, int K,
                                                         const uint4* __restrict__ wp, const uint16_t* __restrict__ bias,
                                                         int R, int mode, uint16_t* __restrict__ out_bf16,
                                                         float* __restrict__ out_f32) {
  extern __shared__ __align__(16) uint8_t psm[];
  const int row_stride = 2 * K + 16;  // bf16 row of a token + 16 bytes: conflict-free B fragments
  uint8_t* hs = psm;                                                            // [16][row_stride]
  float* red = reinterpret_cast<float*>(psm + kTokChunk * row_stride);          // [8 warps][16 rows][16 tok]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int strip = blockIdx.x;
  const int kpw = K / kPWarps;  // K per warp (<= 256): kpw / 16 k-steps
  const int ks0 = warp * (kpw / 16);
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
  for (int c0 = 0; c0 < M; c0 += kTokChunk) {
    // stage x rows c0..c0+15 (zero rows past M)
    const int vecs = K / 8;
    for (int i = threadIdx.x; i < kTokChunk * vecs; i += kPThreads) {
      const int n = i / vecs, v = i % vecs;
      uint4 val = make_uint4(0u, 0u, 0u, 0u);
      if (c0 + n < M) val = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(c0 + n) * K)[v];
      *reinterpret_cast<uint4*>(hs + n * row_stride + v * 16) = val;
    }
    __syncthreads();
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int i = 0; i < kMaxKPerWarp / 16; ++i) {
      if (i < kpw / 16) {
        const int k = (ks0 + i) * 16 + 2 * t;
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
      if (m < M) {
        if (bias) v += __bfloat162float(__ushort_as_bfloat16(bias[orow]));
        if (mode == 0) {
          out_bf16[static_cast<int64_t>(m) * R + orow] = __bfloat16_as_ushort(__float2bfloat16(v / (1.f + expf(-v))));
        } else {
          out_f32[static_cast<int64_t>(m) * R + orow] = v;
        }
      }
    }
    __syncthreads();
  }
}

// Top-k of each row of E logits (one warp per row; E <= 1024, k <= 32):
// descending, exact ties to the lower index.
__global__ void topk_rows_kernel(const float* __restrict__ logits, int rows, int E, int k,
                                 int32_t* __restrict__ ids) {
  extern __shared__ float tv[];  // [warps][E]
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + warp;
  if (row >= rows) return;
  float* v = tv + warp * E;
  const float* src = logits + static_cast<int64_t>(row) * E;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = lane; i < E; i += 32) {
    const float x = src[i];
    v[i] = x;
    if (x > bv) {
      bv = x;
      bi = i;
    }
  }
  __syncwarp();
  int my_id = -1;
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
    if (lane == j) my_id = wi < E ? wi : -1;
    if (wi < E && (wi & 31) == lane) {
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
  if (lane < k) ids[static_cast<int64_t>(row) * k + lane] = my_id;
}

size_t gemv_smem(int K) { return static_cast<size_t>(kTokChunk) * (2 * K + 16) + kPWarps * 16 * kTokChunk * 4; }

}  // namespace

int predictor_pack(const uint16_t* w, int rows, int cols, uint16_t* out, cudaStream_t st) {
  const int64_t words = static_cast<int64_t>(rows) * cols / 2;
  pack_kernel<<<static_cast<unsigned>((words + 255) / 256), 256, 0, st>>>(reinterpret_cast<const uint32_t*>(w), rows,
                                                                          cols, reinterpret_cast<uint32_t*>(out));
  return launch_status();
}

int predictor_run(const uint16_t* h, int M, int H, const uint16_t* w1p, const uint16_t* b1, int width,
                  const uint16_t* w2p, const uint16_t* b2, int F, int E, int k, float* logits, int32_t* ids,
                  uint16_t* hidden2, cudaStream_t st) {
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
  cfg.gridDim = dim3(width / 16);
  cfg.dynamicSmemBytes = gemv_smem(H);
  if (cudaLaunchKernelEx(&cfg, gemv_kernel, h, M, H, reinterpret_cast<const uint4*>(w1p), b1, width, 0, hidden2,
                         static_cast<float*>(nullptr)) != cudaSuccess)
    return MTP_ERR_LAUNCH;
  const int R2 = F * E;
  cfg.gridDim = dim3(R2 / 16);
  cfg.dynamicSmemBytes = gemv_smem(width);
  if (cudaLaunchKernelEx(&cfg, gemv_kernel, static_cast<const uint16_t*>(hidden2), M, width,
                         reinterpret_cast<const uint4*>(w2p), b2, R2, 1, static_cast<uint16_t*>(nullptr), logits) !=
      cudaSuccess)
    return MTP_ERR_LAUNCH;
  const int rows = M * F, wpb = 4;
  cfg.blockDim = dim3(wpb * 32);
  cfg.gridDim = dim3((rows + wpb - 1) / wpb);
  cfg.dynamicSmemBytes = static_cast<size_t>(wpb) * E * 4;
  if (cudaLaunchKernelEx(&cfg, topk_rows_kernel, static_cast<const float*>(logits), rows, E, k, ids) != cudaSuccess)
    return MTP_ERR_LAUNCH;
  return launch_status();
}

}  // namespace mtp
