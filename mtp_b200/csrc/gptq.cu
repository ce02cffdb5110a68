// GPTQ int4 weights: the kernel layout, the one-time repack from the GPTQ
// checkpoint form, and a reference fp32 dequantiser.
//
// GPTQ checkpoint form of one projection with N outputs and K inputs
// (repack/gptq_unpack.py:54-131): qweight [K/8, N] int32 with nibble i of word
// j = row k = 8j+i; qzeros [K/G, N/8] int32 with nibble i of word j = column
// 8j+i; scales [K/G, N] fp16.
//
// Kernel layout (this build's own; one expert = one contiguous blob so that a
// slot fill is a single copy). Each projection is cut into row blocks of 128
// output rows, the M of one tensor-core MMA: for w13 (N = 2I) block b holds
// gate rows 64b..64b+63 then up rows I+64b..I+64b+63, so one block yields
// silu(gate) * up for 64 columns of h; for w2 block b holds rows 128b..+127.
//   weights  [N/128 blocks][K/32 chunks][128 rows][16 bytes]: the 16 bytes of
//            (block, chunk, row) hold k = 32c..32c+31 of that row as four
//            32-bit words; word j covers k0 = 32c + 8j and holds, in byte
//            t = 0..3, low nibble q(k0 + t) and high nibble q(k0 + 4 + t), so
//            `w & 0x0F0F0F0F` and `(w >> 4) & 0x0F0F0F0F` are the u8 values
//            of k0..k0+3 and k0+4..k0+7 in order (one tensor-memory column
//            each). A K range of a block is one contiguous byte range.
//   scales   [N/128][K/G][128] fp16.
//   zeros    [N/128][K/G][64] bytes: byte i = zero(row 2i) | zero(row 2i+1) << 4.
// Byte sizes equal the GPTQ ones (N*K/2, 2*N*K/G, N*K/(2G)).
#include "internal.cuh"

namespace mtp {

struct ProjLayout {
  int64_t qw, sc, zp;  // section sizes in bytes
};

__host__ __device__ inline ProjLayout proj_sizes(int64_t N, int64_t K, int64_t G) {
  ProjLayout p;
  p.qw = N * K / 2;
  p.sc = N * (K / G) * 2;
  p.zp = N * (K / G) / 2;
  return p;
}

int expert_layout(int hidden, int inter, int G, MtpExpertLayout* out) {
  const ProjLayout a = proj_sizes(2LL * inter, hidden, G);
  const ProjLayout b = proj_sizes(hidden, inter, G);
  int64_t o = 0;
  out->w13_qweight = o; o = round_up(o + a.qw, 256);
  out->w13_scales = o;  o = round_up(o + a.sc, 256);
  out->w13_zeros = o;   o = round_up(o + a.zp, 256);
  out->w2_qweight = o;  o = round_up(o + b.qw, 256);
  out->w2_scales = o;   o = round_up(o + b.sc, 256);
  out->w2_zeros = o;    o = round_up(o + b.zp, 256);
  out->bytes = o;
  return MTP_OK;
}

__device__ __forceinline__ uint32_t gptq_nib_rows(const int32_t* q, int N, int k, int n) {
  return (static_cast<uint32_t>(q[static_cast<int64_t>(k >> 3) * N + n]) >> ((k & 7) * 4)) & 0xFu;
}

// Source row (output channel) of row r of block b.
__device__ __forceinline__ int block_row(int N, int gated, int b, int r) {
  if (gated) return r < 64 ? 64 * b + r : N / 2 + 64 * b + (r - 64);
  return 128 * b + r;
}

__global__ void repack_qweight_kernel(const int32_t* __restrict__ gq, int N, int K, int gated, int E,
                                      uint8_t* __restrict__ blobs, int64_t stride, int64_t off) {
  const int64_t words = static_cast<int64_t>(N) * K / 8;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= words * E) return;
  const int e = static_cast<int>(gid / words);
  const int64_t w = gid % words;
  const int j = static_cast<int>(w & 3);
  const int r = static_cast<int>((w >> 2) & 127);
  const int64_t bc = w >> 9;
  const int chunks = K / 32;
  const int c = static_cast<int>(bc % chunks);
  const int b = static_cast<int>(bc / chunks);
  const int row = block_row(N, gated, b, r);
  const int k0 = 32 * c + 8 * j;
  const int32_t* q = gq + static_cast<int64_t>(e) * (K / 8) * N;
  uint32_t word = 0;
#pragma unroll
  for (int t = 0; t < 4; ++t)
    word |= (gptq_nib_rows(q, N, k0 + t, row) | gptq_nib_rows(q, N, k0 + 4 + t, row) << 4) << (8 * t);
  reinterpret_cast<uint32_t*>(blobs + e * stride + off)[w] = word;
}

__global__ void repack_scales_kernel(const uint16_t* __restrict__ gs, int N, int K, int G, int gated, int E,
                                     uint8_t* __restrict__ blobs, int64_t stride, int64_t off) {
  const int groups = K / G;
  const int64_t per = static_cast<int64_t>(N) * groups;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= per * E) return;
  const int e = static_cast<int>(gid / per);
  const int64_t i = gid % per;
  const int r = static_cast<int>(i & 127);
  const int64_t bg = i >> 7;
  const int grp = static_cast<int>(bg % groups);
  const int b = static_cast<int>(bg / groups);
  const int n = block_row(N, gated, b, r);
  reinterpret_cast<uint16_t*>(blobs + e * stride + off)[i] =
      gs[static_cast<int64_t>(e) * groups * N + static_cast<int64_t>(grp) * N + n];
}

__device__ __forceinline__ uint32_t gptq_nib_cols(const int32_t* z, int N, int grp, int n) {
  return (static_cast<uint32_t>(z[static_cast<int64_t>(grp) * (N / 8) + (n >> 3)]) >> ((n & 7) * 4)) &
         0xFu;
}

__global__ void repack_zeros_kernel(const int32_t* __restrict__ gz, int N, int K, int G, int gated, int E,
                                    uint8_t* __restrict__ blobs, int64_t stride, int64_t off) {
  const int groups = K / G;
  const int64_t per = static_cast<int64_t>(N) * groups / 2;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= per * E) return;
  const int e = static_cast<int>(gid / per);
  const int64_t i = gid % per;
  const int rp = static_cast<int>(i & 63);
  const int64_t bg = i >> 6;
  const int grp = static_cast<int>(bg % groups);
  const int b = static_cast<int>(bg / groups);
  const int32_t* z = gz + static_cast<int64_t>(e) * groups * (N / 8);
  const uint32_t v = gptq_nib_cols(z, N, grp, block_row(N, gated, b, 2 * rp)) |
                     gptq_nib_cols(z, N, grp, block_row(N, gated, b, 2 * rp + 1)) << 4;
  (blobs + e * stride + off)[i] = static_cast<uint8_t>(v);
}

static int repack_proj(const int32_t* q, const int32_t* z, const uint16_t* s, int N, int K, int G,
                       int gated, int E, uint8_t* blobs, int64_t stride, int64_t off_q, int64_t off_s,
                       int64_t off_z, cudaStream_t st) {
  const int T = 256;
  const int64_t nq = static_cast<int64_t>(N) * K / 8 * E;
  const int64_t ns = static_cast<int64_t>(N) * (K / G) * E;
  const int64_t nz = ns / 2;
  repack_qweight_kernel<<<static_cast<unsigned>((nq + T - 1) / T), T, 0, st>>>(q, N, K, gated, E, blobs, stride,
                                                                                off_q);
  repack_scales_kernel<<<static_cast<unsigned>((ns + T - 1) / T), T, 0, st>>>(s, N, K, G, gated, E, blobs, stride,
                                                                               off_s);
  repack_zeros_kernel<<<static_cast<unsigned>((nz + T - 1) / T), T, 0, st>>>(z, N, K, G, gated, E, blobs, stride,
                                                                              off_z);
  return launch_status();
}

int repack_gptq(const int32_t* w13q, const int32_t* w13z, const uint16_t* w13s, const int32_t* w2q,
                const int32_t* w2z, const uint16_t* w2s, int E, int H, int I, int G, uint8_t* out,
                cudaStream_t st) {
  MtpExpertLayout L;
  expert_layout(H, I, G, &L);
  int r = repack_proj(w13q, w13z, w13s, 2 * I, H, G, 1, E, out, L.bytes, L.w13_qweight, L.w13_scales,
                      L.w13_zeros, st);
  if (r != MTP_OK) return r;
  return repack_proj(w2q, w2z, w2s, H, I, G, 0, E, out, L.bytes, L.w2_qweight, L.w2_scales, L.w2_zeros, st);
}

__global__ void gptq_dequant_kernel(const int32_t* __restrict__ q, const int32_t* __restrict__ z,
                                    const uint16_t* __restrict__ s, const int32_t* __restrict__ gidx,
                                    int K, int N, int G, int zero_mode, float* __restrict__ out) {
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= static_cast<int64_t>(N) * K) return;
  const int n = static_cast<int>(gid / K);
  const int k = static_cast<int>(gid % K);
  const int grp = gidx ? gidx[k] : k / G;
  const uint32_t qv = gptq_nib_rows(q, N, k, n);
  const float zv = zero_mode == MTP_ZERO_SYM8 ? 8.0f : static_cast<float>(gptq_nib_cols(z, N, grp, n));
  const float sv = __half2float(__ushort_as_half(s[static_cast<int64_t>(grp) * N + n]));
  out[gid] = (static_cast<float>(qv) - zv) * sv;
}

int gptq_dequant(const int32_t* q, const int32_t* z, const uint16_t* s, const int32_t* gidx, int K,
                 int N, int G, int zero_mode, float* out, cudaStream_t st) {
  const int T = 256;
  const int64_t n = static_cast<int64_t>(N) * K;
  gptq_dequant_kernel<<<static_cast<unsigned>((n + T - 1) / T), T, 0, st>>>(q, z, s, gidx, K, N, G,
                                                                         zero_mode, out);
  return launch_status();
}

}  // namespace mtp
