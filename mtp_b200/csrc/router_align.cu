// Standalone router and moe_align_block_size kernels (the C-ABI entry points
// mtp_router_topk and mtp_moe_align); the algorithms are in route.cuh.
#include "internal.cuh"
#include "route.cuh"

namespace mtp {

template <int VPT>
__global__ void __launch_bounds__(256) router_topk_kernel(
    const float* __restrict__ logits, int M, int E, int k, int renorm,
    float* __restrict__ topk_w, int32_t* __restrict__ topk_ids,
    int32_t* __restrict__ tei) {
  const int lane = threadIdx.x & 31;
  const int token = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (token >= M) return;
  float w;
  int id;
  router_token<VPT>(logits + static_cast<int64_t>(token) * E, E, k, renorm, &w, &id);
  if (lane < k) {
    const int64_t o = static_cast<int64_t>(token) * k + lane;
    topk_w[o] = w;
    topk_ids[o] = id;
    if (tei) tei[o] = lane;
  }
}

int launch_router_topk(const float* logits, int M, int E, int k, int renorm,
                       float* w, int32_t* ids, int32_t* tei, cudaStream_t st) {
  const int threads = 256;
  const int blocks = (M * 32 + threads - 1) / threads;
  const int vpt = (E + 31) / 32;
  if (vpt <= 1)
    router_topk_kernel<1><<<blocks, threads, 0, st>>>(logits, M, E, k, renorm, w, ids, tei);
  else if (vpt <= 2)
    router_topk_kernel<2><<<blocks, threads, 0, st>>>(logits, M, E, k, renorm, w, ids, tei);
  else if (vpt <= 4)
    router_topk_kernel<4><<<blocks, threads, 0, st>>>(logits, M, E, k, renorm, w, ids, tei);
  else if (vpt <= 8)
    router_topk_kernel<8><<<blocks, threads, 0, st>>>(logits, M, E, k, renorm, w, ids, tei);
  else if (vpt <= 16)
    router_topk_kernel<16><<<blocks, threads, 0, st>>>(logits, M, E, k, renorm, w, ids, tei);
  else
    router_topk_kernel<32><<<blocks, threads, 0, st>>>(logits, M, E, k, renorm, w, ids, tei);
  return launch_status();
}

// ---------------------------------------------------------------------------
// moe_align_block_size
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kAlignThreads) moe_align_kernel(
    const int32_t* __restrict__ ids, int numel, int E, int BM,
    const int32_t* __restrict__ emap, int ignore_invalid, int cap, int max_blocks,
    int max_seg, int32_t* __restrict__ sorted, int32_t* __restrict__ eids,
    int32_t* __restrict__ ntpp, int32_t* __restrict__ segs, int32_t* __restrict__ nseg) {
  extern __shared__ int sm[];
  __shared__ int scan_tmp[32];
  align_block(ids, numel, E, BM, emap, ignore_invalid, cap, max_blocks, max_seg, sorted, eids, ntpp,
              segs, nseg, sm, scan_tmp);
}

int launch_moe_align(const int32_t* ids, int numel, int E, int BM, const int32_t* emap,
                     int ignore_invalid, int cap, int max_blocks, int max_seg,
                     int32_t* sorted, int32_t* eids, int32_t* ntpp, int32_t* segs,
                     int32_t* nseg, cudaStream_t st) {
  const size_t smem = align_smem_bytes(E);
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    if (cudaFuncSetAttribute(moe_align_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(align_smem_bytes(1024))) != cudaSuccess)
      return MTP_ERR_CUDA;
    configured_device = dev;
  }
  moe_align_kernel<<<1, kAlignThreads, smem, st>>>(ids, numel, E, BM, emap, ignore_invalid,
                                                   cap, max_blocks, max_seg, sorted, eids,
                                                   ntpp, segs, nseg);
  return launch_status();
}

}  // namespace mtp
