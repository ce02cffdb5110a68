// mtp_w4a16_moe_layer_noalloc: the MoE layer forward for callers that cannot
// allocate device memory.
//
// Who needs it: a host that only hands the library pointers to buffers it was
// given (an FFI caller with no handle on a CUDA allocator), and serving loops
// that run under a no-allocation rule because another allocator owns the
// device memory, where a cudaMalloc could fail, fragment that pool or
// synchronise the device in the middle of a decode step. Such callers cannot
// provide the layer's workspace, so this entry point uses a fixed scratch
// array compiled into the library instead.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes
// (6 MiB, enough for M <= 48 tokens at H = 2048, I = 512, E = 256, top-8);
// every GPU that loads the library holds it until the process exits. Larger
// requests are rejected with MTP_ERR_WORKSPACE before anything is launched.
//
// The array's name is only a host-side stand-in in host code, so its device
// address is looked up with cudaGetSymbolAddress, once per device, with that
// device current, on the first call made on that device; that first call
// should therefore come before any stream capture. The address is kept for
// the life of the process, keyed by device index: after cudaDeviceReset (or
// any teardown of the device's primary context) it is stale, so a process
// that resets a device must not call this entry point on it again. All calls
// share the one
// array and it keeps the last call's contents: the counters that must start
// at zero are zero when the library loads (a __device__ array starts zeroed)
// and every completed call leaves them zero again; everything else is written
// before it is read. Calls that overlap on the GPU (other streams,
// other host threads) race on the array and must be serialised by the caller.
//
// Nothing here allocates: no cudaMalloc, no cudaFree, no allocating library
// call; the work itself is mtp_w4a16_moe_layer with the workspace replaced.
#include "internal.cuh"

#include <mutex>

namespace {

constexpr size_t kNoAllocScratchBytes = MTP_NOALLOC_SCRATCH_BYTES;

static __device__ __align__(256) unsigned char g_layer_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once).
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return MTP_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_layer_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return MTP_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return MTP_OK;
}

}  // namespace

extern "C" int mtp_w4a16_moe_layer_noalloc(const MtpMoeLayerArgs* args, void* stream) {
  if (!args) return MTP_ERR_NULL;
  int64_t need = 0;
  const int r = mtp_w4a16_moe_layer_workspace_size(args->num_tokens, args->num_experts, args->top_k,
                                                   args->hidden, args->inter, &need);
  if (r != MTP_OK) return r;
  if (need > static_cast<int64_t>(kNoAllocScratchBytes)) return MTP_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int s = scratch_for_current_device(&scratch);
  if (s != MTP_OK) return s;
  MtpMoeLayerArgs a = *args;
  a.workspace = scratch;
  a.workspace_bytes = static_cast<int64_t>(kNoAllocScratchBytes);
  return mtp_w4a16_moe_layer(&a, stream);
}
