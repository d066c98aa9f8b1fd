// moe_noalloc.cu -- gemms_moe_fwd_noalloc: the full layer forward with its
// scratch memory in a fixed device array instead of a caller workspace.
//
// Some callers cannot allocate device memory at the point where they run the
// layer: plugin hosts whose custom-op interface hands the plugin a stream and
// tensors but no allocator, embedded runtimes that pre-plan every byte of
// device memory up front and forbid driver allocations once serving starts,
// and latency-critical loops where a cudaMalloc (and the synchronisation it
// can imply) is not acceptable.  This entry point lets them run small batches
// (decode-sized) without providing a workspace.
//
// Scratch: a file-scope device array of kNoallocScratchBytes (16 MiB).  Every
// GPU that loads this library holds that memory until the process exits.
// Device code could name the array directly; host code must not pass the
// array's name to a kernel (on the host it is only a stand-in symbol), so the
// first call on each device, with that device current, looks up its device
// address with cudaGetSymbolAddress and caches it.  That first call should
// come before any stream capture.  Nothing here calls cudaMalloc, cudaFree or
// any allocating library routine.
#include "common.cuh"

#include <mutex>

namespace {

constexpr size_t kNoallocScratchBytes = size_t(16) << 20;  // 16 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set-up on first use).
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GEMMS_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return GEMMS_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return GEMMS_ERR_CUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return GEMMS_OK;
}

}  // namespace

extern "C" int gemms_moe_fwd_noalloc(const GemmsMoeArgs* args, gemms_stream_t stream) {
  if (!args) return GEMMS_ERR_ARG;
  const size_t need = gemms_moe_workspace_size(&args->shape);
  if (need == 0) return GEMMS_ERR_SHAPE;
  if (need > kNoallocScratchBytes) return GEMMS_ERR_CAPACITY;
  void* ws = nullptr;
  int rc = scratch_address(&ws);
  if (rc) return rc;
  // gemms_moe_fwd clears, on the stream, every part of the scratch that must
  // start at zero (error word, expert counts, fp32 accumulator); the rest is
  // fully written before it is read.
  return gemms_moe_fwd(args, ws, kNoallocScratchBytes, stream);
}

// The error word of gemms_moe_fwd_noalloc lives in the same fixed array, so
// its callers have no workspace pointer to hand to gemms_moe_check; this looks
// the array up on the current device and reads (and clears) the word there.
// Synchronises the stream, like gemms_moe_check.
extern "C" int gemms_moe_check_noalloc(gemms_stream_t stream, int32_t* flags) {
  if (!flags) return GEMMS_ERR_ARG;
  void* ws = nullptr;
  int rc = scratch_address(&ws);
  if (rc) return rc;
  return gemms_moe_check(ws, stream, flags);
}
