// Pre-decoder forward for callers that cannot allocate device memory.
//
// Some hosts of this library own the device heap themselves: an inference server whose memory pool has carved up
// the GPU before the decoder loads, a real-time control loop that must not call into the CUDA allocator while it
// runs (cudaMalloc can synchronise the device and take unbounded time), or a plugin that is handed only raw input
// and output pointers.  bpc_predecoder_forward needs a workspace from its caller; this entry point instead runs the
// same forward pass on a fixed scratch array that lives in the library's device image, so the caller passes only
// its inputs and outputs.
//
// The scratch array is a file-scope __device__ array of kNoAllocScratchBytes (64 MiB): every GPU on which this
// module is loaded holds it until the process exits.  Host code cannot use the array's name as a device address;
// the first call on each device (with that device current) looks the address up with cudaGetSymbolAddress and
// caches it, so that first call should come before any stream capture.  All calls share the one array and it keeps
// the last call's contents (the forward initialises everything it reads: the tile counter is cleared before each
// step, the residual bits are written from the detectors), and two calls whose work overlaps on the GPU -- on two
// streams, or from two threads -- race on it.
#include <mutex>
#include <string>

#include "bpc.h"
#include "bpc_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once per device).
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return bpc::fail(BPC_ERR_LAUNCH, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return bpc::fail(BPC_ERR_ARG, "device ordinal out of range for the scratch table");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return bpc::fail(BPC_ERR_LAUNCH, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}

}  // namespace

extern "C" size_t bpc_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int bpc_predecoder_forward_noalloc(bpc_predecoder* h, const uint8_t* det, float* logits,
                                              uint8_t* residual, int64_t B, bpc_stream_t stream) {
  if (!h) return bpc::fail(BPC_ERR_ARG, "null pre-decoder");
  const size_t need = bpc_predecoder_workspace_size(h, 256);
  if (need == 0 || need > kNoAllocScratchBytes)
    return bpc::fail(BPC_ERR_SPACE, "this network needs " + std::to_string(need) +
                                        " bytes of scratch for one 256-shot pass; the built-in scratch holds " +
                                        std::to_string(kNoAllocScratchBytes) +
                                        " bytes (use bpc_predecoder_forward with a caller workspace)");
  void* ws = nullptr;
  if (int e = noalloc_scratch(&ws)) return e;
  return bpc_predecoder_forward(h, det, logits, residual, B, ws, kNoAllocScratchBytes, stream);
}
