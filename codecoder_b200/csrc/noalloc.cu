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
// the first call in each CUDA context (with that context's device current) looks the address up with
// cudaGetSymbolAddress and caches it for that context, so that first call should come before any stream capture.
// The address belongs to the context's own copy of the module: a host that makes its own driver context current
// gets an entry of its own, not the primary context's.  Entries are keyed by the context's unique ID, which CUDA
// never reuses within a process, so a context created after a cudaDeviceReset gets a fresh lookup instead of a stale
// address.  The handle must belong to the current
// device: its tables and weights live there, and the call is refused otherwise.  All calls share the one array and
// it keeps the last call's contents (the forward initialises everything it reads: the tile counter is cleared
// before each step, the residual bits are written from the detectors), and two calls whose work overlaps on the GPU
// -- on two streams, or from two threads -- race on it.
#include <map>
#include <mutex>
#include <string>

#include "bpc.h"
#include "bpc_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
std::map<unsigned long long, void*> g_noalloc_ptr;   // CUDA context ID -> the scratch array's address in it

using CtxGetCurrentFn = int (*)(void**);                    // cuCtxGetCurrent(CUcontext*)
using CtxGetIdFn = int (*)(void*, unsigned long long*);     // cuCtxGetId(CUcontext, unsigned long long*)

void* driver_fn(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
    return p;
  return nullptr;
}

CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = reinterpret_cast<CtxGetCurrentFn>(driver_fn("cuCtxGetCurrent"));
  return fn;
}
CtxGetIdFn ctx_get_id() {
  static CtxGetIdFn fn = reinterpret_cast<CtxGetIdFn>(driver_fn("cuCtxGetId"));
  return fn;
}

// Device address of the scratch array in the current context (looked up once per context).
int noalloc_scratch(void** out) {
  CtxGetCurrentFn get = ctx_get_current();
  CtxGetIdFn get_id = ctx_get_id();
  if (!get || !get_id) return bpc::fail(BPC_ERR_DRIVER, "cuCtxGetCurrent / cuCtxGetId not available from the driver");
  void* ctx = nullptr;
  if (get(&ctx) != 0) return bpc::fail(BPC_ERR_DRIVER, "cuCtxGetCurrent failed");
  if (!ctx) {
    // no context bound to this thread yet: bind the current device's primary context (a context the host made
    // current itself is kept as it is)
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaSetDevice(dev);
    if (e != cudaSuccess) return bpc::fail(BPC_ERR_LAUNCH, std::string("context set-up: ") + cudaGetErrorString(e));
    if (get(&ctx) != 0 || !ctx) return bpc::fail(BPC_ERR_DRIVER, "no current CUDA context");
  }
  unsigned long long id = 0;
  if (get_id(ctx, &id) != 0) return bpc::fail(BPC_ERR_DRIVER, "cuCtxGetId failed");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  auto it = g_noalloc_ptr.find(id);
  if (it == g_noalloc_ptr.end()) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return bpc::fail(BPC_ERR_LAUNCH, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    it = g_noalloc_ptr.emplace(id, p).first;
  }
  *out = it->second;
  return 0;
}

}  // namespace

extern "C" size_t bpc_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int bpc_predecoder_forward_noalloc(bpc_predecoder* h, const uint8_t* det, float* logits,
                                              uint8_t* residual, int64_t B, bpc_stream_t stream) {
  if (!h) return bpc::fail(BPC_ERR_ARG, "null pre-decoder");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return bpc::fail(BPC_ERR_LAUNCH, "cudaGetDevice failed");
  if (dev != bpc::predecoder_device(h))
    return bpc::fail(BPC_ERR_ARG, "the pre-decoder was created on device " + std::to_string(bpc::predecoder_device(h)) +
                                      " but device " + std::to_string(dev) + " is current");
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
