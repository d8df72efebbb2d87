// C ABI entry points of libbpc.so that are not tied to the pre-decoder handle: version, errors, the gather_mm op
// (forward, input gradient, weight gradient) and its watchdog status word.
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "bpc.h"
#include "bpc_internal.h"

namespace bpc {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

// Watchdog status word of the op entry points: static device memory (no allocation), one per device.
__device__ int g_op_status = 0;

int* op_status_ptr() {
  static std::mutex mu;
  static std::vector<int*> ptrs;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (static_cast<int>(ptrs.size()) <= dev) ptrs.resize(dev + 1, nullptr);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_op_status) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

}  // namespace bpc

using namespace bpc;

extern "C" int bpc_version(void) { return (0 << 16) | 1; }

extern "C" int bpc_last_error(char* buf, int len) {
  const int n = static_cast<int>(g_last_error.size());
  if (buf && len > 0) {
    const int m = n < len - 1 ? n : len - 1;
    std::memcpy(buf, g_last_error.data(), m);
    buf[m] = 0;
  }
  return n;
}

namespace {

int run_gather_mm(const void* x, const void* w, const int32_t* idx, void* y, int64_t B, int32_t NS, int32_t NT,
                  int32_t K, int32_t Ci, int32_t Co, int32_t n_wtypes, int32_t type_split, int epi,
                  const float* scale, const float* shift, int32_t dtype, bpc_stream_t stream) {
  if (B < 0 || NS < 1 || NT < 0 || K < 1 || Ci < 1 || Co < 1) return fail(BPC_ERR_ARG, "invalid gather_mm shape");
  if (dtype != BPC_DTYPE_BF16 && dtype != BPC_DTYPE_F32) return fail(BPC_ERR_ARG, "dtype must be bf16 or f32");
  if (n_wtypes < 1 || n_wtypes > 2 || type_split < 0 || type_split > NT)
    return fail(BPC_ERR_ARG, "one or two weight sets, split inside [0, NT]");
  if (B == 0 || NT == 0) return 0;
  if (!x || !w || !idx || !y) return fail(BPC_ERR_ARG, "null buffer");
  GmmProblem p;
  p.x = x;
  p.x_shot_stride = static_cast<int64_t>(NS) * Ci;   // x (B, NS, Ci)
  p.x_node_stride = Ci;
  p.shots = B;
  p.NS = NS;
  p.w = w;
  p.n_wtypes = n_wtypes;
  p.type_split = n_wtypes > 1 ? type_split : NT;
  p.idx = idx;
  p.NT = NT;
  p.K = K;
  p.Ci = Ci;
  p.Co = Co;
  p.y = y;
  p.y_shot_stride = static_cast<int64_t>(NT) * Co;   // y (B, NT, Co)
  p.y_node_stride = Co;
  p.epi = epi;
  p.epi_scale = scale;
  p.epi_shift = shift;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == BPC_DTYPE_BF16 && Ci >= 64 && Ci % 8 == 0 && Co % 32 == 0 && Co <= 256 && K <= 16) {
    if (int e = gmm_tc_check(p)) return e;
    GmmMaps maps;
    if (int e = gmm_tc_make_maps(p, &maps)) return e;
    return gmm_tc_launch(p, maps, op_status_ptr(), 2000000000ull, s);
  }
  return gmm_fma_launch(p, dtype == BPC_DTYPE_F32, s);
}

}  // namespace

extern "C" int bpc_gather_mm_fwd(const void* x, const void* w, const int32_t* idx, void* y, int64_t B, int32_t NS,
                                 int32_t NT, int32_t K, int32_t Ci, int32_t Co, int32_t dtype, bpc_stream_t stream) {
  return run_gather_mm(x, w, idx, y, B, NS, NT, K, Ci, Co, 1, NT, kEpiStore, nullptr, nullptr, dtype, stream);
}

extern "C" int bpc_gather_mm_fwd_ex(const void* x, const void* w, const int32_t* idx, void* y, int64_t B, int32_t NS,
                                    int32_t NT, int32_t K, int32_t Ci, int32_t Co, int32_t n_wtypes,
                                    int32_t type_split, int32_t epilogue, const float* scale, const float* shift,
                                    int32_t dtype, bpc_stream_t stream) {
  int epi;
  if (epilogue == BPC_EPILOGUE_STORE) {
    epi = kEpiStore;
  } else if (epilogue == BPC_EPILOGUE_AFFINE_SILU) {
    epi = kEpiAffineSilu;
    if (!scale || !shift) return fail(BPC_ERR_ARG, "the affine + SiLU epilogue needs scale and shift");
  } else if (epilogue == BPC_EPILOGUE_ADD) {
    epi = kEpiAdd;
  } else {
    return fail(BPC_ERR_ARG, "unknown epilogue");
  }
  return run_gather_mm(x, w, idx, y, B, NS, NT, K, Ci, Co, n_wtypes, type_split, epi, scale, shift, dtype, stream);
}

extern "C" int bpc_gather_mm_fwd_gelu(const void* x, const void* w, const int32_t* idx, void* a, int64_t B,
                                     int32_t NS, int32_t NT, int32_t K, int32_t Ci, int32_t Co, const void* h,
                                     int32_t h_dtype, void* out, void* out_bf16, int64_t stream_shot_stride,
                                     bpc_stream_t stream) {
  if (B < 0 || NS < 1 || NT < 0 || K < 1 || Ci < 1 || Co < 1) return fail(BPC_ERR_ARG, "invalid gather_mm shape");
  if (h && h_dtype != BPC_DTYPE_F32 && h_dtype != BPC_DTYPE_BF16) return fail(BPC_ERR_ARG, "h must be f32 or bf16");
  if (stream_shot_stride < static_cast<int64_t>(NT) * Co) return fail(BPC_ERR_ARG, "stream rows overlap");
  if (B == 0 || NT == 0) return 0;
  if (!x || !w || !idx || !a || !out || (h && h_dtype == BPC_DTYPE_F32 && !out_bf16))
    return fail(BPC_ERR_ARG, "null buffer");
  GmmProblem p;
  p.x = x;
  p.x_shot_stride = static_cast<int64_t>(NS) * Ci;
  p.x_node_stride = Ci;
  p.shots = B;
  p.NS = NS;
  p.w = w;
  p.type_split = NT;
  p.idx = idx;
  p.NT = NT;
  p.K = K;
  p.Ci = Ci;
  p.Co = Co;
  p.y = a;
  p.y_shot_stride = static_cast<int64_t>(NT) * Co;
  p.y_node_stride = Co;
  p.epi = kEpiGeluStream;
  p.res_h = h;
  p.res_f32 = h && h_dtype == BPC_DTYPE_F32;
  p.res_out = out;
  p.res_out16 = out_bf16;
  p.res_shot_stride = stream_shot_stride;
  p.res_node_stride = Co;
  if (int e = gmm_tc_check(p)) return e;
  GmmMaps maps;
  if (int e = gmm_tc_make_maps(p, &maps)) return e;
  return gmm_tc_launch(p, maps, op_status_ptr(), 2000000000ull, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int bpc_gather_mm_dgrad(const void* gy, const void* w, const int32_t* tgt, void* gx, void* w_t, int64_t B,
                                   int32_t NT, int32_t NS, int32_t K, int32_t Ci, int32_t Co, int32_t dtype,
                                   bpc_stream_t stream) {
  if (B < 0 || NS < 0 || NT < 1 || K < 1 || Ci < 1 || Co < 1) return fail(BPC_ERR_ARG, "invalid gather_mm shape");
  if (dtype != BPC_DTYPE_BF16 && dtype != BPC_DTYPE_F32) return fail(BPC_ERR_ARG, "dtype must be bf16 or f32");
  if (B == 0 || NS == 0) return 0;
  if (!gy || !w || !tgt || !gx || !w_t) return fail(BPC_ERR_ARG, "null buffer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (int e = transpose_w_launch(w, w_t, K, Ci, Co, dtype, s)) return e;
  // gx = the forward over gy (B, NT, Co) with the target table and W' (Ci, K Co)
  return bpc_gather_mm_fwd(gy, w_t, tgt, gx, B, NT, NS, K, Co, Ci, dtype, stream);
}

extern "C" int bpc_gather_mm_dgrad_ex(const void* gy, const void* w, const int32_t* tgt, void* gx, void* w_t,
                                      int64_t B, int32_t NT, int32_t NS, int32_t K, int32_t Ci, int32_t Co,
                                      int32_t accumulate, int32_t dtype, bpc_stream_t stream) {
  if (B < 0 || NS < 0 || NT < 1 || K < 1 || Ci < 1 || Co < 1) return fail(BPC_ERR_ARG, "invalid gather_mm shape");
  if (dtype != BPC_DTYPE_BF16 && dtype != BPC_DTYPE_F32) return fail(BPC_ERR_ARG, "dtype must be bf16 or f32");
  if (B == 0 || NS == 0) return 0;
  if (!gy || !w || !tgt || !gx || !w_t) return fail(BPC_ERR_ARG, "null buffer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (int e = transpose_w_launch(w, w_t, K, Ci, Co, dtype, s)) return e;
  return run_gather_mm(gy, w_t, tgt, gx, B, NT, NS, K, Co, Ci, 1, NS, accumulate ? kEpiAdd : kEpiStore, nullptr,
                       nullptr, dtype, stream);
}

extern "C" int bpc_gather_mm_wgrad(const void* x, const void* gy, const int32_t* idx, float* dw, void* workspace,
                                   size_t workspace_bytes, int64_t B, int32_t NS, int32_t NT, int32_t K, int32_t Ci,
                                   int32_t Co, int32_t dtype, bpc_stream_t stream) {
  if (B < 0 || NS < 1 || NT < 0 || K < 1 || Ci < 1 || Co < 1) return fail(BPC_ERR_ARG, "invalid gather_mm shape");
  if (dtype != BPC_DTYPE_BF16 && dtype != BPC_DTYPE_F32) return fail(BPC_ERR_ARG, "dtype must be bf16 or f32");
  if (!dw) return fail(BPC_ERR_ARG, "null buffer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (B == 0 || NT == 0) {
    cudaError_t e = cudaMemsetAsync(dw, 0, sizeof(float) * Co * K * Ci, s);
    return e == cudaSuccess ? 0 : fail(BPC_ERR_LAUNCH, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  }
  if (!x || !gy || !idx) return fail(BPC_ERR_ARG, "null buffer");
  return gmm_wgrad_launch(x, gy, idx, dw, workspace, workspace_bytes, B, NS, NT, K, Ci, Co, dtype, op_status_ptr(), s);
}

extern "C" size_t bpc_gather_mm_wgrad_workspace_size(int64_t B, int32_t NS, int32_t NT, int32_t K, int32_t Ci,
                                                     int32_t Co, int32_t dtype) {
  (void)NS;
  if (B <= 0 || NT <= 0 || K < 1 || Ci < 1 || Co < 1) return 0;
  return gmm_wgrad_workspace(B, NT, K, Ci, Co, dtype);
}

extern "C" int bpc_gather_mm_status(bpc_stream_t stream, int* status) {
  if (!status) return fail(BPC_ERR_ARG, "null argument");
  int* p = op_status_ptr();
  if (!p) return fail(BPC_ERR_LAUNCH, "cudaGetSymbolAddress(op status) failed");
  int v = 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(&v, p, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("status read: ") + cudaGetErrorString(e));
  *status = v;
  if (v != 0) {
    const int zero = 0;
    cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice);
    return fail(BPC_ERR_DEVICE, "a gather_mm kernel watchdog fired (status " + std::to_string(v) + ")");
  }
  return 0;
}
