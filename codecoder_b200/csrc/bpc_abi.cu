// C ABI entry points of libbpc.so that are not tied to the pre-decoder handle: version, errors, gather_mm.
#include <cstring>
#include <string>

#include "bpc.h"
#include "bpc_internal.h"

namespace bpc {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
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

extern "C" int bpc_gather_mm_fwd(const void* x, const void* w, const int32_t* idx, void* y, int64_t B, int32_t NS,
                                 int32_t NT, int32_t K, int32_t Ci, int32_t Co, int32_t dtype, bpc_stream_t stream) {
  if (B < 0 || NS < 1 || NT < 0 || K < 1 || Ci < 1 || Co < 1) return fail(BPC_ERR_ARG, "invalid gather_mm shape");
  if (dtype != BPC_DTYPE_BF16 && dtype != BPC_DTYPE_F32) return fail(BPC_ERR_ARG, "dtype must be bf16 or f32");
  if (B == 0 || NT == 0) return 0;
  if (!x || !w || !idx || !y) return fail(BPC_ERR_ARG, "null buffer");
  GmmProblem p;
  p.x = x;
  p.x_shot_stride = static_cast<int64_t>(NS) * Ci;   // x (B, NS, Ci)
  p.x_node_stride = Ci;
  p.shots = B;
  p.NS = NS;
  p.w = w;
  p.n_wtypes = 1;
  p.type_split = NT;
  p.idx = idx;
  p.NT = NT;
  p.K = K;
  p.Ci = Ci;
  p.Co = Co;
  p.y = y;
  p.y_shot_stride = static_cast<int64_t>(NT) * Co;   // y (B, NT, Co)
  p.y_node_stride = Co;
  p.epi = kEpiStore;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == BPC_DTYPE_BF16 && Ci >= 64 && Ci % 8 == 0 && Co % 32 == 0 && Co <= 256 && K <= 16) {
    if (int e = gmm_tc_check(p)) return e;
    GmmMaps maps;
    if (int e = gmm_tc_make_maps(p, &maps)) return e;
    return gmm_tc_launch(p, maps, nullptr, 2000000000ull, s);
  }
  return gmm_fma_launch(p, dtype == BPC_DTYPE_F32, s);
}
