// Memory-bound passes around the bipartite-conv op in the Cascade bottleneck block (cascade_net.py:236-259): the
// residual update of the fp32 stream fused with the next block's inference BatchNorm + SiLU, so that one pass over
// the (rows, H) stream replaces torch's chain of casts, scales, adds and activations.
//
//   v = scale_h h + scale_u u          (u bf16, optional)
//   out = v                            (fp32, optional)
//   x = SiLU(a[c] v + b[c])            (bf16, optional; a, b fp32 per channel: a folded BatchNorm)
//
// 8 channels per thread (two 16-byte fp32 vectors of h and out, one 16-byte bf16 vector of u and x), grid-stride.
#include <algorithm>
#include <string>

#include "bpc.h"
#include "bpc_common.cuh"
#include "bpc_internal.h"

namespace bpc {

namespace {

__global__ void __launch_bounds__(256) residual_affine_silu_kernel(const float* __restrict__ h,
                                                                   const __nv_bfloat16* __restrict__ u,
                                                                   float* __restrict__ out,
                                                                   __nv_bfloat16* __restrict__ x, int64_t groups,
                                                                   int H8, float scale_h, float scale_u,
                                                                   const float* __restrict__ a,
                                                                   const float* __restrict__ b) {
  for (int64_t gi = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; gi < groups;
       gi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c0 = static_cast<int>(gi % H8) * 8;
    const float4 h0 = reinterpret_cast<const float4*>(h)[2 * gi];
    const float4 h1 = reinterpret_cast<const float4*>(h)[2 * gi + 1];
    float v[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] *= scale_h;
    if (u) {
      const uint4 uu = reinterpret_cast<const uint4*>(u)[gi];
      const uint32_t* up = reinterpret_cast<const uint32_t*>(&uu);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        v[2 * e] = fmaf(scale_u, __uint_as_float(up[e] << 16), v[2 * e]);
        v[2 * e + 1] = fmaf(scale_u, __uint_as_float(up[e] & 0xFFFF0000u), v[2 * e + 1]);
      }
    }
    if (out) {
      reinterpret_cast<float4*>(out)[2 * gi] = make_float4(v[0], v[1], v[2], v[3]);
      reinterpret_cast<float4*>(out)[2 * gi + 1] = make_float4(v[4], v[5], v[6], v[7]);
    }
    if (x) {
      uint4 o;
      uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float s0 = silu_exact(fmaf(__ldg(a + c0 + 2 * e), v[2 * e], __ldg(b + c0 + 2 * e)));
        const float s1 = silu_exact(fmaf(__ldg(a + c0 + 2 * e + 1), v[2 * e + 1], __ldg(b + c0 + 2 * e + 1)));
        const __nv_bfloat162 p = __floats2bfloat162_rn(s0, s1);
        op[e] = *reinterpret_cast<const uint32_t*>(&p);
      }
      reinterpret_cast<uint4*>(x)[gi] = o;
    }
  }
}

}  // namespace

}  // namespace bpc

using namespace bpc;

extern "C" int bpc_residual_affine_silu(const float* h, const void* u, float* out, void* x, int64_t rows, int32_t H,
                                        float scale_h, float scale_u, const float* a, const float* b,
                                        bpc_stream_t stream) {
  if (rows < 0 || H < 8 || H % 8) return fail(BPC_ERR_ARG, "rows >= 0 and a channel count that is a multiple of 8");
  if (!h) return fail(BPC_ERR_ARG, "null h");
  if (x && (!a || !b)) return fail(BPC_ERR_ARG, "the SiLU output needs scale and shift");
  if ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(u) | reinterpret_cast<uintptr_t>(out) |
       reinterpret_cast<uintptr_t>(x)) & 15)
    return fail(BPC_ERR_ARG, "h, u, out and x must be 16-byte aligned");
  if (rows == 0) return 0;
  const int64_t groups = rows * (H / 8);
  const int blocks = static_cast<int>(std::min<int64_t>((groups + 255) / 256, 16 * static_cast<int64_t>(num_sms())));
  residual_affine_silu_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      h, static_cast<const __nv_bfloat16*>(u), out, static_cast<__nv_bfloat16*>(x), groups, H / 8, scale_h, scale_u,
      a, b);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("residual_affine_silu_kernel: ") + cudaGetErrorString(e));
  return 0;
}
