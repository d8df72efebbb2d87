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
      // SiLU on the hardware tanh (its result is rounded to bf16 right after), as the block-boundary kernel does
      uint4 o;
      uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint64_t av = f2_pack(__ldg(a + c0 + 2 * e), __ldg(a + c0 + 2 * e + 1));
        const uint64_t bv = f2_pack(__ldg(b + c0 + 2 * e), __ldg(b + c0 + 2 * e + 1));
        op[e] = f2_to_bf2(silu_tanh_fast2(f2_fma(av, f2_pack(v[2 * e], v[2 * e + 1]), bv)));
      }
      reinterpret_cast<uint4*>(x)[gi] = o;
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// The training network's residual steps around the op (one pass each, 8 channels per thread):
//   forward   u = GELU(a) (rounded to bf16, as torch's gelu on bf16 does),  y = h + u
//             h bf16 -> y bf16 (bf16 add, rounded);  h fp32 -> y fp32 and its bf16 copy (the next op's input);
//             no h -> y = u
//   backward  g = gy (+ gy16 for the fp32 stream: the gradient of the bf16 copy);  gh = g;
//             ga = GELU'(a) * g   (g rounded to bf16 first on the fp32 stream, as autograd casts it for the add)
// a and ga hold the pre-activations type-major: (T, B, NT / T, C), so that each target type's op output and input
// gradient is one contiguous (B, NT / T, C) block; h, y, gy, gh are (B, NT, C).
// GELU in the tanh form g(x) = x (1 + tanh(k (x + c x^3))) / 2, k = sqrt(2 / pi), c = 0.044715, with
// g'(x) = (1 + t) / 2 + x (1 - t^2) k (1 + 3 c x^2) / 2, t = tanh(k (x + c x^3)), t from the hardware tanh.approx
// (relative error about 2^-11, below the bf16 rounding both results get; accurate tanhf made these passes
// instruction-bound rather than HBM-bound).
constexpr float kGeluK = 0.7978845608028654f;
constexpr float kGeluC = 0.044715f;

__device__ __forceinline__ float gelu_acc(float x) { return gelu_tanh_pass(x); }
__device__ __forceinline__ float gelu_grad(float x) {
  const float t = tanh_approx(kGeluK * fmaf(kGeluC * x, x * x, x));
  return 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * kGeluK * fmaf(3.0f * kGeluC, x * x, 1.0f);
}
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t bf_pack(float lo, float hi) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&p);
}
__device__ __forceinline__ float bf_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

struct StepShape {
  int64_t units;     // B * NT * C / 8
  int64_t B;
  int32_t NT, NTt, C8;
  bool one_type;     // T = 1: the pre-activation layout is the row layout
  bool small;        // units < 2^32: the index arithmetic fits 32-bit divisions
};

// offset (elements) of pre-activation unit u in the type-major (T, B, NT / T, C) layout
__device__ __forceinline__ int64_t pre_off(const StepShape& sh, int64_t u) {
  if (sh.one_type) return 8 * u;
  if (sh.small) {
    const uint32_t uu = static_cast<uint32_t>(u);
    const uint32_t row = uu / static_cast<uint32_t>(sh.C8);
    const uint32_t c8 = uu - row * static_cast<uint32_t>(sh.C8);
    const uint32_t b = row / static_cast<uint32_t>(sh.NT);
    const uint32_t n = row - b * static_cast<uint32_t>(sh.NT);
    const uint32_t t = n / static_cast<uint32_t>(sh.NTt);
    return ((static_cast<int64_t>(t) * sh.B + b) * sh.NTt + (n - t * sh.NTt)) * (8 * static_cast<int64_t>(sh.C8)) +
           8 * c8;
  }
  const int64_t row = u / sh.C8;
  const int c8 = static_cast<int>(u - row * sh.C8);
  const int64_t b = row / sh.NT;
  const int n = static_cast<int>(row - b * sh.NT);
  const int t = n / sh.NTt;
  return ((t * sh.B + b) * sh.NTt + (n - t * sh.NTt)) * (8 * static_cast<int64_t>(sh.C8)) + 8 * c8;
}

// HMODE: 0 no h, 1 h bf16, 2 h fp32 (+ bf16 copy)
template <int HMODE>
__global__ void __launch_bounds__(256) gelu_residual_fwd_kernel(const __nv_bfloat16* __restrict__ a,
                                                                const void* __restrict__ h, void* __restrict__ y,
                                                                __nv_bfloat16* __restrict__ y16, StepShape sh) {
  for (int64_t u = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; u < sh.units;
       u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint4 av = *reinterpret_cast<const uint4*>(a + pre_off(sh, u));
    const uint32_t* aw = reinterpret_cast<const uint32_t*>(&av);
    float g[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      g[2 * e] = bf_round(gelu_acc(bf_lo(aw[e])));
      g[2 * e + 1] = bf_round(gelu_acc(bf_hi(aw[e])));
    }
    if (HMODE == 2) {
      const float4 h0 = reinterpret_cast<const float4*>(h)[2 * u];
      const float4 h1 = reinterpret_cast<const float4*>(h)[2 * u + 1];
      const float v[8] = {h0.x + g[0], h0.y + g[1], h0.z + g[2], h0.w + g[3],
                          h1.x + g[4], h1.y + g[5], h1.z + g[6], h1.w + g[7]};
      reinterpret_cast<float4*>(y)[2 * u] = make_float4(v[0], v[1], v[2], v[3]);
      reinterpret_cast<float4*>(y)[2 * u + 1] = make_float4(v[4], v[5], v[6], v[7]);
      uint4 o;
      o.x = bf_pack(v[0], v[1]);
      o.y = bf_pack(v[2], v[3]);
      o.z = bf_pack(v[4], v[5]);
      o.w = bf_pack(v[6], v[7]);
      reinterpret_cast<uint4*>(y16)[u] = o;
    } else {
      if (HMODE == 1) {
        const uint4 hv = reinterpret_cast<const uint4*>(h)[u];
        const uint32_t* hw = reinterpret_cast<const uint32_t*>(&hv);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          g[2 * e] += bf_lo(hw[e]);
          g[2 * e + 1] += bf_hi(hw[e]);
        }
      }
      uint4 o;
      o.x = bf_pack(g[0], g[1]);
      o.y = bf_pack(g[2], g[3]);
      o.z = bf_pack(g[4], g[5]);
      o.w = bf_pack(g[6], g[7]);
      reinterpret_cast<uint4*>(y)[u] = o;
    }
  }
}

// F32: the fp32 stream (gy fp32, optional gy16 bf16, gh fp32); else the bf16 stream (gy bf16, gh unused: the
// residual gradient is gy itself)
template <bool F32>
__global__ void __launch_bounds__(256) gelu_residual_bwd_kernel(const void* __restrict__ gy,
                                                                const __nv_bfloat16* __restrict__ gy16,
                                                                const __nv_bfloat16* __restrict__ a,
                                                                float* __restrict__ gh,
                                                                __nv_bfloat16* __restrict__ ga, StepShape sh) {
  for (int64_t u = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; u < sh.units;
       u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float g[8];
    if (F32) {
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 g0 = gy ? reinterpret_cast<const float4*>(gy)[2 * u] : z;       // no gy: that output is unused
      const float4 g1 = gy ? reinterpret_cast<const float4*>(gy)[2 * u + 1] : z;
      g[0] = g0.x; g[1] = g0.y; g[2] = g0.z; g[3] = g0.w;
      g[4] = g1.x; g[5] = g1.y; g[6] = g1.z; g[7] = g1.w;
      if (gy16) {
        const uint4 v = reinterpret_cast<const uint4*>(gy16)[u];
        const uint32_t* w = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          g[2 * e] += bf_lo(w[e]);
          g[2 * e + 1] += bf_hi(w[e]);
        }
      }
      if (gh) {
        reinterpret_cast<float4*>(gh)[2 * u] = make_float4(g[0], g[1], g[2], g[3]);
        reinterpret_cast<float4*>(gh)[2 * u + 1] = make_float4(g[4], g[5], g[6], g[7]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) g[e] = bf_round(g[e]);
    } else {
      const uint4 v = reinterpret_cast<const uint4*>(gy)[u];
      const uint32_t* w = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        g[2 * e] = bf_lo(w[e]);
        g[2 * e + 1] = bf_hi(w[e]);
      }
    }
    const int64_t po = pre_off(sh, u);
    const uint4 av = *reinterpret_cast<const uint4*>(a + po);
    const uint32_t* aw = reinterpret_cast<const uint32_t*>(&av);
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e)
      ow[e] = bf_pack(g[2 * e] * gelu_grad(bf_lo(aw[e])), g[2 * e + 1] * gelu_grad(bf_hi(aw[e])));
    *reinterpret_cast<uint4*>(ga + po) = o;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Token embedding of the training network, tok[b, n] = 2 type[n] + det[b, n] in {0..3} (cascade_net.py:279-285):
//   forward   h[b, n, :] = E[tok, :] (fp32) and its bf16 copy, one pass
//   backward  dE[k, :] = sum over (b, n) with tok = k of (g + g_bf16)[b, n, :]: per-block partial sums (each warp
//             a fixed set of rows, warps added in order in shared memory), then a fixed-order sum over the blocks;
//             deterministic, no atomics (the per-type sums below)
constexpr int kEmbBwdBlocks = 1024;
constexpr int kEmbBwdThreads = 256;
constexpr int kEmbMaxC = 256;

__global__ void __launch_bounds__(256) embed_tokens_fwd_kernel(const uint8_t* __restrict__ det,
                                                               const uint8_t* __restrict__ ctype,
                                                               const float* __restrict__ E, float* __restrict__ h,
                                                               __nv_bfloat16* __restrict__ h16, int64_t units, int N,
                                                               int C8) {
  for (int64_t u = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; u < units;
       u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = u / C8;
    const int c8 = static_cast<int>(u - row * C8);
    const int tok = 2 * __ldg(ctype + row % N) + __ldg(det + row);
    const float4 e0 = __ldg(reinterpret_cast<const float4*>(E + static_cast<int64_t>(tok) * C8 * 8 + c8 * 8));
    const float4 e1 = __ldg(reinterpret_cast<const float4*>(E + static_cast<int64_t>(tok) * C8 * 8 + c8 * 8 + 4));
    reinterpret_cast<float4*>(h)[2 * u] = e0;
    reinterpret_cast<float4*>(h)[2 * u + 1] = e1;
    uint4 o;
    o.x = bf_pack(e0.x, e0.y);
    o.y = bf_pack(e0.z, e0.w);
    o.z = bf_pack(e1.x, e1.y);
    o.w = bf_pack(e1.z, e1.w);
    reinterpret_cast<uint4*>(h16)[u] = o;
  }
}

// The backward as two sums per check type t, because a token is 2 t + det and det = 1 is rare: S_t over every row of
// type t and D_t over its rows with det = 1, so dE[2 t + 1] = D_t and dE[2 t] = S_t - D_t.  Each warp takes a fixed
// run of rows, one row per step with eight (C <= 128) or four rows' loads in flight; lane l holds channels
// 4 l .. 4 l + 3 (+ 128), read as
// one 16-byte (fp32) and one 8-byte (bf16) vector; the type and det branches are uniform across the warp.  The
// block's warps are added in order in shared memory: deterministic, no atomics.
// SLOTS: 128-channel slots per row (C <= 128 SLOTS); ROWS: rows whose loads are in flight per warp.
template <int SLOTS, int ROWS>
__global__ void __launch_bounds__(kEmbBwdThreads) embed_tokens_bwd_partial_kernel(
    const uint8_t* __restrict__ det, const uint8_t* __restrict__ ctype, const float* __restrict__ g,
    const __nv_bfloat16* __restrict__ g16, float* __restrict__ partial, int64_t rows, int N, int C) {
  __shared__ float red[kEmbBwdThreads / 32][4][kEmbMaxC];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kSlots = SLOTS;                          // 4 channels per lane per slot
  float S[2][kSlots][4], D[2][kSlots][4];
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int j = 0; j < kSlots; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) S[t][j][e] = D[t][j][e] = 0.f;
  const int64_t per_block = (rows + gridDim.x - 1) / gridDim.x;
  const int64_t r0 = blockIdx.x * per_block, r1 = min(rows, r0 + per_block);
  const int64_t per_warp = (r1 - r0 + kEmbBwdThreads / 32 - 1) / (kEmbBwdThreads / 32);
  const int64_t w0 = r0 + warp * per_warp, w1 = min(r1, w0 + per_warp);
  int n = w0 < w1 ? static_cast<int>(w0 % N) : 0;      // node of row w0; advanced without a division per row
  for (int64_t r = w0; r < w1; r += ROWS) {
    float v[ROWS][kSlots][4];
    int ty[ROWS], dt[ROWS];
#pragma unroll
    for (int u = 0; u < ROWS; ++u) {
      const int64_t rr = r + u;
      int nn = n + u;
      while (nn >= N) nn -= N;
      const bool ok = rr < w1;
      ty[u] = ok ? __ldg(ctype + nn) : 0;
      dt[u] = ok ? __ldg(det + rr) : 0;
#pragma unroll
      for (int j = 0; j < kSlots; ++j) {
        const int c = 4 * lane + 128 * j;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (ok && c < C) {
          if (g) x = __ldg(reinterpret_cast<const float4*>(g + rr * C + c));
          if (g16) {
            const uint2 h = __ldg(reinterpret_cast<const uint2*>(g16 + rr * C + c));
            x.x += __uint_as_float(h.x << 16);
            x.y += __uint_as_float(h.x & 0xFFFF0000u);
            x.z += __uint_as_float(h.y << 16);
            x.w += __uint_as_float(h.y & 0xFFFF0000u);
          }
        }
        v[u][j][0] = x.x;
        v[u][j][1] = x.y;
        v[u][j][2] = x.z;
        v[u][j][3] = x.w;
      }
    }
#pragma unroll
    for (int u = 0; u < ROWS; ++u) {
#pragma unroll
      for (int j = 0; j < kSlots; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (ty[u]) S[1][j][e] += v[u][j][e];
          else S[0][j][e] += v[u][j][e];
        }
      if (dt[u]) {
#pragma unroll
        for (int j = 0; j < kSlots; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (ty[u]) D[1][j][e] += v[u][j][e];
            else D[0][j][e] += v[u][j][e];
          }
      }
    }
    n += ROWS;
    while (n >= N) n -= N;
  }
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int j = 0; j < kSlots; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int c = 4 * lane + 128 * j + e;
        if (c < C) {
          red[warp][2 * t][c] = S[t][j][e] - D[t][j][e];
          red[warp][2 * t + 1][c] = D[t][j][e];
        }
      }
  __syncthreads();
  for (int i = threadIdx.x; i < 4 * C; i += blockDim.x) {
    const int k = i / C, c = i - k * C;
    float s = 0.f;
    for (int w = 0; w < kEmbBwdThreads / 32; ++w) s += red[w][k][c];
    partial[static_cast<int64_t>(blockIdx.x) * 4 * C + i] = s;
  }
}

__global__ void embed_tokens_bwd_sum_kernel(const float* __restrict__ partial, float* __restrict__ dE, int n, int blocks) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float v = 0.f;
  for (int b = 0; b < blocks; ++b) v += partial[static_cast<int64_t>(b) * n + i];
  dE[i] = v;
}

int step_shape(int64_t B, int32_t NT, int32_t C, int32_t n_types, StepShape* sh) {
  if (B < 0 || NT < 1 || C < 8 || C % 8 || n_types < 1 || NT % n_types)
    return fail(BPC_ERR_ARG, "B >= 0, NT a multiple of the type count, C a multiple of 8");
  sh->B = B;
  sh->NT = NT;
  sh->NTt = NT / n_types;
  sh->C8 = C / 8;
  sh->units = B * NT * (C / 8);
  sh->one_type = n_types == 1;
  sh->small = sh->units < (int64_t(1) << 32);
  return 0;
}

int elementwise_grid(int64_t units) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((units + 255) / 256, 8 * num_sms())));
}

}  // namespace

}  // namespace bpc

using namespace bpc;

extern "C" int bpc_gelu_residual_fwd(const void* a, const void* h, void* y, void* y_bf16, int64_t B, int32_t NT,
                                     int32_t C, int32_t n_types, int32_t h_dtype, bpc_stream_t stream) {
  StepShape sh;
  if (int e = step_shape(B, NT, C, n_types, &sh)) return e;
  if (h && h_dtype != BPC_DTYPE_BF16 && h_dtype != BPC_DTYPE_F32) return fail(BPC_ERR_ARG, "h must be bf16 or f32");
  const bool f32 = h && h_dtype == BPC_DTYPE_F32;
  if (sh.units == 0) return 0;
  if (!a || !y || (f32 && !y_bf16)) return fail(BPC_ERR_ARG, "null buffer");
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(y) |
       reinterpret_cast<uintptr_t>(y_bf16)) & 15)
    return fail(BPC_ERR_ARG, "a, h, y and y_bf16 must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const auto* ab = static_cast<const __nv_bfloat16*>(a);
  auto* yb = static_cast<__nv_bfloat16*>(y_bf16);
  const int grid = elementwise_grid(sh.units);
  if (!h)
    gelu_residual_fwd_kernel<0><<<grid, 256, 0, s>>>(ab, h, y, yb, sh);
  else if (!f32)
    gelu_residual_fwd_kernel<1><<<grid, 256, 0, s>>>(ab, h, y, yb, sh);
  else
    gelu_residual_fwd_kernel<2><<<grid, 256, 0, s>>>(ab, h, y, yb, sh);
  cudaError_t le = cudaGetLastError();
  if (le != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("gelu_residual_fwd_kernel launch: ") + cudaGetErrorString(le));
  return 0;
}

extern "C" int bpc_gelu_residual_bwd(const void* gy, const void* gy_bf16, const void* a, void* gh, void* ga,
                                     int64_t B, int32_t NT, int32_t C, int32_t n_types, int32_t gy_dtype,
                                     bpc_stream_t stream) {
  StepShape sh;
  if (int e = step_shape(B, NT, C, n_types, &sh)) return e;
  if (gy_dtype != BPC_DTYPE_BF16 && gy_dtype != BPC_DTYPE_F32) return fail(BPC_ERR_ARG, "gy must be bf16 or f32");
  const bool f32 = gy_dtype == BPC_DTYPE_F32;
  if (!f32 && (gy_bf16 || gh)) return fail(BPC_ERR_ARG, "the bf16 stream takes no second gradient and no gh");
  if (sh.units == 0) return 0;
  if ((!gy && !(f32 && gy_bf16)) || !a || !ga) return fail(BPC_ERR_ARG, "null buffer");
  if ((reinterpret_cast<uintptr_t>(gy) | reinterpret_cast<uintptr_t>(gy_bf16) | reinterpret_cast<uintptr_t>(a) |
       reinterpret_cast<uintptr_t>(gh) | reinterpret_cast<uintptr_t>(ga)) & 15)
    return fail(BPC_ERR_ARG, "gy, gy_bf16, a, gh and ga must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int grid = elementwise_grid(sh.units);
  const auto* ab = static_cast<const __nv_bfloat16*>(a);
  auto* gab = static_cast<__nv_bfloat16*>(ga);
  if (f32)
    gelu_residual_bwd_kernel<true><<<grid, 256, 0, s>>>(gy, static_cast<const __nv_bfloat16*>(gy_bf16), ab,
                                                        static_cast<float*>(gh), gab, sh);
  else
    gelu_residual_bwd_kernel<false><<<grid, 256, 0, s>>>(gy, nullptr, ab, nullptr, gab, sh);
  cudaError_t le = cudaGetLastError();
  if (le != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("gelu_residual_bwd_kernel launch: ") + cudaGetErrorString(le));
  return 0;
}

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

extern "C" int bpc_embed_tokens_fwd(const uint8_t* det, const uint8_t* check_type, const float* E, float* h,
                                    void* h_bf16, int64_t B, int32_t N, int32_t C, bpc_stream_t stream) {
  if (B < 0 || N < 1 || C < 8 || C % 8) return fail(BPC_ERR_ARG, "B >= 0, N >= 1, C a multiple of 8");
  if (B == 0) return 0;
  if (!det || !check_type || !E || !h || !h_bf16) return fail(BPC_ERR_ARG, "null buffer");
  if ((reinterpret_cast<uintptr_t>(E) | reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(h_bf16)) & 15)
    return fail(BPC_ERR_ARG, "E, h and h_bf16 must be 16-byte aligned");
  const int64_t units = B * N * (C / 8);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  embed_tokens_fwd_kernel<<<elementwise_grid(units), 256, 0, s>>>(det, check_type, E, h,
                                                                  static_cast<__nv_bfloat16*>(h_bf16), units, N, C / 8);
  cudaError_t le = cudaGetLastError();
  if (le != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("embed_tokens_fwd_kernel launch: ") + cudaGetErrorString(le));
  return 0;
}

extern "C" size_t bpc_embed_tokens_bwd_workspace_size(int32_t C) {
  return C < 1 ? 0 : static_cast<size_t>(kEmbBwdBlocks) * 4 * C * sizeof(float);
}

extern "C" int bpc_embed_tokens_bwd(const uint8_t* det, const uint8_t* check_type, const float* g, const void* g_bf16,
                                    float* dE, void* workspace, size_t workspace_bytes, int64_t B, int32_t N, int32_t C,
                                    bpc_stream_t stream) {
  if (B < 0 || N < 1 || C < 4 || C > kEmbMaxC || C % 4) return fail(BPC_ERR_ARG, "B >= 0, N >= 1, C in 4..256, a multiple of 4");
  if (!dE) return fail(BPC_ERR_ARG, "null dE");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (B == 0) {
    cudaError_t e = cudaMemsetAsync(dE, 0, sizeof(float) * 4 * C, s);
    return e == cudaSuccess ? 0 : fail(BPC_ERR_LAUNCH, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  }
  if (!det || !check_type || (!g && !g_bf16) || !workspace) return fail(BPC_ERR_ARG, "null buffer");
  if ((reinterpret_cast<uintptr_t>(g) & 15) || (reinterpret_cast<uintptr_t>(g_bf16) & 7))
    return fail(BPC_ERR_ARG, "g must be 16-byte and g_bf16 8-byte aligned");
  if (workspace_bytes < bpc_embed_tokens_bwd_workspace_size(C)) return fail(BPC_ERR_SPACE, "embedding workspace too small");
  float* partial = static_cast<float*>(workspace);
  auto partial_kernel = C <= 128 ? embed_tokens_bwd_partial_kernel<1, 8> : embed_tokens_bwd_partial_kernel<2, 4>;
  // every block resident at once (no partial last wave): the blocks that fit on the SMs, at most the workspace's
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, reinterpret_cast<const void*>(partial_kernel),
                                                    kEmbBwdThreads, 0) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const int grid = std::min(kEmbBwdBlocks, per_sm * num_sms());
  partial_kernel<<<grid, kEmbBwdThreads, 0, s>>>(det, check_type, g, static_cast<const __nv_bfloat16*>(g_bf16),
                                                 partial, B * N, N, C);
  embed_tokens_bwd_sum_kernel<<<(4 * C + 127) / 128, 128, 0, s>>>(partial, dE, 4 * C, grid);
  cudaError_t le = cudaGetLastError();
  if (le != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("embed_tokens_bwd launch: ") + cudaGetErrorString(le));
  return 0;
}
