// Bipartite-conv step on the CUDA cores, for narrow channel widths (C < 64) and fp32 networks, where the tensor
// cores do not apply (fp32 storage) or would idle (K C < 512).  Same arithmetic and epilogues as gmm_tc.cu.
//
// gmm_fma_narrow_kernel (C_in = C_out <= 32, contiguous channels) keeps the step's relation matrices resident in
// shared memory and gives each thread two shots and all output channels.  gmm_fma_kernel takes every other shape:
// tile = one target node n x 64 shots, 256 threads, thread t handles shot t / 4 and a quarter of the output
// channels, so the 4 threads of a shot are adjacent lanes (the head's dot product is two shuffles); for every
// non-pad relation the relation's weight W_r (C_out x C_in) is staged transposed in shared memory, in slices of
// C_in that fit 48 KB, and every thread runs C_in x C_out / 4 FMAs in fp32.
#include <algorithm>
#include <string>

#include "bpc_common.cuh"
#include "bpc_internal.h"

namespace bpc {

namespace {

constexpr int kFmaShots = 64;
constexpr int kFmaThreads = 256;
constexpr int kFmaSmemFloats = 12288;  // 48 KB

template <typename T>
__device__ __forceinline__ float ld_elem(const T* p);
template <>
__device__ __forceinline__ float ld_elem<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld_elem<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <typename T>
__device__ __forceinline__ T st_conv(float v);
template <>
__device__ __forceinline__ float st_conv<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 st_conv<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

struct FmaArgs {
  const void* x;
  int64_t x_shot_stride, x_node_stride, x_cg_stride;
  int64_t shots;
  int NS;
  const void* w;
  int type_split;
  const int32_t* idx;
  int NT, K, Ci, Co;
  void* y;
  int64_t y_shot_stride, y_node_stride, y_cg_stride;
  int epi;
  const float* epi_scale;
  const float* epi_shift;
  HeadEpilogue head;
};

// offset of channel c within a (shot, node) row whose 8-channel groups are cg_stride elements apart
__device__ __forceinline__ int64_t ch_off(int c, int64_t cg_stride) { return (c >> 3) * cg_stride + (c & 7); }

template <typename T>
__global__ void __launch_bounds__(kFmaThreads) gmm_fma_kernel(const FmaArgs a) {
  __shared__ float ws[kFmaSmemFloats];
  const int64_t tile = blockIdx.x;
  const int n = static_cast<int>(tile % a.NT);
  const int64_t s0 = (tile / a.NT) * kFmaShots;
  const int t = threadIdx.x;
  const int g = t & 3;
  const int64_t shot = s0 + (t >> 2);
  const bool ok = shot < a.shots;
  const int cq = a.Co >> 2;                  // output channels per thread (<= 64)
  const int o0 = g * cq;
  const T* x = reinterpret_cast<const T*>(a.x);
  const T* w = reinterpret_cast<const T*>(a.w) + ((n >= a.type_split) ? static_cast<int64_t>(a.Co) * a.K * a.Ci : 0);
  float acc[64];
#pragma unroll
  for (int i = 0; i < 64; ++i) acc[i] = 0.f;
  const int chunk = min(a.Ci, kFmaSmemFloats / a.Co);
  for (int r = 0; r < a.K; ++r) {
    const int src = __ldg(a.idx + static_cast<int64_t>(n) * a.K + r);
    if (src < 0 || src >= a.NS) continue;   // uniform across the block
    const T* xr = x + shot * a.x_shot_stride + static_cast<int64_t>(src) * a.x_node_stride;
    for (int i0 = 0; i0 < a.Ci; i0 += chunk) {
      const int ni = min(chunk, a.Ci - i0);
      __syncthreads();
      for (int e = t; e < ni * a.Co; e += kFmaThreads) {     // ws[i][o] = W[o, r Ci + i0 + i]
        const int o = e / ni, i = e - o * ni;
        ws[i * a.Co + o] = ld_elem(w + static_cast<int64_t>(o) * a.K * a.Ci + static_cast<int64_t>(r) * a.Ci + i0 + i);
      }
      __syncthreads();
      if (ok) {
        for (int i = 0; i < ni; ++i) {
          const float xv = ld_elem(xr + ch_off(i0 + i, a.x_cg_stride));
          const float* wrow = ws + i * a.Co + o0;
#pragma unroll
          for (int j = 0; j < 64; ++j)
            if (j < cq) acc[j] = fmaf(xv, wrow[j], acc[j]);
        }
      }
    }
  }
  float lg0 = 0.f, lg1 = 0.f;
  if (ok) {
    T* yr = reinterpret_cast<T*>(a.y) + shot * a.y_shot_stride + static_cast<int64_t>(n) * a.y_node_stride;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      if (j < cq) {
        float v = acc[j];
        T* yp = yr + ch_off(o0 + j, a.y_cg_stride);
        if (a.epi == kEpiGeluInit) v = gelu_tanh(v);
        else if (a.epi == kEpiGeluResid) v = ld_elem(yp) + gelu_tanh(v);
        else if (a.epi == kEpiAdd) v = ld_elem(yp) + v;
        else if (a.epi == kEpiAffineSilu) v = silu_exact(fmaf(v, __ldg(a.epi_scale + o0 + j), __ldg(a.epi_shift + o0 + j)));
        const T sv = st_conv<T>(v);
        *yp = sv;
        if (a.head.head_w) {
          const float f = ld_elem(&sv);
          lg0 = fmaf(f, __ldg(a.head.head_w + o0 + j), lg0);
          lg1 = fmaf(f, __ldg(a.head.head_w + a.Co + o0 + j), lg1);
        }
      }
    }
  }
  if (a.head.head_w) {
    lg0 += __shfl_xor_sync(0xffffffffu, lg0, 1);
    lg0 += __shfl_xor_sync(0xffffffffu, lg0, 2);
    lg1 += __shfl_xor_sync(0xffffffffu, lg1, 1);
    lg1 += __shfl_xor_sync(0xffffffffu, lg1, 2);
    lg0 += __ldg(a.head.head_b);
    lg1 += __ldg(a.head.head_b + 1);
    if (ok && g == 0) {
      float* lp = a.head.logits + shot * a.head.lg_shot_stride + static_cast<int64_t>(n) * a.head.lg_node_stride;
      lp[0] = lg0;
      lp[1] = lg1;
    }
    if (a.head.res_bits) {
      const int lane = t & 31;
      const uint32_t b0 = __ballot_sync(0xffffffffu, ok && g == 0 && lg0 > 0.f);
      const uint32_t b1 = __ballot_sync(0xffffffffu, ok && g == 0 && lg1 > 0.f);
      uint32_t m0 = 0, m1 = 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) {             // lanes 4k hold shot k of this warp
        m0 |= ((b0 >> (4 * k)) & 1u) << k;
        m1 |= ((b1 >> (4 * k)) & 1u) << k;
      }
      const int64_t wshot = s0 + (t >> 5) * 8;  // first shot of this warp, a multiple of 8
      if (lane < 4) {
        const int j = lane >> 1;
        const int32_t c = __ldg(a.head.xor_nbr + static_cast<int64_t>(n) * 4 + lane);
        const uint32_t m = (j ? m1 : m0) << (wshot & 31);
        if (c >= 0 && m) atomicXor(a.head.res_bits + static_cast<int64_t>(c) * a.head.res_words + (wshot >> 5), m);
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Narrow steps (C_in = C_out = C <= 32, channels contiguous): a persistent block keeps the step's relation matrices
// of both target types in shared memory, transposed to ws[type][r][i][o] (fp32), for its whole life.  Tile = one
// target node x 256 shots; thread t owns shots t and t + 128 of the tile and all C outputs of both (2 C fp32
// accumulators), so every weight it reads from shared memory (a broadcast: the block's threads read the same word)
// feeds two FMAs, and its rows are C contiguous elements (vector loads and stores; the 32 lanes of a warp cover 32
// consecutive shots, contiguous in the node-major layouts).  Accumulation order per output: relations in order, input
// channels in order, as gmm_fma_kernel: the same bits.  The head's four quarter sums are added as that kernel's
// shuffles add them.
constexpr int kNarrowThreads = 128;

// the value a store of type T keeps
template <typename T>
__device__ __forceinline__ float as_stored(float v) {
  if constexpr (sizeof(T) == 4) return v;
  else return __bfloat162float(__float2bfloat16_rn(v));
}
constexpr int kNarrowShots = 2 * kNarrowThreads;

// a row of C contiguous elements; RO: through the read-only path (rows this kernel does not write)
template <typename T, int C, bool RO = true>
__device__ __forceinline__ void ld_row(const T* p, float (&v)[C]) {
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < C / 4; ++i) {
      const float4 f = RO ? __ldg(reinterpret_cast<const float4*>(p) + i) : reinterpret_cast<const float4*>(p)[i];
      v[4 * i] = f.x;
      v[4 * i + 1] = f.y;
      v[4 * i + 2] = f.z;
      v[4 * i + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < C / 8; ++i) {
      const uint4 u = RO ? __ldg(reinterpret_cast<const uint4*>(p) + i) : reinterpret_cast<const uint4*>(p)[i];
      const uint32_t* w = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        v[8 * i + 2 * e] = __uint_as_float(w[e] << 16);
        v[8 * i + 2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u);
      }
    }
  }
}

template <typename T, int C>
__device__ __forceinline__ void st_row(T* p, const float (&v)[C]) {
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < C / 4; ++i)
      reinterpret_cast<float4*>(p)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < C / 8; ++i) {
      uint4 u;
      uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) w[e] = f2_to_bf2(f2_pack(v[8 * i + 2 * e], v[8 * i + 2 * e + 1]));
      reinterpret_cast<uint4*>(p)[i] = u;
    }
  }
}

template <typename T, int C>
__global__ void __launch_bounds__(kNarrowThreads) gmm_fma_narrow_kernel(const FmaArgs a, int64_t num_tiles) {
  extern __shared__ float4 ws4[];
  float* ws = reinterpret_cast<float*>(ws4);
  const int n_types = a.type_split < a.NT ? 2 : 1;
  const int t = threadIdx.x;
  const T* x = reinterpret_cast<const T*>(a.x);
  const T* w = reinterpret_cast<const T*>(a.w);
  // ws[(ty K + r) C C + i C + o] = W_ty[o, r C + i]
  for (int e = t; e < n_types * a.K * C * C; e += kNarrowThreads) {
    const int o = e % C, i = (e / C) % C, tr = e / (C * C);
    ws[e] = ld_elem(w + (static_cast<int64_t>(tr / a.K) * C + o) * a.K * C + static_cast<int64_t>(tr % a.K) * C + i);
  }
  __syncthreads();
  for (int64_t tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
    const int n = static_cast<int>(tile % a.NT);
    const int64_t s0 = (tile / a.NT) * kNarrowShots;
    const int64_t sh[2] = {s0 + t, s0 + kNarrowThreads + t};
    const bool ok[2] = {sh[0] < a.shots, sh[1] < a.shots};
    const float* wt = ws + static_cast<int64_t>(n >= a.type_split ? 1 : 0) * a.K * C * C;
    float acc[2][C];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int o = 0; o < C; ++o) acc[h][o] = 0.f;
    for (int r = 0; r < a.K; ++r) {
      const int src = __ldg(a.idx + static_cast<int64_t>(n) * a.K + r);
      if (src < 0 || src >= a.NS) continue;   // uniform across the block
      float xv[2][C];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (ok[h]) {
          ld_row<T, C>(x + sh[h] * a.x_shot_stride + static_cast<int64_t>(src) * a.x_node_stride, xv[h]);
        } else {
#pragma unroll
          for (int i = 0; i < C; ++i) xv[h][i] = 0.f;
        }
      }
      const float4* wr = reinterpret_cast<const float4*>(wt + r * C * C);
#pragma unroll
      for (int i = 0; i < C; ++i)
#pragma unroll
        for (int o4 = 0; o4 < C / 4; ++o4) {
          const float4 wv = wr[i * (C / 4) + o4];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            acc[h][4 * o4] = fmaf(xv[h][i], wv.x, acc[h][4 * o4]);
            acc[h][4 * o4 + 1] = fmaf(xv[h][i], wv.y, acc[h][4 * o4 + 1]);
            acc[h][4 * o4 + 2] = fmaf(xv[h][i], wv.z, acc[h][4 * o4 + 2]);
            acc[h][4 * o4 + 3] = fmaf(xv[h][i], wv.w, acc[h][4 * o4 + 3]);
          }
        }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      T* yr = reinterpret_cast<T*>(a.y) + sh[h] * a.y_shot_stride + static_cast<int64_t>(n) * a.y_node_stride;
      float out[C];
      float res[C];
      const bool resid = a.epi == kEpiGeluResid || a.epi == kEpiAdd;
      if (resid && ok[h]) ld_row<T, C, false>(yr, res);   // this kernel writes these rows
#pragma unroll
      for (int o = 0; o < C; ++o) {
        float v = acc[h][o];
        if (a.epi == kEpiGeluInit) v = gelu_tanh(v);
        else if (a.epi == kEpiGeluResid) v = res[o] + gelu_tanh(v);
        else if (a.epi == kEpiAdd) v = res[o] + v;
        else if (a.epi == kEpiAffineSilu) v = silu_exact(fmaf(v, __ldg(a.epi_scale + o), __ldg(a.epi_shift + o)));
        out[o] = v;
      }
      if (ok[h]) st_row<T, C>(yr, out);
      if (a.head.head_w) {
        // the values as stored, four quarter sums added pairwise (as the four-thread shuffle does)
        float q0[4], q1[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          q0[g] = 0.f;
          q1[g] = 0.f;
#pragma unroll
          for (int j = 0; j < C / 4; ++j) {
            const int o = g * (C / 4) + j;
            const float f = as_stored<T>(out[o]);
            q0[g] = fmaf(f, __ldg(a.head.head_w + o), q0[g]);
            q1[g] = fmaf(f, __ldg(a.head.head_w + C + o), q1[g]);
          }
        }
        const float l0 = ((q0[0] + q0[1]) + (q0[2] + q0[3])) + __ldg(a.head.head_b);
        const float l1 = ((q1[0] + q1[1]) + (q1[2] + q1[3])) + __ldg(a.head.head_b + 1);
        if (ok[h]) {
          float* lp = a.head.logits + sh[h] * a.head.lg_shot_stride + static_cast<int64_t>(n) * a.head.lg_node_stride;
          lp[0] = l0;
          lp[1] = l1;
        }
        if (a.head.res_bits) {
          const int lane = t & 31;
          const uint32_t m0 = __ballot_sync(0xffffffffu, ok[h] && l0 > 0.f);
          const uint32_t m1 = __ballot_sync(0xffffffffu, ok[h] && l1 > 0.f);
          const int64_t wshot = sh[h] - lane;        // first shot of this warp's 32, a multiple of 32
          if (lane < 4) {
            const int j = lane >> 1;
            const int32_t c = __ldg(a.head.xor_nbr + static_cast<int64_t>(n) * 4 + lane);
            const uint32_t m = j ? m1 : m0;
            if (c >= 0 && m) atomicXor(a.head.res_bits + static_cast<int64_t>(c) * a.head.res_words + (wshot >> 5), m);
          }
        }
      }
    }
  }
}

}  // namespace

int gmm_fma_launch(const GmmProblem& p, bool f32, cudaStream_t stream) {
  if (p.Co < 4 || p.Co > 256 || p.Co % 4 != 0) return fail(2, "CUDA-core path needs C_out in 4..256, multiple of 4");
  if (p.Ci < 1) return fail(2, "C_in must be positive");
  if (p.K < 1 || p.NT < 1 || p.NS < 1) return fail(2, "empty problem");
  if (p.epi == kEpiAffineSilu && (!p.epi_scale || !p.epi_shift))
    return fail(2, "the affine + SiLU epilogue needs scale and shift vectors");
  if (p.shots <= 0) return 0;
  FmaArgs a;
  a.x = p.x;
  a.x_shot_stride = p.x_shot_stride;
  a.x_node_stride = p.x_node_stride;
  a.x_cg_stride = p.x_cg_stride;
  a.shots = p.shots;
  a.NS = p.NS;
  a.w = p.w;
  a.type_split = p.n_wtypes > 1 ? p.type_split : p.NT;
  a.idx = p.idx;
  a.NT = p.NT;
  a.K = p.K;
  a.Ci = p.Ci;
  a.Co = p.Co;
  a.y = p.y;
  a.y_shot_stride = p.y_shot_stride;
  a.y_node_stride = p.y_node_stride;
  a.y_cg_stride = p.y_cg_stride;
  a.epi = p.epi;
  a.epi_scale = p.epi_scale;
  a.epi_shift = p.epi_shift;
  a.head = p.head;
  // narrow equal-width steps with contiguous, 16-byte aligned rows: the persistent kernel with resident weights
  const size_t es = f32 ? 4 : 2;
  const bool aligned = ((reinterpret_cast<uintptr_t>(p.x) | reinterpret_cast<uintptr_t>(p.y)) & 15) == 0 &&
                       ((p.x_shot_stride | p.x_node_stride | p.y_shot_stride | p.y_node_stride) * static_cast<int64_t>(es)) %
                               16 == 0;
  if (p.Ci == p.Co && (p.Ci == 8 || p.Ci == 16 || p.Ci == 32) && p.K <= 16 && p.x_cg_stride == 8 &&
      p.y_cg_stride == 8 && aligned) {
    const int n_types = a.type_split < a.NT ? 2 : 1;
    const int smem = n_types * p.K * p.Ci * p.Ci * 4;
    const void* fn = nullptr;
    switch (p.Ci) {
      case 8: fn = f32 ? reinterpret_cast<const void*>(&gmm_fma_narrow_kernel<float, 8>)
                       : reinterpret_cast<const void*>(&gmm_fma_narrow_kernel<__nv_bfloat16, 8>); break;
      case 16: fn = f32 ? reinterpret_cast<const void*>(&gmm_fma_narrow_kernel<float, 16>)
                        : reinterpret_cast<const void*>(&gmm_fma_narrow_kernel<__nv_bfloat16, 16>); break;
      default: fn = f32 ? reinterpret_cast<const void*>(&gmm_fma_narrow_kernel<float, 32>)
                        : reinterpret_cast<const void*>(&gmm_fma_narrow_kernel<__nv_bfloat16, 32>); break;
    }
    if (int e = allow_smem(fn, smem)) return e;
    const int64_t ntiles = static_cast<int64_t>(p.NT) * ((p.shots + kNarrowShots - 1) / kNarrowShots);
    const int per_sm = std::max(1, std::min(8, (200 * 1024) / std::max(smem, 1)));
    const int64_t grid = std::min<int64_t>(ntiles, static_cast<int64_t>(num_sms()) * per_sm);
    void* args[] = {&a, const_cast<int64_t*>(&ntiles)};
    cudaError_t le = cudaLaunchKernel(fn, dim3(static_cast<unsigned>(grid)), dim3(kNarrowThreads), args,
                                      static_cast<size_t>(smem), stream);
    if (le != cudaSuccess) {
      cudaGetLastError();   // a refused launch leaves nothing behind for the caller's next error check
      return fail(4, std::string("gmm_fma_narrow_kernel launch: ") + cudaGetErrorString(le));
    }
    return 0;
  }
  const int64_t tiles = static_cast<int64_t>(p.NT) * ((p.shots + kFmaShots - 1) / kFmaShots);
  if (tiles > 0x7fffffffLL) return fail(2, "too many tiles for one launch");
  if (f32)
    gmm_fma_kernel<float><<<static_cast<unsigned>(tiles), kFmaThreads, 0, stream>>>(a);
  else
    gmm_fma_kernel<__nv_bfloat16><<<static_cast<unsigned>(tiles), kFmaThreads, 0, stream>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(4, std::string("gmm_fma_kernel launch: ") + cudaGetErrorString(e));
  return 0;
}

}  // namespace bpc
