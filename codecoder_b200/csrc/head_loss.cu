// The training network's X/Z head and its loss in one pass each way (the pre-decoder network in training: logits =
// linear(h_d, W, b) under bf16 autocast, loss = mean BCE-with-logits against the sampled 0/1 data-qubit errors, the
// reference's training step, cascade_train.py:292-320).  torch runs the head as three cuBLAS GEMMs with an output
// of width 2 (poor tiles for N = 2) and the loss as separate elementwise kernels; here each pass reads the data
// stream once:
//
//   forward    z_j = bf16(sum_c h[c] W_j[c] + b_j) (W, b rounded to bf16, fp32 sums), j = X, Z flip
//              loss = mean over rows and j of (1 - y) z + m + log(exp(-m) + exp(-z - m)),  m = max(-z, 0)
//   backward   s = grad_loss / n;  g_j = bf16((sigmoid(z_j) - y_j) s)  (the mean's and the loss's gradients, then the
//              cast back to the logits' bf16)
//              dh[c] = bf16(g_0 W_0[c] + g_1 W_1[c]);  dW_j = bf16(sum g_j h);  db_j = bf16(sum g_j)
//
// which are the roundings of torch's bf16 autocast path (the logits, their gradient, the GEMM outputs) with fp32
// sums.  Four lanes per row, lane l holding the 8-channel chunks l % 4, l % 4 + 4, ... (C a multiple of 8, at most
// 128), so that a warp pass covers 8 rows and the two dot products need two exchanges; several passes are in
// flight per warp.  Each warp takes a fixed run of rows, and the partial sums are added in a fixed order (within the
// warp, then over the block's warps, then over the blocks): deterministic, no atomics.
#include <algorithm>
#include <string>

#include "bpc.h"
#include "bpc_common.cuh"
#include "bpc_internal.h"

namespace bpc {
namespace {

constexpr int kHeadBlocks = 592;                // upper bound of the grid (the workspace holds this many partials)
constexpr int kHeadThreads = 256;
constexpr int kHeadMaxC = 128;
constexpr int kHeadLPR = 4;                     // lanes per row: lane l holds 8-channel chunks l % 4, + 4, + 8, ...
constexpr int kHeadRPW = 32 / kHeadLPR;         // rows per warp pass

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// partial sums per block: BWD: [db_0, db_1, dW_0[C], dW_1[C]]; forward: [loss].  NCH: 8-channel chunks per lane
// (C / 32 rounded up), U: warp passes (of 8 rows) in flight.
template <bool BWD, int NCH, int U>
__global__ void __launch_bounds__(kHeadThreads) head_bce_partial_kernel(
    const __nv_bfloat16* __restrict__ hd, const float* __restrict__ W, const float* __restrict__ bias,
    const uint8_t* __restrict__ y, const float* __restrict__ grad_loss, __nv_bfloat16* __restrict__ dh,
    float* __restrict__ partial, int64_t rows, int C, float n) {
  __shared__ float red[kHeadThreads / 32][2 + 2 * kHeadMaxC];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane & (kHeadLPR - 1), rw = lane / kHeadLPR;   // this lane's chunks, its row within a pass
  const int nchunk = C >> 3;
  float w0[NCH][8], w1[NCH][8];
  bool act[NCH];
#pragma unroll
  for (int m = 0; m < NCH; ++m) {
    act[m] = sub + kHeadLPR * m < nchunk;
    const int c = 8 * (sub + kHeadLPR * m);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      w0[m][e] = act[m] ? bf16r(__ldg(W + c + e)) : 0.f;
      w1[m][e] = act[m] ? bf16r(__ldg(W + C + c + e)) : 0.f;
    }
  }
  const float b0 = bf16r(__ldg(bias)), b1 = bf16r(__ldg(bias + 1));
  const float s = BWD ? __ldg(grad_loss) / n : 0.f;
  float loss = 0.f, db0 = 0.f, db1 = 0.f;
  float dw0[BWD ? NCH : 1][8], dw1[BWD ? NCH : 1][8];
#pragma unroll
  for (int m = 0; m < (BWD ? NCH : 1); ++m)
#pragma unroll
    for (int e = 0; e < 8; ++e) dw0[m][e] = dw1[m][e] = 0.f;
  const int64_t per_block = (rows + gridDim.x - 1) / gridDim.x;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * per_block, r1 = min(rows, r0 + per_block);
  const int64_t per_warp = (r1 - r0 + kHeadThreads / 32 - 1) / (kHeadThreads / 32);
  const int64_t wr0 = r0 + warp * per_warp, wr1 = min(r1, wr0 + per_warp);
  for (int64_t r = wr0; r < wr1; r += kHeadRPW * U) {
    uint4 hv[U][NCH];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t row = r + u * kHeadRPW + rw;
#pragma unroll
      for (int m = 0; m < NCH; ++m)
        hv[u][m] = (row < wr1 && act[m])
                       ? __ldg(reinterpret_cast<const uint4*>(hd + row * C + 8 * (sub + kHeadLPR * m)))
                       : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (r + u * kHeadRPW >= wr1) break;       // uniform across the warp
      const int64_t row = r + u * kHeadRPW + rw;
      const bool valid = row < wr1;
      float h[NCH][8];
      float p0 = 0.f, p1 = 0.f;
#pragma unroll
      for (int m = 0; m < NCH; ++m) {
        const uint32_t* hw = reinterpret_cast<const uint32_t*>(&hv[u][m]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          h[m][2 * e] = __uint_as_float(hw[e] << 16);
          h[m][2 * e + 1] = __uint_as_float(hw[e] & 0xFFFF0000u);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          p0 = fmaf(h[m][e], w0[m][e], p0);
          p1 = fmaf(h[m][e], w1[m][e], p1);
        }
      }
      // the row's four lanes hold the whole dot products after two exchanges
#pragma unroll
      for (int o = 1; o < kHeadLPR; o <<= 1) {
        p0 += __shfl_xor_sync(0xffffffffu, p0, o);
        p1 += __shfl_xor_sync(0xffffffffu, p1, o);
      }
      if (!valid) continue;
      const float z0 = bf16r(p0 + b0), z1 = bf16r(p1 + b1);
      const float y0 = static_cast<float>(__ldg(y + 2 * row) & 1), y1 = static_cast<float>(__ldg(y + 2 * row + 1) & 1);
      if (!BWD) {
        if (sub == 0) {
          const float m0 = fmaxf(-z0, 0.f), m1 = fmaxf(-z1, 0.f);
          loss += (1.f - y0) * z0 + m0 + logf(expf(-m0) + expf(-z0 - m0));
          loss += (1.f - y1) * z1 + m1 + logf(expf(-m1) + expf(-z1 - m1));
        }
      } else {
        const float g0 = bf16r((1.f / (1.f + expf(-z0)) - y0) * s);
        const float g1 = bf16r((1.f / (1.f + expf(-z1)) - y1) * s);
#pragma unroll
        for (int m = 0; m < NCH; ++m) {
          if (!act[m]) continue;
          uint4 o;
          uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            ow[e] = f2_to_bf2(f2_pack(fmaf(g1, w1[m][2 * e], g0 * w0[m][2 * e]),
                                      fmaf(g1, w1[m][2 * e + 1], g0 * w0[m][2 * e + 1])));
          *reinterpret_cast<uint4*>(dh + row * C + 8 * (sub + kHeadLPR * m)) = o;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            dw0[m][e] = fmaf(g0, h[m][e], dw0[m][e]);
            dw1[m][e] = fmaf(g1, h[m][e], dw1[m][e]);
          }
        }
        if (sub == 0) {
          db0 += g0;
          db1 += g1;
        }
      }
    }
  }
  // the warp's row groups added in a fixed order (lanes with the same chunks), then the block's warps in order
  for (int o = kHeadLPR; o < 32; o <<= 1) {
    if (!BWD) {
      loss += __shfl_xor_sync(0xffffffffu, loss, o);
    } else {
      db0 += __shfl_xor_sync(0xffffffffu, db0, o);
      db1 += __shfl_xor_sync(0xffffffffu, db1, o);
#pragma unroll
      for (int m = 0; m < NCH; ++m)
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          dw0[m][e] += __shfl_xor_sync(0xffffffffu, dw0[m][e], o);
          dw1[m][e] += __shfl_xor_sync(0xffffffffu, dw1[m][e], o);
        }
    }
  }
  if (!BWD) {
    if (lane == 0) red[warp][0] = loss;
  } else {
    if (lane == 0) {
      red[warp][0] = db0;
      red[warp][1] = db1;
    }
    if (lane < kHeadLPR)
#pragma unroll
      for (int m = 0; m < NCH; ++m)
        if (act[m])
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int c = 8 * (sub + kHeadLPR * m) + e;
            red[warp][2 + c] = dw0[m][e];
            red[warp][2 + C + c] = dw1[m][e];
          }
  }
  __syncthreads();
  const int slots = BWD ? 2 + 2 * C : 1;
  for (int i = threadIdx.x; i < slots; i += blockDim.x) {
    float t = 0.f;
    for (int w = 0; w < kHeadThreads / 32; ++w) t += red[w][i];
    partial[static_cast<int64_t>(blockIdx.x) * slots + i] = t;
  }
}

using HeadFn = void (*)(const __nv_bfloat16*, const float*, const float*, const uint8_t*, const float*,
                        __nv_bfloat16*, float*, int64_t, int, float);

// the kernel for C (a multiple of 8, at most 128) and its grid: as many blocks as fit on the SMs at once
template <bool BWD>
int head_kernel(int C, HeadFn* fn) {
  const int nch = (C / 8 + kHeadLPR - 1) / kHeadLPR;
  constexpr int U = BWD ? 2 : 4;
  *fn = nch <= 1 ? &head_bce_partial_kernel<BWD, 1, U>
      : nch == 2 ? &head_bce_partial_kernel<BWD, 2, U>
      : nch == 3 ? &head_bce_partial_kernel<BWD, 3, U>
                 : &head_bce_partial_kernel<BWD, 4, U>;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, reinterpret_cast<const void*>(*fn), kHeadThreads, 0) !=
          cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  return std::min(kHeadBlocks, per_sm * num_sms());
}

// fixed-order sum over the blocks: the loss (mean) or the bf16-rounded db, dW
__global__ void head_bce_sum_kernel(const float* __restrict__ partial, int slots, int blocks, float n, int bwd,
                                    float* __restrict__ loss, float* __restrict__ db, float* __restrict__ dW) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= slots) return;
  float t = 0.f;
  for (int k = 0; k < blocks; ++k) t += partial[static_cast<int64_t>(k) * slots + i];
  if (!bwd) {
    *loss = t / n;
  } else if (i < 2) {
    db[i] = bf16r(t);
  } else {
    dW[i - 2] = bf16r(t);
  }
}

int head_check(const void* hd, const float* W, const float* b, const uint8_t* y, int64_t rows, int32_t C, void* ws,
               size_t ws_bytes) {
  if (rows < 0 || C < 8 || C > kHeadMaxC || C % 8) return fail(BPC_ERR_ARG, "rows >= 0, C a multiple of 8 up to 128");
  if (rows > 0 && (!hd || !W || !b || !y)) return fail(BPC_ERR_ARG, "null buffer");
  if (reinterpret_cast<uintptr_t>(hd) & 15) return fail(BPC_ERR_ARG, "hd must be 16-byte aligned");
  if (!ws || ws_bytes < static_cast<size_t>(kHeadBlocks) * (2 + 2 * C) * sizeof(float))
    return fail(BPC_ERR_SPACE, "workspace smaller than bpc_head_bce_workspace_size(C)");
  return 0;
}

}  // namespace
}  // namespace bpc

using namespace bpc;

extern "C" size_t bpc_head_bce_workspace_size(int32_t C) {
  return C < 1 ? 0 : static_cast<size_t>(kHeadBlocks) * (2 + 2 * C) * sizeof(float);
}

extern "C" int bpc_head_bce_fwd(const void* hd, const float* W, const float* b, const uint8_t* labels, float* loss,
                                void* workspace, size_t workspace_bytes, int64_t rows, int32_t C, bpc_stream_t stream) {
  if (int e = head_check(hd, W, b, labels, rows, C, workspace, workspace_bytes)) return e;
  if (!loss) return fail(BPC_ERR_ARG, "null loss");
  if (rows == 0) return fail(BPC_ERR_ARG, "the mean over no rows is undefined");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  float* partial = static_cast<float*>(workspace);
  const float n = static_cast<float>(2 * rows);
  HeadFn fn;
  const int grid = head_kernel<false>(C, &fn);
  fn<<<grid, kHeadThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(hd), W, b, labels, nullptr, nullptr, partial, rows,
                                   C, n);
  head_bce_sum_kernel<<<1, 32, 0, s>>>(partial, 1, grid, n, 0, loss, nullptr, nullptr);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("head_bce forward: ") + cudaGetErrorString(e));
  return 0;
}

extern "C" int bpc_head_bce_bwd(const void* hd, const float* W, const float* b, const uint8_t* labels,
                                const float* grad_loss, void* dh, float* dW, float* db, void* workspace,
                                size_t workspace_bytes, int64_t rows, int32_t C, bpc_stream_t stream) {
  if (int e = head_check(hd, W, b, labels, rows, C, workspace, workspace_bytes)) return e;
  if (!grad_loss || !dW || !db || (rows > 0 && !dh)) return fail(BPC_ERR_ARG, "null buffer");
  if (reinterpret_cast<uintptr_t>(dh) & 15) return fail(BPC_ERR_ARG, "dh must be 16-byte aligned");
  if (rows == 0) return fail(BPC_ERR_ARG, "the mean over no rows is undefined");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  float* partial = static_cast<float*>(workspace);
  const float n = static_cast<float>(2 * rows);
  const int slots = 2 + 2 * C;
  HeadFn fn;
  const int grid = head_kernel<true>(C, &fn);
  fn<<<grid, kHeadThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(hd), W, b, labels, grad_loss,
                                   static_cast<__nv_bfloat16*>(dh), partial, rows, C, n);
  head_bce_sum_kernel<<<(slots + 127) / 128, 128, 0, s>>>(partial, slots, grid, n, 1, nullptr, db, dW);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("head_bce backward: ") + cudaGetErrorString(e));
  return 0;
}
