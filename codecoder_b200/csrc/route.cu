// Routing of pre-decoded shots to a fallback decoder, and the hand-off buffer it reads.
//
// The reference decides per shot whether its network's answer stands or the shot goes to PyMatching: a shot whose
// network logit lies within tau of zero is routed (evaluation/convlines/decoder.py:116-142, `route(c, tau)` and
// `decode`), and the routed shots' fired detectors go to the matcher (evaluation/timing/d7/router.cc:142-168,
// `pm_decode_row`).  For the pre-decoder the same rule reads its per-data-qubit logits and its residual syndrome:
//
//   conf[b]    = min over data nodes and X / Z of |logit[b, n, j]|
//   weight[b]  = number of set bits of residual[b, :]
//   routed[b]  = conf[b] < tau  or  (route_residual and weight[b] > 0)
//
// and the hand-off packs the routed shots, in ascending shot order, as (index[i], residual rows handoff[i, :]) for a
// matcher that decodes the residual.  Three kernels: per-shot statistics and flags (one warp per shot, coalesced row
// reads), the block counts' exclusive scan (one block), and the ordered scatter of indices and rows.
#include <algorithm>
#include <string>

#include "bpc.h"
#include "bpc_common.cuh"
#include "bpc_internal.h"

namespace bpc {
namespace {

constexpr int kRouteThreads = 256;          // 8 shots (warps) per block in the statistics kernel
constexpr int kScanChunk = 1024;            // shots per block of the scatter kernel

__global__ void __launch_bounds__(kRouteThreads) route_stats_kernel(const float* __restrict__ logits,
                                                                    const uint8_t* __restrict__ residual, int64_t B,
                                                                    int32_t n_logits, int32_t N_c, float tau,
                                                                    int route_residual, uint8_t* __restrict__ routed,
                                                                    float* __restrict__ conf,
                                                                    int32_t* __restrict__ weight) {
  const int lane = threadIdx.x & 31;
  const int64_t b = static_cast<int64_t>(blockIdx.x) * (kRouteThreads / 32) + (threadIdx.x >> 5);
  if (b >= B) return;
  const float* lg = logits + b * n_logits;
  float m = __int_as_float(0x7f800000);       // +inf
  for (int i = lane; i < n_logits; i += 32) m = fminf(m, fabsf(__ldg(lg + i)));
  const uint8_t* rs = residual + b * N_c;
  int w = 0;
  for (int i = lane; i < N_c; i += 32) w += __ldg(rs + i) & 1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    m = fminf(m, __shfl_xor_sync(0xffffffffu, m, o));
    w += __shfl_xor_sync(0xffffffffu, w, o);
  }
  if (lane == 0) {
    routed[b] = (m < tau || (route_residual && w > 0)) ? 1 : 0;
    if (conf) conf[b] = m;
    if (weight) weight[b] = w;
  }
}

// per-chunk counts of routed shots
__global__ void __launch_bounds__(kRouteThreads) route_count_kernel(const uint8_t* __restrict__ routed, int64_t B,
                                                                    int64_t* __restrict__ counts) {
  __shared__ int64_t part[kRouteThreads / 32];
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kScanChunk;
  int64_t n = 0;
  for (int i = threadIdx.x; i < kScanChunk; i += kRouteThreads)
    if (c0 + i < B) n += routed[c0 + i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = n;
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t s = 0;
    for (int i = 0; i < kRouteThreads / 32; ++i) s += part[i];
    counts[blockIdx.x] = s;
  }
}

// exclusive scan of the chunk counts in place (one block); *total = the number of routed shots
__global__ void __launch_bounds__(kRouteThreads) route_scan_kernel(int64_t* __restrict__ counts, int64_t n_chunks,
                                                                   int64_t* __restrict__ total) {
  __shared__ int64_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int64_t base = 0; base < n_chunks; base += kRouteThreads) {
    const int64_t i = base + threadIdx.x;
    const int64_t v = i < n_chunks ? counts[i] : 0;
    // inclusive warp scan, then across warps
    int64_t x = v;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    __shared__ int64_t wsum[kRouteThreads / 32];
    if (lane == 31) wsum[warp] = x;
    __syncthreads();
    int64_t off = 0;
    for (int k = 0; k < warp; ++k) off += wsum[k];
    const int64_t incl = carry + off + x;
    if (i < n_chunks) counts[i] = incl - v;
    __syncthreads();
    if (threadIdx.x == kRouteThreads - 1) carry = incl;
    __syncthreads();
  }
  if (threadIdx.x == 0) *total = carry;
}

// ordered scatter: each chunk writes its routed shots' indices from its scanned offset, then their residual rows
__global__ void __launch_bounds__(kRouteThreads) route_scatter_kernel(const uint8_t* __restrict__ routed, int64_t B,
                                                                      const int64_t* __restrict__ offsets,
                                                                      const uint8_t* __restrict__ residual,
                                                                      int32_t N_c, int64_t* __restrict__ index,
                                                                      uint8_t* __restrict__ handoff) {
  __shared__ int64_t wbase[kRouteThreads / 32 + 1];
  __shared__ int64_t pos[kScanChunk];
  __shared__ int n_here;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kScanChunk;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // shots c0 + 4 t .. 4 t + 3 per thread, in order: a per-thread count, a block scan, then positions
  int cnt = 0;
  uint32_t bits = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int64_t s = c0 + 4 * threadIdx.x + k;
    const uint32_t f = (s < B && routed[s]) ? 1u : 0u;
    bits |= f << k;
    cnt += static_cast<int>(f);
  }
  int x = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wbase[warp + 1] = x;
  __syncthreads();
  if (threadIdx.x == 0) {
    wbase[0] = 0;
    for (int k = 1; k <= kRouteThreads / 32; ++k) wbase[k] += wbase[k - 1];
    n_here = static_cast<int>(wbase[kRouteThreads / 32]);
  }
  __syncthreads();
  int64_t p = offsets[blockIdx.x] + wbase[warp] + (x - cnt);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (bits & (1u << k)) {
      const int64_t s = c0 + 4 * threadIdx.x + k;
      index[p] = s;
      pos[p - offsets[blockIdx.x]] = s;
      ++p;
    }
  }
  __syncthreads();
  if (!handoff) return;
  // rows of this chunk's routed shots, one warp per row, consecutive bytes over the lanes
  for (int r = warp; r < n_here; r += kRouteThreads / 32) {
    const int64_t s = pos[r];
    const uint8_t* src = residual + s * N_c;
    uint8_t* dst = handoff + (offsets[blockIdx.x] + r) * N_c;
    for (int i = lane; i < N_c; i += 32) dst[i] = src[i];
  }
}

}  // namespace
}  // namespace bpc

using namespace bpc;

extern "C" size_t bpc_route_workspace_size(int64_t B) {
  if (B < 0) return 0;
  const int64_t chunks = (B + kScanChunk - 1) / kScanChunk;
  return static_cast<size_t>(chunks + 2) * sizeof(int64_t);
}

extern "C" int bpc_route(const float* logits, const uint8_t* residual, int64_t B, int32_t n_data, int32_t n_checks,
                         float tau, int32_t route_residual, uint8_t* routed, int64_t* index, uint8_t* handoff,
                         int64_t* n_routed, float* conf, int32_t* weight, void* workspace, size_t workspace_bytes,
                         bpc_stream_t stream) {
  if (B < 0 || n_data < 1 || n_checks < 1) return fail(BPC_ERR_ARG, "B >= 0 and positive node counts");
  if (!(tau >= 0.f)) return fail(BPC_ERR_ARG, "tau must be a number >= 0");
  if (!n_routed) return fail(BPC_ERR_ARG, "null n_routed");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (B == 0) {   // an empty batch routes nothing (its buffers may be empty)
    cudaError_t e = cudaMemsetAsync(n_routed, 0, sizeof(int64_t), s);
    return e == cudaSuccess ? 0 : fail(BPC_ERR_LAUNCH, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  }
  if (!logits || !residual || !routed || !index) return fail(BPC_ERR_ARG, "null buffer");
  const int64_t chunks = (B + kScanChunk - 1) / kScanChunk;
  if (!workspace || workspace_bytes < bpc_route_workspace_size(B) || (reinterpret_cast<uintptr_t>(workspace) & 7))
    return fail(BPC_ERR_SPACE, "workspace smaller than bpc_route_workspace_size(B) or not 8-byte aligned");
  int64_t* counts = static_cast<int64_t*>(workspace);
  const int64_t stat_blocks = (B + kRouteThreads / 32 - 1) / (kRouteThreads / 32);
  if (stat_blocks > 0x7fffffffLL || chunks > 0x7fffffffLL) return fail(BPC_ERR_ARG, "batch too large");
  route_stats_kernel<<<static_cast<unsigned>(stat_blocks), kRouteThreads, 0, s>>>(
      logits, residual, B, 2 * n_data, n_checks, tau, route_residual, routed, conf, weight);
  route_count_kernel<<<static_cast<unsigned>(chunks), kRouteThreads, 0, s>>>(routed, B, counts);
  route_scan_kernel<<<1, kRouteThreads, 0, s>>>(counts, chunks, n_routed);
  route_scatter_kernel<<<static_cast<unsigned>(chunks), kRouteThreads, 0, s>>>(routed, B, counts, residual, n_checks,
                                                                             index, handoff);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("routing kernels: ") + cudaGetErrorString(e));
  return 0;
}
