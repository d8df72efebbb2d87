// Bipartite-conv step on the 5th-generation tensor cores (sm_100a): one persistent, warp-specialised kernel.
//
//   y[s, n, :] (op)= sum_r x[s, idx[n, r], :] W_{type(n), r}^T            (cascade_triton.py:5,40 -- same arithmetic)
//
// Tile = one target node n x 128 shots.  The 128 rows of the MMA are shots, so for a given relation r every row of
// the tile reads the same source node idx[n, r]: the neighbour "gather" is one strided TMA box per (tile, relation,
// 64-channel block) -- x viewed as the 3D tensor (channel, shot, node) -- and a pad slot (idx outside [0, NS)) is a
// relation the tile skips entirely (no load, no MMA).  The same kernel serves shot-major x (B, NS, C), the layout of
// the reference's op, and the node-major (NS, B, C) layout the pre-decoder keeps its activations in; only the
// tensor-map strides differ.
//
// Roles (192 threads, one CTA per SM):
//   warp 0     TMA producer: A box (128 shots x 64 channels, 16 KB) + W box (Co rows x 64 channels) per stage
//   warp 1     TMEM owner and MMA issuer: tcgen05.mma M=128 N=Co K=16 from two 128B-swizzled K-major operands,
//              fp32 accumulator in TMEM, double-buffered (2 x Co columns) so the epilogue of tile i overlaps the
//              MMAs of tile i + 1
//   warps 2-5  epilogue: tcgen05.ld of the accumulator (one shot per thread), GELU / residual add, bf16 store,
//              and for the pre-decoder's last check -> data step the X / Z head, the threshold and the XOR of the
//              predicted flips into the bit-packed residual syndrome (one ballot + atomicXor per warp and check)
// Every wait is bounded (mbar_wait); a timeout sets the status word and the CTA drains and returns.
#include <cstdio>
#include <mutex>
#include <string>
#include <unordered_map>

#include <cudaTypedefs.h>

#include "bpc_common.cuh"
#include "bpc_internal.h"

namespace bpc {

namespace {

constexpr int kThreads = 320;         // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kEpiWarps = 8;
constexpr int kBlockM = 128;          // rows of one MMA (shots)
constexpr int kKBlock = 64;           // channels per 128-byte swizzled row
constexpr int kSubBytes = kBlockM * kKBlock * 2;   // one 128-row x 64-channel A block
constexpr int kMaxStages = 8;
constexpr int kSmemLimit = 232448;    // 227 KB opt-in per CTA

// Shots per tile = 128 MT: MT = 2 lets two MMAs share every W stage (half the W traffic per FLOP) while the
// accumulators (2 buffers x MT x Co fp32 columns) still fit the 512 TMEM columns.
__host__ __device__ constexpr int mt_for(int Co) { return Co <= 128 ? 2 : 1; }

struct TcArgs {
  const int32_t* idx;
  int NT, NS, K, Ci, Co;
  int type_split, n_kb, stages;
  int64_t shots;
  int64_t num_tiles;
  void* y;
  int64_t y_shot_stride, y_node_stride;
  int epi;
  HeadEpilogue head;
  int* status;
  uint64_t timeout_ns;
  uint32_t tmem_cols;
};

__device__ __forceinline__ uint32_t valid_mask(const int32_t* idx, int n, int K, int NS) {
  uint32_t m = 0;
  for (int r = 0; r < K; ++r) {
    const int s = __ldg(idx + static_cast<int64_t>(n) * K + r);
    if (s >= 0 && s < NS) m |= 1u << r;
  }
  return m;
}

__device__ __forceinline__ void ld_row_chunk(const __nv_bfloat16* p, uint4 (&r)[4]) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int j = 0; j < 4; ++j) r[j] = q[j];
}

template <int MT, int NCH>
__global__ void __launch_bounds__(kThreads, 1)
    gmm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW, const TcArgs a) {
  constexpr int Co = NCH * 32;
  constexpr int kTileM = kBlockM * MT;
  constexpr uint32_t kABytes = kSubBytes * MT;
  constexpr uint32_t kStageBytes = kABytes + Co * 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * kStageBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* accf = bars + 2 * S;
  uint64_t* acce = bars + 2 * S + 2;
  uint64_t* drain = bars + 2 * S + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(smem_u32(&full[i]), 1);
      mbar_init(smem_u32(&empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&accf[i]), 1);
      mbar_init(smem_u32(&acce[i]), kEpiWarps);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), a.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_parity = 0;   // stages with a load in flight and the parity it completes
      bool ok = true;
      for (int64_t tile = blockIdx.x; tile < a.num_tiles && ok; tile += gridDim.x) {
        const int n = static_cast<int>(tile % a.NT);
        const int s0 = static_cast<int>((tile / a.NT) * kTileM);
        const int wrow = (n >= a.type_split) ? Co : 0;
        for (int r = 0; r < a.K && ok; ++r) {
          const int src = __ldg(a.idx + static_cast<int64_t>(n) * a.K + r);
          if (src < 0 || src >= a.NS) continue;
          for (int kb = 0; kb < a.n_kb; ++kb) {
            if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, a.status, a.timeout_ns)) {
              ok = false;
              break;
            }
            const uint32_t sa = smem_u32(smem + stage * kStageBytes);
            const uint32_t fb = smem_u32(&full[stage]);
            mbar_arrive_expect_tx(fb, kStageBytes);
            tma_load_3d(sa, &tmA, kb * kKBlock, s0, src, fb);          // kTileM shots x 64 channels
            tma_load_3d(sa + kABytes, &tmW, kb * kKBlock, r, wrow, fb);  // Co rows x 64 channels of W_r
            armed |= 1u << stage;
            armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
            if (++stage == S) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
      if (!ok) {
        // drain: wait (bounded) for every load this thread issued before leaving the CTA's shared memory
        for (int i = 0; i < S; ++i)
          if (armed & (1u << i)) {
            const uint32_t par = (armed_parity >> i) & 1u;
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(smem_u32(&full[i]), par) && globaltimer_ns() - t0 < a.timeout_ns) {
            }
          }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kBlockM, Co);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; tile < a.num_tiles && ok; tile += gridDim.x) {
        const int n = static_cast<int>(tile % a.NT);
        const uint32_t vm = valid_mask(a.idx, n, a.K, a.NS);
        if (!mbar_wait(smem_u32(&acce[acc]), acc_phase ^ 1u, abort_flag, a.status, a.timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * MT * Co);
        uint32_t accumulate = 0;
        for (int r = 0; r < a.K && ok; ++r) {
          if (!(vm & (1u << r))) continue;
          for (int kb = 0; kb < a.n_kb; ++kb) {
            if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, a.status, a.timeout_ns)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sa = smem_u32(smem + stage * kStageBytes);
            const int ksteps = min(4, (a.Ci - kb * kKBlock + 15) / 16);
            for (int k = 0; k < ksteps; ++k) {
              const uint64_t bd = sdesc_k_sw128(sa + kABytes + k * 32);
#pragma unroll
              for (int m = 0; m < MT; ++m)
                tc_mma_ss(d_tmem + m * Co, sdesc_k_sw128(sa + m * kSubBytes + k * 32), bd, idesc, accumulate);
              accumulate = 1;
            }
            tc_commit(smem_u32(&empty[stage]));   // frees the stage when these MMAs have read it
            if (++stage == S) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
        if (!ok) break;
        tc_commit(smem_u32(&accf[acc]));          // accumulators ready for the epilogue
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      // drain outstanding MMAs before the CTA releases tensor memory
      tc_commit(smem_u32(drain));
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(smem_u32(drain), 0) && globaltimer_ns() - t0 < a.timeout_ns) {
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..9)
    const int q = warp & 3;                   // TMEM lane quarter this warp may access
    const int m = (warp - 2) >> 2;            // which 128-shot sub-tile
    const int row = q * 32 + lane;
    const bool active = m < MT;
    const bool resid = a.epi == kEpiGeluResid;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int64_t tile = blockIdx.x; tile < a.num_tiles; tile += gridDim.x) {
      const int n = static_cast<int>(tile % a.NT);
      const int64_t s0 = (tile / a.NT) * kTileM + m * kBlockM;
      const int64_t shot = s0 + row;
      const bool ok = active && shot < a.shots;
      __nv_bfloat16* yrow = reinterpret_cast<__nv_bfloat16*>(a.y) + shot * a.y_shot_stride +
                            static_cast<int64_t>(n) * a.y_node_stride;
      // the residual rows do not depend on the MMAs: start loading them before waiting for the accumulator
      uint4 r0[4], r1[4];
      if (resid && ok) {
        ld_row_chunk(yrow, r0);
        if (NCH > 1) ld_row_chunk(yrow + 32, r1);
      }
      const uint32_t vm = active ? valid_mask(a.idx, n, a.K, a.NS) : 0u;
      if (!mbar_wait(smem_u32(&accf[acc]), acc_phase, abort_flag, a.status, a.timeout_ns)) break;
      tc_fence_after();
      float lg0 = 0.f, lg1 = 0.f;
      if (active) {
        const uint32_t taddr =
            tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * MT * Co + m * Co);
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          float v[32];
          tmem_ld32(taddr + c * 32, v);
          if (vm == 0) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0.f;
          }
          uint4 cur[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) cur[j] = (c & 1) ? r1[j] : r0[j];
          if (resid && ok && c + 2 < NCH) {
            if (c & 1) ld_row_chunk(yrow + (c + 2) * 32, r1);
            else ld_row_chunk(yrow + (c + 2) * 32, r0);
          }
          if (ok) {
            uint4* yp = reinterpret_cast<uint4*>(yrow + c * 32);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&cur[j]);
              uint4 u;
              __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float x0 = v[j * 8 + 2 * e], x1 = v[j * 8 + 2 * e + 1];
                if (a.epi != kEpiStore) {
                  x0 = gelu_tanh_fast(x0);
                  x1 = gelu_tanh_fast(x1);
                }
                if (resid) {
                  const float2 f = __bfloat1622float2(h[e]);
                  x0 += f.x;
                  x1 += f.y;
                }
                o[e] = __floats2bfloat162_rn(x0, x1);
                if (a.head.head_w) {
                  const float2 f = __bfloat1622float2(o[e]);   // the stored (rounded) value feeds the head
                  const int col = c * 32 + j * 8 + 2 * e;
                  lg0 = fmaf(f.x, __ldg(a.head.head_w + col), lg0);
                  lg0 = fmaf(f.y, __ldg(a.head.head_w + col + 1), lg0);
                  lg1 = fmaf(f.x, __ldg(a.head.head_w + Co + col), lg1);
                  lg1 = fmaf(f.y, __ldg(a.head.head_w + Co + col + 1), lg1);
                }
              }
              yp[j] = u;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&acce[acc]));
      if (active && a.head.head_w) {
        lg0 += __ldg(a.head.head_b);
        lg1 += __ldg(a.head.head_b + 1);
        if (ok) {
          float2* lp = reinterpret_cast<float2*>(a.head.logits + shot * a.head.lg_shot_stride +
                                                 static_cast<int64_t>(n) * a.head.lg_node_stride);
          *lp = make_float2(lg0, lg1);
        }
        if (a.head.res_bits) {
          const uint32_t m0 = __ballot_sync(0xffffffffu, ok && lg0 > 0.f);
          const uint32_t m1 = __ballot_sync(0xffffffffu, ok && lg1 > 0.f);
          if (lane < 4) {
            const int j = lane >> 1;
            const int32_t c = __ldg(a.head.xor_nbr + static_cast<int64_t>(n) * 4 + lane);
            const uint32_t msk = j ? m1 : m0;
            if (c >= 0 && msk)
              atomicXor(a.head.res_bits + static_cast<int64_t>(c) * a.head.res_words + (s0 >> 5) + q, msk);
          }
        }
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, a.tmem_cols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int smem_bytes_for(int Co, int stages) {
  return 1024 + stages * (kSubBytes * mt_for(Co) + Co * 128) + (2 * stages + 5) * 8 + 8;
}

int stages_for(int Co) {
  int s = kMaxStages;
  while (s > 2 && smem_bytes_for(Co, s) > kSmemLimit) --s;
  return s;
}

using KernelFn = void (*)(CUtensorMap, CUtensorMap, TcArgs);

template <int NCH>
KernelFn kernel_for() {
  return &gmm_tc_kernel<mt_for(NCH * 32), NCH>;
}

KernelFn select_kernel(int Co) {
  switch (Co / 32) {
    case 1: return kernel_for<1>();
    case 2: return kernel_for<2>();
    case 3: return kernel_for<3>();
    case 4: return kernel_for<4>();
    case 5: return kernel_for<5>();
    case 6: return kernel_for<6>();
    case 7: return kernel_for<7>();
    case 8: return kernel_for<8>();
    default: return nullptr;
  }
}

}  // namespace

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 1;
  }
  return n;
}

int gmm_tc_check(const GmmProblem& p) {
  if (p.Ci < 64 || p.Ci % 8 != 0) return fail(2, "tcgen05 path needs C_in >= 64 and a multiple of 8");
  if (p.Co < 32 || p.Co > 256 || p.Co % 32 != 0) return fail(2, "tcgen05 path needs C_out in 32..256, multiple of 32");
  if (p.K < 1 || p.K > 32) return fail(2, "relation count K must be in 1..32");
  if (p.NT < 1 || p.NS < 1) return fail(2, "empty node set");
  if (p.n_wtypes < 1 || p.n_wtypes > 2) return fail(2, "one or two weight sets");
  const uintptr_t xa = reinterpret_cast<uintptr_t>(p.x), wa = reinterpret_cast<uintptr_t>(p.w),
                  ya = reinterpret_cast<uintptr_t>(p.y);
  if ((xa | wa | ya) & 15) return fail(2, "x, w and y must be 16-byte aligned");
  if ((p.x_shot_stride | p.x_node_stride | p.y_shot_stride | p.y_node_stride) & 7)
    return fail(2, "strides must be multiples of 8 elements");
  if (p.head.head_w && (!p.head.logits || (reinterpret_cast<uintptr_t>(p.head.logits) & 7) ||
                        ((p.head.lg_shot_stride | p.head.lg_node_stride) & 1)))
    return fail(2, "head logits must be 8-byte aligned with even strides");
  return 0;
}

int gmm_tc_make_maps(const GmmProblem& p, GmmMaps* maps) {
  auto enc = get_encode();
  if (!enc) return fail(3, "cuTensorMapEncodeTiled is not available from the CUDA driver");
  {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(p.Ci), static_cast<cuuint64_t>(p.shots),
                          static_cast<cuuint64_t>(p.NS)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(p.x_shot_stride) * 2, static_cast<cuuint64_t>(p.x_node_stride) * 2};
    cuuint32_t box[3] = {kKBlock, static_cast<cuuint32_t>(kBlockM * mt_for(p.Co)), 1};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = enc(&maps->x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(p.x), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(3, "cuTensorMapEncodeTiled(x) failed: " + std::to_string(int(r)));
  }
  {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(p.Ci), static_cast<cuuint64_t>(p.K),
                          static_cast<cuuint64_t>(p.Co) * p.n_wtypes};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(p.Ci) * 2, static_cast<cuuint64_t>(p.K) * p.Ci * 2};
    cuuint32_t box[3] = {kKBlock, 1, static_cast<cuuint32_t>(p.Co)};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = enc(&maps->w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(p.w), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(3, "cuTensorMapEncodeTiled(w) failed: " + std::to_string(int(r)));
  }
  return 0;
}

int gmm_tc_launch(const GmmProblem& p, const GmmMaps& maps, int* status, uint64_t timeout_ns, cudaStream_t stream) {
  if (int e = gmm_tc_check(p)) return e;
  if (p.shots <= 0) return 0;
  TcArgs a;
  a.idx = p.idx;
  a.NT = p.NT;
  a.NS = p.NS;
  a.K = p.K;
  a.Ci = p.Ci;
  a.Co = p.Co;
  a.type_split = p.n_wtypes > 1 ? p.type_split : p.NT;
  a.n_kb = (p.Ci + kKBlock - 1) / kKBlock;
  a.stages = stages_for(p.Co);
  a.shots = p.shots;
  const int64_t tile_m = kBlockM * mt_for(p.Co);
  a.num_tiles = ((p.shots + tile_m - 1) / tile_m) * p.NT;
  a.y = p.y;
  a.y_shot_stride = p.y_shot_stride;
  a.y_node_stride = p.y_node_stride;
  a.epi = p.epi;
  a.head = p.head;
  a.status = status;
  a.timeout_ns = timeout_ns;
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(2 * mt_for(p.Co) * p.Co)) cols <<= 1;
  a.tmem_cols = cols;
  const int smem = smem_bytes_for(p.Co, a.stages);
  KernelFn fn = select_kernel(p.Co);
  if (!fn) return fail(2, "unsupported C_out for the tcgen05 path");
  static bool configured[9] = {false};
  if (!configured[p.Co / 32]) {
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemLimit);
    if (e != cudaSuccess) return fail(4, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    configured[p.Co / 32] = true;
  }
  const int64_t grid = std::min<int64_t>(a.num_tiles, num_sms());
  void* args[] = {const_cast<CUtensorMap*>(&maps.x), const_cast<CUtensorMap*>(&maps.w), &a};
  cudaError_t le = cudaLaunchKernel(reinterpret_cast<const void*>(fn), dim3(static_cast<unsigned>(grid)),
                                    dim3(kThreads), args, static_cast<size_t>(smem), stream);
  if (le != cudaSuccess) return fail(4, std::string("gmm_tc_kernel launch: ") + cudaGetErrorString(le));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(4, std::string("gmm_tc_kernel launch: ") + cudaGetErrorString(e));
  return 0;
}

}  // namespace bpc
