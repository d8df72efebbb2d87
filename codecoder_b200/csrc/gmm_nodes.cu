// Bipartite-conv step for small batches (streaming, batch 1): the rows of the MMA are target NODES of one shot.
//
//   y[s, n, :] (op)= sum_r x[s, idx[n, r], :] W_{type(n), r}^T            (same arithmetic as gmm_tc.cu)
//
// The shot-tiled kernel (gmm_tc.cu) makes the MMA rows shots, so at batch 1 each of its tiles carries one valid row
// out of 256 and moves 256 rows' worth of data.  Here a CTA owns 128 target nodes of one shot (a tile never mixes
// the two weight types of a data -> check step): for every relation r its 128 source rows (C bf16 each, 16-byte
// pieces) are gathered with cp.async straight into the 128-byte-swizzled K-major layout, W_r comes by TMA, and one
// thread issues M=128 N=Co K=16 tcgen05 MMAs into a TMEM accumulator.  The relations stream through a ring of
// stages (all 8 in flight at C = 64), each gathering thread owning one row, so the gathers of later relations
// overlap the MMAs of earlier ones.
//
// Bit-compatibility with the shot-tiled kernel: the accumulation runs in the same order (relations ascending, then
// 64-channel blocks, then 16-channel steps), a pad relation contributes exact zeros (its rows are zero-filled)
// instead of being skipped, and the epilogue (GELU, residual add, bf16 rounding, head) is the same sequence of
// packed fp32 operations, so both kernels give the same bits for the same shot.
//
// Roles (160 threads): warps 0-3 gather (thread = row = node) and run the epilogue on TMEM lanes 0-127; warp 4
// allocates TMEM, loads W_r by TMA and issues the MMAs.  Every wait is bounded (mbar_wait); a timeout sets the
// status word and the CTA drains its copies and returns.
#include <algorithm>
#include <string>

#include <cudaTypedefs.h>

#include "bpc.h"
#include "bpc_common.cuh"
#include "bpc_internal.h"

namespace bpc {

namespace {

constexpr int kNodeThreads = 160;
constexpr int kNodeRows = 128;
constexpr int kNodeMaxK = 16;
constexpr int kNodeSmemLimit = 232448;

struct NodeArgs {
  const __nv_bfloat16* x;
  int64_t x_shot_stride, x_node_stride;   // elements; channels contiguous
  const int32_t* idx;
  int NT, NS, K, type_split;
  int tiles_a, tiles;                     // tiles of type 0 (targets < type_split), all tiles of one shot
  __nv_bfloat16* y;
  int64_t y_shot_stride, y_node_stride;
  HeadEpilogue head;
  int stages;
  int* status;
  uint64_t timeout_ns;
  uint32_t tmem_cols;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(reinterpret_cast<uint64_t>(src)),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// wait until at most n (runtime, 0..7) of this thread's cp.async groups are pending
__device__ __forceinline__ void cp_async_wait_n(int n) {
  switch (n) {
    case 0: cp_async_wait<0>(); break;
    case 1: cp_async_wait<1>(); break;
    case 2: cp_async_wait<2>(); break;
    case 3: cp_async_wait<3>(); break;
    case 4: cp_async_wait<4>(); break;
    case 5: cp_async_wait<5>(); break;
    case 6: cp_async_wait<6>(); break;
    default: cp_async_wait<7>(); break;
  }
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <int NKB, int NCH, int EPI, bool HEAD>
__global__ void __launch_bounds__(kNodeThreads, 1)
    gmm_nodes_kernel(const __grid_constant__ CUtensorMap tmW, const NodeArgs a) {
  constexpr int Co = NCH * 32;
  constexpr uint32_t kABytes = NKB * kNodeRows * 128;   // 128 rows x Ci channels, 64-channel blocks
  constexpr uint32_t kWBytes = NKB * Co * 128;          // Co rows x Ci channels of W_r
  constexpr uint32_t kStageBytes = kABytes + kWBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * kStageBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* accf = bars + 2 * S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int64_t shot = blockIdx.y;
  const bool second = tile >= a.tiles_a;
  const int n_begin = second ? a.type_split + (tile - a.tiles_a) * kNodeRows : tile * kNodeRows;
  const int n_end = second ? a.NT : min(a.type_split, n_begin + kNodeRows);

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(smem_u32(&full[i]), kNodeRows + 1);   // one arrival per gathering thread + the W expect_tx
      mbar_init(smem_u32(&empty[i]), 1);
    }
    mbar_init(smem_u32(accf), 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmW);
  }
  if (warp == 4) {
    tmem_alloc(smem_u32(tmem_slot), a.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < 4) {
    // ---------------------------------------------------------------- gather: thread m owns row m (node n_begin+m)
    const int m = threadIdx.x;
    const int n = n_begin + m;
    const bool row_ok = n < n_end;
    const int32_t* irow = a.idx + static_cast<int64_t>(row_ok ? n : 0) * a.K;
    int src[kNodeMaxK];
#pragma unroll
    for (int r = 0; r < kNodeMaxK; ++r) src[r] = (row_ok && r < a.K) ? __ldg(irow + r) : -1;
    const __nv_bfloat16* xs = a.x + shot * a.x_shot_stride;
    bool ok = true;
    int pending = 0;                 // committed copy groups whose relation has not been arrived for yet
    int arrive_r = 0;                // the oldest such relation
    for (int r = 0; r < a.K; ++r) {
      const int stage = r % S;
      if (r >= S) {
        // the stage is free again once the MMAs of relation r - S have read it
        if (!mbar_wait(smem_u32(&empty[stage]), ((r / S) - 1) & 1u, abort_flag, a.status, a.timeout_ns)) {
          ok = false;
          break;
        }
      }
      const bool valid = src[r] >= 0 && src[r] < a.NS;
      const __nv_bfloat16* xr = xs + static_cast<int64_t>(valid ? src[r] : 0) * a.x_node_stride;
      const uint32_t sa = smem_u32(smem + stage * kStageBytes) + m * 128;
#pragma unroll
      for (int kb = 0; kb < NKB; ++kb)
#pragma unroll
        for (int j = 0; j < 8; ++j)   // 16-byte piece j of the row -> swizzled position j ^ (m % 8)
          cp_async16(sa + kb * (kNodeRows * 128) + ((j ^ (m & 7)) << 4), xr + kb * 64 + j * 8, valid ? 16u : 0u);
      cp_async_commit();
      if (++pending == S) {
        // every stage holds copies in flight: hand over the oldest relation once its copies have landed
        cp_async_wait_n(S - 1);
        fence_proxy_async_smem();       // the tensor cores read what the generic proxy wrote
        mbar_arrive(smem_u32(&full[arrive_r % S]));
        ++arrive_r;
        --pending;
      }
    }
    while (ok && pending > 0) {
      cp_async_wait_n(pending - 1);
      fence_proxy_async_smem();
      mbar_arrive(smem_u32(&full[arrive_r % S]));
      ++arrive_r;
      --pending;
    }
    if (!ok) cp_async_wait<0>();        // nothing may land in shared memory after the CTA leaves

    // ---------------------------------------------------------------- epilogue: thread m = TMEM lane m = node n
    if (ok && mbar_wait(smem_u32(accf), 0, abort_flag, a.status, a.timeout_ns)) {
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(warp * 32) << 16);
      __nv_bfloat16* yrow = a.y + shot * a.y_shot_stride + static_cast<int64_t>(row_ok ? n : 0) * a.y_node_stride;
      uint64_t lg0 = 0, lg1 = 0;
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        float v[32];
        tmem_ld32(taddr + c * 32, v);
        if (row_ok) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4 u;
            uint32_t* o = reinterpret_cast<uint32_t*>(&u);
            uint4 cur = make_uint4(0, 0, 0, 0);
            if (EPI == kEpiGeluResid) cur = *reinterpret_cast<const uint4*>(yrow + (4 * c + j) * 8);
            const uint32_t* hres = reinterpret_cast<const uint32_t*>(&cur);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              uint64_t xv = f2_pack(v[j * 8 + 2 * e], v[j * 8 + 2 * e + 1]);
              if (EPI != kEpiStore) xv = gelu_tanh_fast2(xv);
              if (EPI == kEpiGeluResid) xv = f2_add(xv, bf2_to_f2(hres[e]));
              o[e] = f2_to_bf2(xv);
              if (HEAD) {
                const uint64_t f = bf2_to_f2(o[e]);
                const int col = c * 32 + j * 8 + 2 * e;
                lg0 = f2_fma(f, *reinterpret_cast<const uint64_t*>(a.head.head_w + col), lg0);
                lg1 = f2_fma(f, *reinterpret_cast<const uint64_t*>(a.head.head_w + Co + col), lg1);
              }
            }
            *reinterpret_cast<uint4*>(yrow + (4 * c + j) * 8) = u;
          }
        }
      }
      if (HEAD && row_ok) {
        const float l0 = f2_lo(lg0) + f2_hi(lg0) + __ldg(a.head.head_b);
        const float l1 = f2_lo(lg1) + f2_hi(lg1) + __ldg(a.head.head_b + 1);
        float2* lp = reinterpret_cast<float2*>(a.head.logits + shot * a.head.lg_shot_stride +
                                               static_cast<int64_t>(n) * a.head.lg_node_stride);
        *lp = make_float2(l0, l1);
        if (a.head.res_bits) {
          const uint32_t bit = 1u << (shot & 31);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const bool flip = (k >> 1) ? (l1 > 0.f) : (l0 > 0.f);
            const int32_t cidx = __ldg(a.head.xor_nbr + static_cast<int64_t>(n) * 4 + k);
            if (flip && cidx >= 0)
              atomicXor(a.head.res_bits + static_cast<int64_t>(cidx) * a.head.res_words + (shot >> 5), bit);
          }
        }
      }
    }
  } else if (lane == 0) {
    // ---------------------------------------------------------------- W loads and MMAs (warp 4, one thread)
    const uint32_t idesc = idesc_bf16_f32(kNodeRows, Co);
    const int wrow = second ? Co : 0;
    bool ok = true;
    // W of the first min(S, K) relations, then one more per freed stage
    int w_next = 0;
    auto load_w = [&](int r) {
      const int stage = r % S;
      const uint32_t fb = smem_u32(&full[stage]);
      mbar_arrive_expect_tx(fb, kWBytes);
      const uint32_t sw = smem_u32(smem + stage * kStageBytes + kABytes);
#pragma unroll
      for (int kb = 0; kb < NKB; ++kb) tma_load_3d(sw + kb * (Co * 128), &tmW, kb * 64, r, wrow, fb);
    };
    for (; w_next < a.K && w_next < S; ++w_next) load_w(w_next);
    uint32_t armed = 0;
    for (int r = 0; r < a.K && ok; ++r) {
      const int stage = r % S;
      if (!mbar_wait(smem_u32(&full[stage]), (r / S) & 1u, abort_flag, a.status, a.timeout_ns)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sa = smem_u32(smem + stage * kStageBytes);
#pragma unroll
      for (int kb = 0; kb < NKB; ++kb) {
        const uint64_t ad = sdesc_k_sw128(sa + kb * (kNodeRows * 128));
        const uint64_t bd = sdesc_k_sw128(sa + kABytes + kb * (Co * 128));
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma_ss(tmem_base, ad + ((k * 32) >> 4), bd + ((k * 32) >> 4), idesc, (r | kb | k) ? 1u : 0u);
      }
      tc_commit(smem_u32(&empty[stage]));
      if (w_next < a.K) {
        // the stage of relation w_next = r + S is the one these MMAs read: refill it once they are done
        if (!mbar_wait(smem_u32(&empty[stage]), (r / S) & 1u, abort_flag, a.status, a.timeout_ns)) {
          ok = false;
          break;
        }
        load_w(w_next);
        armed |= 1u << stage;
        ++w_next;
      }
    }
    tc_commit(smem_u32(accf));
    if (!ok) {
      // bounded drain of the W loads in flight before the CTA leaves
      const uint64_t t0 = globaltimer_ns();
      for (int i = 0; i < S; ++i)
        while (!mbar_try_wait(smem_u32(&full[i]), 0) && !mbar_try_wait(smem_u32(&full[i]), 1) &&
               globaltimer_ns() - t0 < a.timeout_ns) {
        }
      (void)armed;
    }
    // every MMA must be done before TMEM is released
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(smem_u32(accf), 0) && globaltimer_ns() - t0 < a.timeout_ns) {
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem_base, a.tmem_cols);
  }
}

using NodeFn = void (*)(CUtensorMap, NodeArgs);

template <int NKB, int NCH>
NodeFn node_kernel_for(int epi, bool head) {
  if (epi == kEpiStore) return head ? nullptr : &gmm_nodes_kernel<NKB, NCH, kEpiStore, false>;
  if (epi == kEpiGeluInit)
    return head ? &gmm_nodes_kernel<NKB, NCH, kEpiGeluInit, true> : &gmm_nodes_kernel<NKB, NCH, kEpiGeluInit, false>;
  if (epi == kEpiGeluResid)
    return head ? &gmm_nodes_kernel<NKB, NCH, kEpiGeluResid, true>
                : &gmm_nodes_kernel<NKB, NCH, kEpiGeluResid, false>;
  return nullptr;
}

NodeFn select_node_kernel(int Ci, int Co, int epi, bool head) {
  const int nkb = Ci / 64;
  if (nkb == 1) {
    switch (Co) {
      case 64: return node_kernel_for<1, 2>(epi, head);
      case 128: return node_kernel_for<1, 4>(epi, head);
    }
  } else if (nkb == 2) {
    switch (Co) {
      case 64: return node_kernel_for<2, 2>(epi, head);
      case 128: return node_kernel_for<2, 4>(epi, head);
    }
  }
  return nullptr;
}

}  // namespace

bool gmm_nodes_supported(const GmmProblem& p) {
  return (p.Ci == 64 || p.Ci == 128) && (p.Co == 64 || p.Co == 128) && p.K >= 1 && p.K <= kNodeMaxK &&
         !p.blocked && p.x_cg_stride == 8 && p.y_cg_stride == 8 && p.n_wtypes >= 1 && p.n_wtypes <= 2;
}

int gmm_nodes_launch(const GmmProblem& p, int* status, uint64_t timeout_ns, cudaStream_t stream) {
  if (!gmm_nodes_supported(p)) return fail(BPC_ERR_ARG, "node-tiled path: unsupported shape or layout");
  if (p.shots <= 0 || p.NT <= 0) return 0;
  if (p.shots > 65535) return fail(BPC_ERR_ARG, "node-tiled path: at most 65535 shots per launch");
  const uintptr_t xa = reinterpret_cast<uintptr_t>(p.x), ya = reinterpret_cast<uintptr_t>(p.y),
                  wa = reinterpret_cast<uintptr_t>(p.w);
  if ((xa | ya | wa) & 15) return fail(BPC_ERR_ARG, "x, w and y must be 16-byte aligned");
  if ((p.x_shot_stride | p.x_node_stride | p.y_shot_stride | p.y_node_stride) & 7)
    return fail(BPC_ERR_ARG, "strides must be multiples of 8 elements");
  if (p.head.head_w && (!p.head.logits || (reinterpret_cast<uintptr_t>(p.head.logits) & 7) ||
                        ((p.head.lg_shot_stride | p.head.lg_node_stride) & 1)))
    return fail(BPC_ERR_ARG, "head logits must be 8-byte aligned with even strides");
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return fail(BPC_ERR_DRIVER, "cuTensorMapEncodeTiled is not available from the CUDA driver");
  CUtensorMap tmW;
  {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(p.Ci), static_cast<cuuint64_t>(p.K),
                          static_cast<cuuint64_t>(p.Co) * p.n_wtypes};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(p.Ci) * 2, static_cast<cuuint64_t>(p.K) * p.Ci * 2};
    cuuint32_t box[3] = {64, 1, static_cast<cuuint32_t>(p.Co)};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = enc(&tmW, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(p.w), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(BPC_ERR_DRIVER, "cuTensorMapEncodeTiled(w) failed: " + std::to_string(int(r)));
  }
  NodeArgs a;
  a.x = static_cast<const __nv_bfloat16*>(p.x);
  a.x_shot_stride = p.x_shot_stride;
  a.x_node_stride = p.x_node_stride;
  a.idx = p.idx;
  a.NT = p.NT;
  a.NS = p.NS;
  a.K = p.K;
  a.type_split = p.n_wtypes > 1 ? p.type_split : p.NT;
  a.tiles_a = (a.type_split + kNodeRows - 1) / kNodeRows;
  a.tiles = a.tiles_a + (p.NT - a.type_split + kNodeRows - 1) / kNodeRows;
  a.y = static_cast<__nv_bfloat16*>(p.y);
  a.y_shot_stride = p.y_shot_stride;
  a.y_node_stride = p.y_node_stride;
  a.head = p.head;
  a.status = status;
  a.timeout_ns = timeout_ns;
  a.tmem_cols = p.Co <= 32 ? 32 : (p.Co <= 64 ? 64 : (p.Co <= 128 ? 128 : 256));
  const int nkb = p.Ci / 64;
  const int stage_bytes = nkb * kNodeRows * 128 + nkb * p.Co * 128;
  int stages = std::min(p.K, 8);
  while (stages > 1 && 1024 + stages * stage_bytes + (2 * stages + 1) * 8 + 16 > kNodeSmemLimit) --stages;
  a.stages = stages;
  const int smem = 1024 + stages * stage_bytes + (2 * stages + 1) * 8 + 16;
  NodeFn fn = select_node_kernel(p.Ci, p.Co, p.epi, p.head.head_w != nullptr);
  if (!fn) return fail(BPC_ERR_ARG, "node-tiled path: unsupported epilogue");
  if (int e = allow_smem(reinterpret_cast<const void*>(fn), kNodeSmemLimit)) return e;
  void* args[] = {&tmW, &a};
  cudaError_t le = cudaLaunchKernel(reinterpret_cast<const void*>(fn), dim3(a.tiles, static_cast<unsigned>(p.shots)),
                                    dim3(kNodeThreads), args, static_cast<size_t>(smem), stream);
  if (le != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("gmm_nodes_kernel launch: ") + cudaGetErrorString(le));
  return 0;
}

}  // namespace bpc
