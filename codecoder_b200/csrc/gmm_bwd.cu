// Backward of the bipartite-conv step (the reference's _GatherMM.backward and the Triton gmm(transposed=True) /
// gmm_wgrad pair, training/bb/ising_compare/bb/cascade_triton.py:64-136,173-186).
//
// Input gradient:  gx[b, s] = sum_r gy[b, tgt[s, r]] W_r, with tgt the target table derived from the inverse table.
//   It is the forward with W rearranged as W'(Ci, K Co), W'[i, r Co + o] = W[o, r Ci + i]: one small transpose
//   kernel, then the forward kernels (tensor cores or CUDA cores) unchanged.
// Weight gradient: dW[o, r Ci + i] = sum_{b, n} gy[b, n, o] x[b, idx[n, r], i].
//   Tensor cores (bf16): the reduction runs over rows (shot, target), so both operands are MN-major -- channel
//   contiguous -- exactly as the activations lie in memory.  A TMA box of 128 shots x 64 channels with the 128-byte
//   swizzle is the canonical MN-major SW128 layout, so no operand is transposed anywhere.  Item = one target node
//   x 128 shots; the CTA owns a group of up to 4 relations, keeps one 128 x N fp32 accumulator per relation in
//   tensor memory (4 x 128 columns), loads the item's gy block once and the x block of every non-pad relation of
//   the group, and runs 8 MMAs (K = 16 shots each) per relation.  The CTAs of split s take the items s, s + splits,
//   ... (so all CTAs sweep one window of consecutive items together and share its blocks in L2), write fp32
//   partial sums, and a second kernel adds the splits in a fixed order: deterministic,
//   no atomics (the reference's split-K with a torch sum, cascade_triton.py:120-136).
//   CUDA cores (fp32, or shapes the tensor-core path does not take): 32 x 32 output tiles, rows staged in shared
//   memory, the same partial-sum format and reduction.
#include <algorithm>
#include <cstdio>
#include <string>

#include <cudaTypedefs.h>

#include "bpc.h"
#include "bpc_common.cuh"
#include "bpc_internal.h"

namespace bpc {

namespace {

// ------------------------------------------------------------------------------------------------------------------
// W (Co, K, Ci) -> W' (Ci, K, Co)
template <typename T>
__global__ void transpose_w_kernel(const T* __restrict__ w, T* __restrict__ wt, int K, int Ci, int Co) {
  __shared__ T tile[32][33];
  const int r = blockIdx.z;
  const int o0 = blockIdx.y * 32, i0 = blockIdx.x * 32;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int o = o0 + k, i = i0 + threadIdx.x;
    if (o < Co && i < Ci) tile[k][threadIdx.x] = w[(static_cast<int64_t>(o) * K + r) * Ci + i];
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int i = i0 + k, o = o0 + threadIdx.x;
    if (o < Co && i < Ci) wt[(static_cast<int64_t>(i) * K + r) * Co + o] = tile[threadIdx.x][k];
  }
}

// ------------------------------------------------------------------------------------------------------------------
// Weight gradient on the tensor cores
constexpr int kWgThreads = 192;        // warp 0 producer, warp 1 MMA + TMEM owner, warps 2-5 epilogue
constexpr int kWgShots = 128;          // shots per item = K extent of one item's MMAs (8 x 16)
constexpr int kWgBoxBytes = kWgShots * 128;   // one TMA box: 128 shots x 64 channels bf16
constexpr int kWgMaxRel = 4;           // relations (accumulators) per CTA
constexpr int kWgASlots = 2;
constexpr int kWgBStages = 4;
constexpr int kWgSlotBytes = 2 * kWgBoxBytes;   // up to 128 channels
constexpr int kWgSmem = 1024 + (kWgASlots + kWgBStages) * kWgSlotBytes + 256;

struct WgArgs {
  const int32_t* idx;
  int NT, NS, K, Ci, Co;
  int64_t num_items;          // NT x ceil(B / 128), item = stile * NT + n
  int64_t splits;             // split s takes items s, s + splits, s + 2 splits, ...
  int rg, n_groups, n_otiles, n_itiles;
  int n_abox, n_bbox;         // boxes per A (gy) and B (x) operand
  int n_mma;                  // N of the MMAs (channels of the i tile rounded up to 16)
  uint32_t tmem_cols, acc_cols;
  float* partial;             // (splits, Co, K Ci)
  int* status;
  uint64_t timeout_ns;
};

__device__ __forceinline__ uint32_t group_mask(const WgArgs& a, int n, int r0, int rn, int (&src)[kWgMaxRel]) {
  uint32_t vm = 0;
  const int32_t* row = a.idx + static_cast<int64_t>(n) * a.K + r0;
#pragma unroll
  for (int j = 0; j < kWgMaxRel; ++j) {
    src[j] = j < rn ? __ldg(row + j) : -1;
    if (src[j] >= 0 && src[j] < a.NS) vm |= 1u << j;
  }
  return vm;
}

__global__ void __launch_bounds__(kWgThreads, 1)
    gmm_wgrad_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmG,
                        const WgArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kWgASlots * kWgSlotBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (kWgASlots + kWgBStages) * kWgSlotBytes);
  uint64_t* a_full = bars;
  uint64_t* a_empty = bars + kWgASlots;
  uint64_t* b_full = bars + 2 * kWgASlots;
  uint64_t* b_empty = bars + 2 * kWgASlots + kWgBStages;
  uint64_t* accf = bars + 2 * kWgASlots + 2 * kWgBStages;
  uint64_t* done = accf + 1;            // the MMA thread's `started` mask is published
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile uint32_t* started_s = reinterpret_cast<volatile uint32_t*>(tmem_slot + 2);

  int b = blockIdx.x;
  const int it = b % a.n_itiles;
  b /= a.n_itiles;
  const int ot = b % a.n_otiles;
  b /= a.n_otiles;
  const int g = b % a.n_groups;
  const int split = b / a.n_groups;
  const int r0 = g * a.rg;
  const int rn = min(a.rg, a.K - r0);
  // items split, split + splits, ...: at any time the CTAs of every split work on one window of consecutive items
  // (consecutive target nodes of one shot tile), so the source and gradient blocks they share are read from L2
  const int64_t n_mine = split < a.num_items ? (a.num_items - split + a.splits - 1) / a.splits : 0;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kWgASlots; ++i) {
      mbar_init(smem_u32(&a_full[i]), 1);
      mbar_init(smem_u32(&a_empty[i]), 1);
    }
    for (int i = 0; i < kWgBStages; ++i) {
      mbar_init(smem_u32(&b_full[i]), 1);
      mbar_init(smem_u32(&b_empty[i]), 1);
    }
    mbar_init(smem_u32(accf), 1);
    mbar_init(smem_u32(done), 1);
    *abort_flag = 0;
    *started_s = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmG);
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
    if (lane == 0) {
      // ---------------------------------------------------------------- producer
      int as = 0, bs = 0;
      uint32_t aph = 0, bph = 0;
      uint32_t armed_a = 0, armed_b = 0, par_a = 0, par_b = 0;
      bool ok = true;
      for (int64_t item = split; item < a.num_items && ok; item += a.splits) {
        const int n = static_cast<int>(item % a.NT);
        const int32_t s0 = static_cast<int32_t>((item / a.NT) * kWgShots);
        int src[kWgMaxRel];
        const uint32_t vm = group_mask(a, n, r0, rn, src);
        if (!vm) continue;
        if (!mbar_wait(smem_u32(&a_empty[as]), aph ^ 1u, abort_flag, a.status, a.timeout_ns)) break;
        const uint32_t fa = smem_u32(&a_full[as]);
        mbar_arrive_expect_tx(fa, a.n_abox * kWgBoxBytes);
        for (int j = 0; j < a.n_abox; ++j)
          tma_load_3d(smem_u32(sA + as * kWgSlotBytes + j * kWgBoxBytes), &tmG, ot * 128 + j * 64, s0, n, fa);
        armed_a |= 1u << as;
        par_a = (par_a & ~(1u << as)) | (aph << as);
        if (++as == kWgASlots) {
          as = 0;
          aph ^= 1u;
        }
        for (int j = 0; j < rn; ++j) {
          if (!(vm & (1u << j))) continue;
          if (!mbar_wait(smem_u32(&b_empty[bs]), bph ^ 1u, abort_flag, a.status, a.timeout_ns)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&b_full[bs]);
          mbar_arrive_expect_tx(fb, a.n_bbox * kWgBoxBytes);
          for (int q = 0; q < a.n_bbox; ++q)
            tma_load_3d(smem_u32(sB + bs * kWgSlotBytes + q * kWgBoxBytes), &tmX, it * 128 + q * 64, s0, src[j], fb);
          armed_b |= 1u << bs;
          par_b = (par_b & ~(1u << bs)) | (bph << bs);
          if (++bs == kWgBStages) {
            bs = 0;
            bph ^= 1u;
          }
        }
      }
      if (*abort_flag) {
        // drain: wait (bounded) for the loads in flight before the CTA's shared memory goes away
        const uint64_t t0 = globaltimer_ns();
        for (int i = 0; i < kWgASlots; ++i)
          if (armed_a & (1u << i))
            while (!mbar_try_wait(smem_u32(&a_full[i]), (par_a >> i) & 1u) && globaltimer_ns() - t0 < a.timeout_ns) {
            }
        for (int i = 0; i < kWgBStages; ++i)
          if (armed_b & (1u << i))
            while (!mbar_try_wait(smem_u32(&b_full[i]), (par_b >> i) & 1u) && globaltimer_ns() - t0 < a.timeout_ns) {
            }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      const uint32_t idesc = idesc_bf16_f32_mn(128, a.n_mma);
      int as = 0, bs = 0;
      uint32_t aph = 0, bph = 0;
      uint32_t started = 0;
      bool ok = true;
      for (int64_t item = split; item < a.num_items && ok; item += a.splits) {
        const int n = static_cast<int>(item % a.NT);
        int src[kWgMaxRel];
        const uint32_t vm = group_mask(a, n, r0, rn, src);
        if (!vm) continue;
        if (!mbar_wait(smem_u32(&a_full[as]), aph, abort_flag, a.status, a.timeout_ns)) break;
        tc_fence_after();
        const uint64_t ad = sdesc_mn_sw128(smem_u32(sA + as * kWgSlotBytes), kWgBoxBytes, 1024);
        for (int j = 0; j < rn; ++j) {
          if (!(vm & (1u << j))) continue;
          if (!mbar_wait(smem_u32(&b_full[bs]), bph, abort_flag, a.status, a.timeout_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bd = sdesc_mn_sw128(smem_u32(sB + bs * kWgSlotBytes), kWgBoxBytes, 1024);
          const uint32_t d = tmem_base + j * a.acc_cols;
          const uint32_t acc0 = (started >> j) & 1u;
#pragma unroll
          for (int k = 0; k < kWgShots / 16; ++k) {      // 16 shots = 2 K groups of 8 rows = 2048 bytes
            const uint64_t off = static_cast<uint64_t>((k * 2048) >> 4);
            tc_mma_ss(d, ad + off, bd + off, idesc, (k > 0) ? 1u : acc0);
          }
          started |= 1u << j;
          tc_commit(smem_u32(&b_empty[bs]));
          if (++bs == kWgBStages) {
            bs = 0;
            bph ^= 1u;
          }
        }
        tc_commit(smem_u32(&a_empty[as]));
        if (++as == kWgASlots) {
          as = 0;
          aph ^= 1u;
        }
      }
      *started_s = started;
      mbar_arrive(smem_u32(done));
      tc_commit(smem_u32(accf));             // every MMA of this CTA done: accumulators final
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5): TMEM -> partials
    const int q = warp & 3;
    const int row = q * 32 + lane;            // output channel o within the tile
    const int o = ot * 128 + row;
    // the accumulators are final only when this CTA's whole item range is done: allow 20 us per item on top of the
    // watchdog limit (an item is at most 32 MMAs)
    const uint64_t limit = a.timeout_ns + static_cast<uint64_t>(n_mine) * 20000ull;
    bool ok = mbar_wait(smem_u32(done), 0, abort_flag, a.status, limit);
    ok = ok && mbar_wait(smem_u32(accf), 0, abort_flag, a.status, limit);
    ok = ok && !*abort_flag;
    if (ok) {
      tc_fence_after();
      const uint32_t started = *started_s;
      const int ci_tile = min(128, a.Ci - it * 128);
      const int nch = (ci_tile + 31) / 32;
      for (int j = 0; j < rn; ++j) {
        const int r = r0 + j;
        float* prow = a.partial + (static_cast<int64_t>(split) * a.Co + o) * a.K * a.Ci +
                      static_cast<int64_t>(r) * a.Ci + it * 128;
        for (int c = 0; c < nch; ++c) {
          float v[32];
          if (started & (1u << j)) {
            tmem_ld32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + j * a.acc_cols + c * 32, v);
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = 0.f;
          }
          if (o < a.Co) {
            if (c * 32 + 32 <= ci_tile) {
#pragma unroll
              for (int e = 0; e < 32; e += 4)
                *reinterpret_cast<float4*>(prow + c * 32 + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
            } else {
#pragma unroll
              for (int e = 0; e < 32; ++e)
                if (c * 32 + e < ci_tile) prow[c * 32 + e] = v[e];
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, a.tmem_cols);
  }
}

// ------------------------------------------------------------------------------------------------------------------
// Weight gradient on the CUDA cores: block = (relation, 32 x 32 output tile, split), rows staged 64 at a time.
constexpr int kWfThreads = 256;
constexpr int kWfRows = 64;

struct WfArgs {
  const void* x;
  const void* gy;
  const int32_t* idx;
  int NT, NS, K, Ci, Co;
  int64_t rows;               // B NT
  int64_t rows_per_split;
  int n_ot, n_it;
  float* partial;
};

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__global__ void __launch_bounds__(kWfThreads) gmm_wgrad_fma_kernel(const WfArgs a) {
  __shared__ float gs[kWfRows][33];
  __shared__ float xs[kWfRows][33];
  int b = blockIdx.x;
  const int it = b % a.n_it;
  b /= a.n_it;
  const int ot = b % a.n_ot;
  const int r = b / a.n_ot;
  const int split = blockIdx.y;
  const int t = threadIdx.x;
  const int o_l = t >> 3, i_l = (t & 7) * 4;
  const T* x = static_cast<const T*>(a.x);
  const T* gy = static_cast<const T*>(a.gy);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const int64_t m_begin = split * a.rows_per_split;
  const int64_t m_end = min(a.rows, m_begin + a.rows_per_split);
  for (int64_t m0 = m_begin; m0 < m_end; m0 += kWfRows) {
    __syncthreads();
    for (int e = t; e < kWfRows * 32; e += kWfThreads) {
      const int ml = e >> 5, c = e & 31;
      const int64_t m = m0 + ml;
      float gv = 0.f, xv = 0.f;
      if (m < m_end) {
        const int64_t shot = m / a.NT;
        const int n = static_cast<int>(m - shot * a.NT);
        const int o = ot * 32 + c, i = it * 32 + c;
        if (o < a.Co) gv = to_f(gy[m * a.Co + o]);
        const int src = __ldg(a.idx + static_cast<int64_t>(n) * a.K + r);
        if (src >= 0 && src < a.NS && i < a.Ci) xv = to_f(x[(shot * a.NS + src) * a.Ci + i]);
      }
      gs[ml][c] = gv;
      xs[ml][c] = xv;
    }
    __syncthreads();
#pragma unroll 8
    for (int ml = 0; ml < kWfRows; ++ml) {
      const float gv = gs[ml][o_l];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = fmaf(gv, xs[ml][i_l + j], acc[j]);
    }
  }
  const int o = ot * 32 + o_l;
  if (o < a.Co) {
    float* p = a.partial + (static_cast<int64_t>(split) * a.Co + o) * a.K * a.Ci + static_cast<int64_t>(r) * a.Ci;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = it * 32 + i_l + j;
      if (i < a.Ci) p[i] = acc[j];
    }
  }
}

// dw[j] = sum over splits of partial[split, j], in split order
__global__ void wgrad_reduce_kernel(const float* __restrict__ partial, float* __restrict__ dw, int64_t n, int splits) {
  for (int64_t j = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; j < n;
       j += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < splits; ++k) s += partial[k * n + j];
    dw[j] = s;
  }
}

// ------------------------------------------------------------------------------------------------------------------
// Planning: which path, how many splits (a pure function of the shapes and the device's SM count, so the workspace
// size query and the launch agree).
struct WgPlan {
  bool tc;
  int rg, n_groups, n_otiles, n_itiles, splits;
  int64_t items;                    // tensor-core path
  int n_ot, n_it;                   // CUDA-core path (32 x 32 tiles)
  int64_t rows, rows_per_split;
};

bool wgrad_tc_ok(int64_t B, int32_t K, int32_t Ci, int32_t Co, int32_t dtype) {
  (void)B;
  return dtype == BPC_DTYPE_BF16 && Ci % 16 == 0 && Co % 8 == 0 && Ci >= 16 && Co >= 8 && K >= 1;
}

WgPlan plan_wgrad(int64_t B, int32_t NT, int32_t K, int32_t Ci, int32_t Co, int32_t dtype) {
  WgPlan p{};
  const int sms = num_sms();
  p.tc = wgrad_tc_ok(B, K, Ci, Co, dtype);
  if (p.tc) {
    p.rg = std::min<int>(K, kWgMaxRel);
    p.n_groups = (K + p.rg - 1) / p.rg;
    p.n_otiles = (Co + 127) / 128;
    p.n_itiles = (Ci + 127) / 128;
    p.items = static_cast<int64_t>(NT) * ((B + kWgShots - 1) / kWgShots);
    const int per = p.n_groups * p.n_otiles * p.n_itiles;
    int64_t splits = std::max<int64_t>(1, sms / per);
    splits = std::min<int64_t>(splits, std::max<int64_t>(1, p.items));
    p.splits = static_cast<int>(splits);   // every split has at least one item (splits <= items)
  } else {
    p.n_ot = (Co + 31) / 32;
    p.n_it = (Ci + 31) / 32;
    p.rows = B * static_cast<int64_t>(NT);
    const int64_t tiles = static_cast<int64_t>(K) * p.n_ot * p.n_it;
    int64_t splits = std::max<int64_t>(1, (4 * sms + tiles - 1) / tiles);
    splits = std::min<int64_t>(splits, std::max<int64_t>(1, (p.rows + kWfRows - 1) / kWfRows));
    const int64_t per = (p.rows + splits - 1) / splits;
    p.rows_per_split = std::max<int64_t>(kWfRows, (per + kWfRows - 1) / kWfRows * kWfRows);
    p.splits = static_cast<int>(std::max<int64_t>(1, (p.rows + p.rows_per_split - 1) / p.rows_per_split));
  }
  return p;
}

size_t workspace_for(const WgPlan& p, int32_t K, int32_t Ci, int32_t Co) {
  return static_cast<size_t>(p.splits) * Co * K * Ci * sizeof(float);
}

int make_act_map(CUtensorMap* m, const void* base, int C, int64_t B, int N) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return fail(BPC_ERR_DRIVER, "cuTensorMapEncodeTiled is not available from the CUDA driver");
  // (channel, shot, node) view of a (B, N, C) tensor; box = 64 channels x 128 shots x 1 node, 128-byte swizzle
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(B), static_cast<cuuint64_t>(N)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(N) * C * 2, static_cast<cuuint64_t>(C) * 2};
  cuuint32_t box[3] = {64, kWgShots, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(BPC_ERR_DRIVER, "cuTensorMapEncodeTiled(activations) failed: " + std::to_string(int(r)));
  return 0;
}

}  // namespace

int gmm_wgrad_launch(const void* x, const void* gy, const int32_t* idx, float* dw, void* ws, size_t ws_bytes,
                     int64_t B, int32_t NS, int32_t NT, int32_t K, int32_t Ci, int32_t Co, int32_t dtype,
                     int* status, cudaStream_t stream) {
  const WgPlan p = plan_wgrad(B, NT, K, Ci, Co, dtype);
  const size_t need = workspace_for(p, K, Ci, Co);
  if (ws_bytes < need || (need && !ws)) return fail(BPC_ERR_SPACE, "wgrad workspace too small: need " + std::to_string(need) + " bytes");
  if (reinterpret_cast<uintptr_t>(ws) & 15) return fail(BPC_ERR_ARG, "wgrad workspace must be 16-byte aligned");
  float* partial = static_cast<float*>(ws);
  if (p.tc) {
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(gy)) & 15)
      return fail(BPC_ERR_ARG, "x and gy must be 16-byte aligned");
    CUtensorMap tmX, tmG;
    if (int e = make_act_map(&tmX, x, Ci, B, NS)) return e;
    if (int e = make_act_map(&tmG, gy, Co, B, NT)) return e;
    WgArgs a;
    a.idx = idx;
    a.NT = NT;
    a.NS = NS;
    a.K = K;
    a.Ci = Ci;
    a.Co = Co;
    a.num_items = p.items;
    a.splits = p.splits;
    a.rg = p.rg;
    a.n_groups = p.n_groups;
    a.n_otiles = p.n_otiles;
    a.n_itiles = p.n_itiles;
    const int co_tile = std::min(128, Co);
    const int ci_tile = std::min(128, Ci);
    a.n_abox = (co_tile + 63) / 64;
    a.n_bbox = (ci_tile + 63) / 64;
    a.n_mma = (ci_tile + 15) / 16 * 16;
    a.acc_cols = static_cast<uint32_t>((ci_tile + 31) / 32 * 32);
    uint32_t cols = 32;
    while (cols < a.acc_cols * p.rg) cols <<= 1;
    a.tmem_cols = cols;
    a.partial = partial;
    a.status = status;
    a.timeout_ns = 2000000000ull;
    if (int e = allow_smem(reinterpret_cast<const void*>(&gmm_wgrad_tc_kernel), kWgSmem)) return e;
    const int grid = p.splits * p.n_groups * p.n_otiles * p.n_itiles;
    void* args[] = {&tmX, &tmG, &a};
    cudaError_t le = cudaLaunchKernel(reinterpret_cast<const void*>(&gmm_wgrad_tc_kernel), dim3(grid),
                                      dim3(kWgThreads), args, kWgSmem, stream);
    if (le != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("gmm_wgrad_tc_kernel launch: ") + cudaGetErrorString(le));
  } else {
    WfArgs a;
    a.x = x;
    a.gy = gy;
    a.idx = idx;
    a.NT = NT;
    a.NS = NS;
    a.K = K;
    a.Ci = Ci;
    a.Co = Co;
    a.rows = p.rows;
    a.rows_per_split = p.rows_per_split;
    a.n_ot = p.n_ot;
    a.n_it = p.n_it;
    a.partial = partial;
    const dim3 grid(static_cast<unsigned>(K * p.n_ot * p.n_it), static_cast<unsigned>(p.splits));
    if (dtype == BPC_DTYPE_F32)
      gmm_wgrad_fma_kernel<float><<<grid, kWfThreads, 0, stream>>>(a);
    else
      gmm_wgrad_fma_kernel<__nv_bfloat16><<<grid, kWfThreads, 0, stream>>>(a);
    cudaError_t le = cudaGetLastError();
    if (le != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("gmm_wgrad_fma_kernel launch: ") + cudaGetErrorString(le));
  }
  const int64_t n = static_cast<int64_t>(Co) * K * Ci;
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 4 * num_sms()));
  wgrad_reduce_kernel<<<blocks, 256, 0, stream>>>(partial, dw, n, p.splits);
  cudaError_t le = cudaGetLastError();
  if (le != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("wgrad_reduce_kernel launch: ") + cudaGetErrorString(le));
  return 0;
}

size_t gmm_wgrad_workspace(int64_t B, int32_t NT, int32_t K, int32_t Ci, int32_t Co, int32_t dtype) {
  return workspace_for(plan_wgrad(B, NT, K, Ci, Co, dtype), K, Ci, Co);
}

int transpose_w_launch(const void* w, void* wt, int K, int Ci, int Co, int32_t dtype, cudaStream_t stream) {
  const dim3 grid((Ci + 31) / 32, (Co + 31) / 32, K), block(32, 8);
  if (dtype == BPC_DTYPE_F32)
    transpose_w_kernel<float><<<grid, block, 0, stream>>>(static_cast<const float*>(w), static_cast<float*>(wt), K, Ci, Co);
  else
    transpose_w_kernel<__nv_bfloat16><<<grid, block, 0, stream>>>(static_cast<const __nv_bfloat16*>(w),
                                                                  static_cast<__nv_bfloat16*>(wt), K, Ci, Co);
  cudaError_t le = cudaGetLastError();
  if (le != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("transpose_w_kernel launch: ") + cudaGetErrorString(le));
  return 0;
}

}  // namespace bpc
