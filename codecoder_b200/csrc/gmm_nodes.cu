// Bipartite-conv step for small batches (streaming, batch 1): the rows of the MMA are target NODES of one shot.
//
//   y[s, n, :] (op)= sum_r x[s, idx[n, r], :] W_{type(n), r}^T            (same arithmetic as gmm_tc.cu)
//
// The shot-tiled kernel (gmm_tc.cu) makes the MMA rows shots, so at batch 1 each of its tiles carries one valid row
// out of 256 and moves 256 rows' worth of data.  Here a CTA owns 128 target nodes of one shot (a tile never mixes
// the two weight types of a data -> check step): for every relation r its 128 source rows are gathered by TMA
// (tile::gather4, 4 rows per instruction, one-row boxes of 64 channels) straight into the 128-byte-swizzled K-major
// layout, W_r comes by TMA, and one thread issues M=128 N=Co K=16 tcgen05 MMAs into a TMEM accumulator.  The relations stream through a ring of
// stages (all 8 in flight at C = 64), so the gathers of later relations overlap the MMAs of earlier ones.
//
// Bit-compatibility with the shot-tiled kernel: the accumulation runs in the same order (relations ascending, then
// 64-channel blocks, then 16-channel steps), a pad relation contributes exact zeros (its rows are zero-filled)
// instead of being skipped, and the epilogue (GELU, residual add, bf16 rounding, head) is the same sequence of
// packed fp32 operations, so both kernels give the same bits for the same shot.
//
// Roles (160 threads): warps 0-3 issue the gathers for their 32 rows (the tile's index rows are staged in shared
// memory first; the residual rows of the tile come by the same 4-row gathers) and run the epilogue (thread = TMEM
// lane = target node, outputs staged in shared memory and stored 4 whole rows per warp instruction); warp 4
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
  int64_t x_row_node, x_row_shot;         // the same strides in rows of the x tensor map (strides / Ci)
  int64_t y_row_node, y_row_shot;         // ... and of the residual map (strides / Co)
  int32_t x_rows, y_rows;                 // rows of the two tensor maps (a row index >= rows reads zeros)
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

// barrier among the first `count` threads (warps 0-3) only
__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
// Byte offset of 16-byte chunk j (channels 8j .. 8j + 7) of row `row` in the staging buffer: blocks of 64 channels,
// 128 rows x 128 bytes each, chunks XOR-swizzled by row % 8 (the 128-byte TMA swizzle, so the residual gathers land
// in it directly, and 32 threads touching chunk j of 32 rows spread over all banks).
__device__ __forceinline__ uint32_t out_off(int j, int row) {
  return static_cast<uint32_t>((j >> 3) * (kNodeRows * 128) + row * 128 + (((j & 7) ^ (row & 7)) << 4));
}

template <int NKB, int NCH, int EPI, bool HEAD>
__global__ void __launch_bounds__(kNodeThreads, 1)
    gmm_nodes_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                     const __grid_constant__ CUtensorMap tmY, const NodeArgs a) {
  constexpr int Co = NCH * 32;
  constexpr uint32_t kABytes = NKB * kNodeRows * 128;   // 128 rows x Ci channels, 64-channel blocks
  constexpr uint32_t kWBytes = NKB * Co * 128;          // Co rows x Ci channels of W_r
  constexpr uint32_t kStageBytes = kABytes + kWBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  constexpr uint32_t kOutBytes = kNodeRows * Co * 2;   // staging: residual in, output out
  uint8_t* sout = smem + S * kStageBytes;                                     // 1024-byte aligned
  int32_t* sidx = reinterpret_cast<int32_t*>(sout + kOutBytes);               // the tile's index rows
  uint64_t* bars = reinterpret_cast<uint64_t*>(sout + kOutBytes + ((kNodeRows * a.K * 4 + 15) & ~15));
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* accf = bars + 2 * S;
  uint64_t* resb = bars + 2 * S + 1;                    // residual rows landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int64_t shot = blockIdx.y;
  const bool second = tile >= a.tiles_a;
  const int n_begin = second ? a.type_split + (tile - a.tiles_a) * kNodeRows : tile * kNodeRows;
  const int n_end = second ? a.NT : min(a.type_split, n_begin + kNodeRows);
  pdl_launch_dependents();

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(smem_u32(&full[i]), 4 + 1);   // one expect_tx arrival per gathering warp + the W loader's
      mbar_init(smem_u32(&empty[i]), 1);
    }
    mbar_init(smem_u32(accf), 1);
    mbar_init(smem_u32(resb), 4);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
    if (EPI == kEpiGeluResid) tma_prefetch_desc(&tmY);
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
    // ---------------------------------------------------------------- gather by TMA: warp w owns rows 32w .. 32w + 31;
    // lane i computes the tensor-map row of row 32w + i, and lanes 0, 4, .., 28 each issue one 4-row gather per
    // 64-channel block, straight into the 128-byte-swizzled K-major layout (a pad row index reads zeros)
    const int t = threadIdx.x;
    for (int e = t; e < kNodeRows * a.K; e += kNodeRows) {
      const int n = n_begin + e / a.K;
      sidx[e] = n < n_end ? __ldg(a.idx + static_cast<int64_t>(n_begin) * a.K + e) : -1;
    }
    named_bar_sync(1, kNodeRows);
    pdl_wait();                           // the activations are the previous kernels' outputs
    const int row = t;                    // = 32 warp + lane
    const int q4 = lane & ~3;             // first row (within the warp) of this lane's 4-row group
    bool ok = true;
    if (EPI == kEpiGeluResid) {
      const int n = n_begin + row;
      const int32_t yr = n < n_end ? static_cast<int32_t>(n * a.y_row_node + shot * a.y_row_shot) : a.y_rows;
      const int32_t i0 = __shfl_sync(0xffffffffu, yr, q4), i1 = __shfl_sync(0xffffffffu, yr, q4 + 1),
                    i2 = __shfl_sync(0xffffffffu, yr, q4 + 2), i3 = __shfl_sync(0xffffffffu, yr, q4 + 3);
      if (lane == 0) mbar_arrive_expect_tx(smem_u32(resb), 32 * Co * 2);
      __syncwarp();
      if ((lane & 3) == 0)
#pragma unroll
        for (int h = 0; h < NCH / 2; ++h)
          tma_gather4(smem_u32(sout + h * (kNodeRows * 128) + (warp * 32 + lane) * 128), &tmY, h * 64, i0, i1, i2, i3,
                      smem_u32(resb));
    }
    for (int r = 0; r < a.K; ++r) {
      const int stage = r % S;
      if (r >= S) {
        // the stage is free again once the MMAs of relation r - S have read it (lane 0 waits for the warp)
        bool free_ok = true;
        if (lane == 0)
          free_ok = mbar_wait(smem_u32(&empty[stage]), ((r / S) - 1) & 1u, abort_flag, a.status, a.timeout_ns);
        if (!__shfl_sync(0xffffffffu, free_ok ? 1 : 0, 0)) {
          ok = false;
          break;
        }
      }
      const int src = sidx[row * a.K + r];
      const int32_t xr = (src >= 0 && src < a.NS) ? static_cast<int32_t>(src * a.x_row_node + shot * a.x_row_shot)
                                                  : a.x_rows;
      const int32_t i0 = __shfl_sync(0xffffffffu, xr, q4), i1 = __shfl_sync(0xffffffffu, xr, q4 + 1),
                    i2 = __shfl_sync(0xffffffffu, xr, q4 + 2), i3 = __shfl_sync(0xffffffffu, xr, q4 + 3);
      const uint32_t fb = smem_u32(&full[stage]);
      if (lane == 0) mbar_arrive_expect_tx(fb, 32 * 128 * NKB);
      __syncwarp();
      if ((lane & 3) == 0) {
        const uint32_t sa = smem_u32(smem + stage * kStageBytes) + (warp * 32 + lane) * 128;
#pragma unroll
        for (int kb = 0; kb < NKB; ++kb) tma_gather4(sa + kb * (kNodeRows * 128), &tmX, kb * 64, i0, i1, i2, i3, fb);
      }
    }
    if (!ok) {
      // bounded drain of this warp's gathers in flight before the CTA leaves
      const uint64_t t0 = globaltimer_ns();
      for (int i = 0; i < S; ++i)
        while (!mbar_try_wait(smem_u32(&full[i]), 0) && !mbar_try_wait(smem_u32(&full[i]), 1) &&
               globaltimer_ns() - t0 < a.timeout_ns) {
        }
      if (EPI == kEpiGeluResid)
        while (!mbar_try_wait(smem_u32(resb), 0) && globaltimer_ns() - t0 < a.timeout_ns) {
        }
    }

    // ---------------------------------------------------------------- epilogue: thread m = TMEM lane m = node n
    bool acc_ok = ok && mbar_wait(smem_u32(accf), 0, abort_flag, a.status, a.timeout_ns);
    if (EPI == kEpiGeluResid && ok) acc_ok = mbar_wait(smem_u32(resb), 0, abort_flag, a.status, a.timeout_ns) && acc_ok;
    if (acc_ok) {
      tc_fence_after();
      const int m = t;
      const int n = n_begin + m;
      const bool row_ok = n < n_end;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(warp * 32) << 16);
      uint64_t lg0 = 0, lg1 = 0;
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        float v[32];
        tmem_ld32(taddr + c * 32, v);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4* slot = reinterpret_cast<uint4*>(sout + out_off(4 * c + j, m));
          uint4 u;
          uint32_t* o = reinterpret_cast<uint32_t*>(&u);
          uint4 cur = make_uint4(0, 0, 0, 0);
          if (EPI == kEpiGeluResid) cur = *slot;
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
          *slot = u;
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
    named_bar_sync(1, kNodeRows);       // every output row is in the staging buffer
    if (acc_ok) {
      // coalesced store: each warp instruction writes 4 whole rows
      __nv_bfloat16* yw = a.y + shot * a.y_shot_stride;
#pragma unroll
      for (int i = 0; i < NCH * 4; ++i) {
        const int p = t + kNodeRows * i;            // block p / 1024, row (p / 8) % 128, chunk p % 8
        const int h = p >> 10, q = p & 1023;
        const int orow = q >> 3, j = h * 8 + (q & 7);
        const int n = n_begin + orow;
        if (n < n_end)
          *reinterpret_cast<uint4*>(yw + n * a.y_node_stride + j * 8) =
              *reinterpret_cast<const uint4*>(sout + out_off(j, orow));
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


// ------------------------------------------------------------------------------------------------------------------
// Relation-split variant for C_in = C_out = 64 and K = 8 (the streaming workload).  One TMA engine moves only a few
// tens of bytes per cycle of scattered 128-byte rows, so the single-CTA tile above spends most of its time pulling
// 128 KB of gathered rows and 64 KB of W through one SM while the other SMs idle.  Here a cluster of 8 CTAs shares
// a 128-node tile: CTA r gathers only relation r's 128 source rows (16 KB) and W_r (8 KB) and runs 4 MMAs into its
// own TMEM accumulator.  Each thread (one accumulator row) writes its fp32 row into a local staging block per
// owner CTA (CTA j owns rows 16 j .. 16 j + 15); one thread then sends block j to slot r of CTA j's receive buffer
// with a bulk shared -> distributed-shared copy whose bytes complete on CTA j's mbarrier.  The owner waits for its
// 8 slots and adds them in relation order (fixed, so the result is deterministic; the same sum as the single-CTA
// kernel's up to the association of the fp32 additions).  The only cluster barrier publishes the mbarrier
// initialisation and is waited for after the loads have been issued; a CTA leaves only after its 8 slots have
// arrived and its own outgoing copies have been read.
constexpr int kSplitThreads = 128;
constexpr int kSplitK = 8;


template <int EPI, bool HEAD>
__global__ void __launch_bounds__(kSplitThreads, 1)
    gmm_nodes_split_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                           const NodeArgs a) {
  constexpr int C = 64;
  constexpr uint32_t kA = kNodeRows * 128;      // relation r's 128 source rows, 128-byte-swizzled K-major
  constexpr uint32_t kW = C * 128;              // W_r
  constexpr uint32_t kR = kSplitK * 16 * C * 4; // receive buffer: 8 slots x 16 rows x 64 fp32 (slot = relation)
  constexpr uint32_t kSlot = 16 * C * 4;        // one slot = one owner's block of the outgoing partial
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sW = smem + kA;
  uint8_t* sR = smem + kA + kW;
  uint8_t* sO = smem + kA + kW + kR;            // outgoing partial, block j = rows 16 j .. 16 j + 15
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kA + kW + 2 * kR);
  uint64_t* full = bars;
  uint64_t* accf = bars + 1;
  uint64_t* recv = bars + 2;                    // the 8 incoming slots (bytes)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31;
  pdl_launch_dependents();
  const int r = static_cast<int>(cluster_ctarank());
  const int tile = blockIdx.x / kSplitK;
  const int64_t shot = blockIdx.y;
  const bool second = tile >= a.tiles_a;
  const int n_begin = second ? a.type_split + (tile - a.tiles_a) * kNodeRows : tile * kNodeRows;
  const int n_end = second ? a.NT : min(a.type_split, n_begin + kNodeRows);
  // the index of this thread's gather row and the residual of its output slice are loaded first
  const int n_src = n_begin + t;
  const int src = n_src < n_end ? __ldg(a.idx + static_cast<int64_t>(n_src) * a.K + r) : -1;
  const int orow = t >> 3;                      // output row 16 r + orow, channels 8 (t % 8) .. + 7
  const int on = n_begin + r * 16 + orow;
  const bool o_ok = on < n_end;

  if (t == 0) {
    mbar_init(smem_u32(full), 4 + 1);          // one expect_tx arrival per gathering warp + W_r's
    mbar_init(smem_u32(accf), 1);
    mbar_init(smem_u32(recv), 1);
    mbar_arrive_expect_tx(smem_u32(recv), kR);  // before any peer can send (the cluster barrier comes after)
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), 64);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  cluster_arrive_release();                     // this CTA's mbarriers are initialised (waited for before pushing)
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (t == 0) {
    mbar_arrive_expect_tx(smem_u32(full), kW);
    tma_load_3d(smem_u32(sW), &tmW, 0, r, second ? C : 0, smem_u32(full));
  }
  pdl_wait();                                   // the activations are the previous kernels' outputs
  uint4 res = make_uint4(0, 0, 0, 0);
  if (EPI == kEpiGeluResid && o_ok)
    res = *reinterpret_cast<const uint4*>(a.y + shot * a.y_shot_stride + static_cast<int64_t>(on) * a.y_node_stride +
                                          (t & 7) * 8);
  {
    // relation r's source rows, 4 per TMA gather (lanes 0, 4, .., 28 of every warp), pads read zeros
    const int32_t xr = (src >= 0 && src < a.NS) ? static_cast<int32_t>(src * a.x_row_node + shot * a.x_row_shot)
                                                : a.x_rows;
    const int q4 = lane & ~3;
    const int32_t i0 = __shfl_sync(0xffffffffu, xr, q4), i1 = __shfl_sync(0xffffffffu, xr, q4 + 1),
                  i2 = __shfl_sync(0xffffffffu, xr, q4 + 2), i3 = __shfl_sync(0xffffffffu, xr, q4 + 3);
    if (lane == 0) mbar_arrive_expect_tx(smem_u32(full), 32 * 128);
    __syncwarp();
    if ((lane & 3) == 0) tma_gather4(smem_u32(sA + t * 128), &tmX, 0, i0, i1, i2, i3, smem_u32(full));
  }
  bool loads_ok = true;
  if (t == 0) {
    loads_ok = mbar_wait(smem_u32(full), 0, abort_flag, a.status, a.timeout_ns);
    if (loads_ok) {
      tc_fence_after();
      const uint64_t ad = sdesc_k_sw128(smem_u32(sA));
      const uint64_t bd = sdesc_k_sw128(smem_u32(sW));
      const uint32_t idesc = idesc_bf16_f32(kNodeRows, C);
#pragma unroll
      for (int k = 0; k < 4; ++k) tc_mma_ss(tmem_base, ad + ((k * 32) >> 4), bd + ((k * 32) >> 4), idesc, k ? 1u : 0u);
    }
    tc_commit(smem_u32(accf));
  }
  cluster_wait_acquire();                       // every CTA of the cluster has initialised its mbarriers
  // accumulator row t (TMEM lane t) -> row t % 16 of outgoing block t / 16; then block j -> slot r of CTA j
  const bool acc_ok = mbar_wait(smem_u32(accf), 0, abort_flag, a.status, a.timeout_ns) && !*abort_flag;
  if (acc_ok) {
    tc_fence_after();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float v[32];
      tmem_ld32(tmem_base + (static_cast<uint32_t>(warp * 32) << 16) + h * 32, v);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        *reinterpret_cast<float4*>(sO + recv_off(t >> 4, t & 15, h * 8 + q)) =
            make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
  }
  fence_proxy_async_smem();                     // the bulk copies read what these stores wrote
  __syncthreads();
  if (t == 0) {
#pragma unroll 1
    for (int j = 0; j < kSplitK; ++j)           // (sent even after a failure, so that no peer waits in vain)
      bulk_s2cluster(map_to_cta(smem_u32(sR + r * kSlot), j), smem_u32(sO + j * kSlot), kSlot,
                     map_to_cta(smem_u32(recv), j));
    bulk_commit();
  }
  // the 8 relations' partials of this CTA's 16 rows, added in relation order
  bool recv_ok = true;
  {
    const uint32_t rb = smem_u32(recv);
    if (!mbar_try_wait_cluster(rb, 0)) {
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait_cluster(rb, 0)) {
        if (globaltimer_ns() - t0 > a.timeout_ns) {
          recv_ok = false;
          if (a.status) atomicExch(a.status, kStatusTimeout);
          break;
        }
      }
    }
  }
  float sum[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) sum[e] = 0.f;
#pragma unroll
  for (int j = 0; j < kSplitK; ++j)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float4 v = *reinterpret_cast<const float4*>(sR + recv_off(j, orow, 2 * (t & 7) + h));
      sum[4 * h] += v.x;
      sum[4 * h + 1] += v.y;
      sum[4 * h + 2] += v.z;
      sum[4 * h + 3] += v.w;
    }
  uint64_t lg0 = 0, lg1 = 0;
  if (o_ok && recv_ok) {
    uint4 u;
    uint32_t* o = reinterpret_cast<uint32_t*>(&u);
    const uint32_t* hres = reinterpret_cast<const uint32_t*>(&res);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      uint64_t xv = f2_pack(sum[2 * e], sum[2 * e + 1]);
      if (EPI != kEpiStore) xv = gelu_tanh_fast2(xv);
      if (EPI == kEpiGeluResid) xv = f2_add(xv, bf2_to_f2(hres[e]));
      o[e] = f2_to_bf2(xv);
      if (HEAD) {
        const uint64_t f = bf2_to_f2(o[e]);
        const int col = (t & 7) * 8 + 2 * e;
        lg0 = f2_fma(f, *reinterpret_cast<const uint64_t*>(a.head.head_w + col), lg0);
        lg1 = f2_fma(f, *reinterpret_cast<const uint64_t*>(a.head.head_w + C + col), lg1);
      }
    }
    *reinterpret_cast<uint4*>(a.y + shot * a.y_shot_stride + static_cast<int64_t>(on) * a.y_node_stride + (t & 7) * 8) =
        u;
  }
  if (HEAD) {
    // the row's 8 threads are 8 consecutive lanes: add their partial dot products
    float l0 = f2_lo(lg0) + f2_hi(lg0), l1 = f2_lo(lg1) + f2_hi(lg1);
#pragma unroll
    for (int m = 1; m < 8; m <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, m);
      l1 += __shfl_xor_sync(0xffffffffu, l1, m);
    }
    if (o_ok && recv_ok && (t & 7) == 0) {
      l0 += __ldg(a.head.head_b);
      l1 += __ldg(a.head.head_b + 1);
      *reinterpret_cast<float2*>(a.head.logits + shot * a.head.lg_shot_stride +
                                 static_cast<int64_t>(on) * a.head.lg_node_stride) = make_float2(l0, l1);
      if (a.head.res_bits) {
        const uint32_t bit = 1u << (shot & 31);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const bool flip = (k >> 1) ? (l1 > 0.f) : (l0 > 0.f);
          const int32_t cidx = __ldg(a.head.xor_nbr + static_cast<int64_t>(on) * 4 + k);
          if (flip && cidx >= 0)
            atomicXor(a.head.res_bits + static_cast<int64_t>(cidx) * a.head.res_words + (shot >> 5), bit);
        }
      }
    }
  }
  if (t == 0 && !loads_ok) {
    // bounded drain of the loads in flight before the CTA leaves
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(smem_u32(full), 0) && globaltimer_ns() - t0 < a.timeout_ns) {
    }
  }
  if (t == 0) bulk_wait_read();                // the outgoing copies have read sO before the CTA leaves
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 64);
  }
}

using SplitFn = void (*)(CUtensorMap, CUtensorMap, NodeArgs);

SplitFn select_split_kernel(int epi, bool head) {
  if (epi == kEpiStore) return head ? nullptr : &gmm_nodes_split_kernel<kEpiStore, false>;
  if (epi == kEpiGeluInit)
    return head ? &gmm_nodes_split_kernel<kEpiGeluInit, true> : &gmm_nodes_split_kernel<kEpiGeluInit, false>;
  if (epi == kEpiGeluResid)
    return head ? &gmm_nodes_split_kernel<kEpiGeluResid, true> : &gmm_nodes_split_kernel<kEpiGeluResid, false>;
  return nullptr;
}

using NodeFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, NodeArgs);

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
  if (p.x_node_stride % p.Ci || p.x_shot_stride % p.Ci || p.y_node_stride % p.Co || p.y_shot_stride % p.Co)
    return fail(BPC_ERR_ARG, "node-tiled path: row strides must be multiples of the channel count");
  const int64_t x_rows = ((p.NS - 1) * p.x_node_stride + (p.shots - 1) * p.x_shot_stride) / p.Ci + 1;
  const int64_t y_rows = ((p.NT - 1) * p.y_node_stride + (p.shots - 1) * p.y_shot_stride) / p.Co + 1;
  if (x_rows >= 0x7fffffffLL || y_rows >= 0x7fffffffLL) return fail(BPC_ERR_ARG, "node-tiled path: tensor too large");
  // the activations as 2D (channel, row) tensors with one-row boxes: the gathers' maps
  CUtensorMap tmX, tmY;
  auto rows_map = [&](CUtensorMap* m, const void* base, int C, int64_t rows) -> int {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(C) * 2};
    cuuint32_t box[2] = {64, 1};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : fail(BPC_ERR_DRIVER, "cuTensorMapEncodeTiled(rows) failed: " + std::to_string(int(r)));
  };
  if (int e = rows_map(&tmX, p.x, p.Ci, x_rows)) return e;
  if (int e = rows_map(&tmY, p.y, p.Co, y_rows)) return e;
  NodeArgs a;
  a.x = static_cast<const __nv_bfloat16*>(p.x);
  a.x_row_node = p.x_node_stride / p.Ci;
  a.x_row_shot = p.x_shot_stride / p.Ci;
  a.y_row_node = p.y_node_stride / p.Co;
  a.y_row_shot = p.y_shot_stride / p.Co;
  a.x_rows = static_cast<int32_t>(x_rows);
  a.y_rows = static_cast<int32_t>(y_rows);
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
  if (p.Ci == 64 && p.Co == 64 && p.K == kSplitK) {
    // relation-split tiles: a cluster of 8 CTAs per 128 target nodes
    SplitFn sf = select_split_kernel(p.epi, p.head.head_w != nullptr);
    if (!sf) return fail(BPC_ERR_ARG, "node-tiled path: unsupported epilogue");
    const int ssmem = 1024 + kNodeRows * 128 + 64 * 128 + 2 * kSplitK * 16 * 64 * 4 + 64;
    if (int e = allow_smem(reinterpret_cast<const void*>(sf), ssmem)) return e;
    void* sargs[] = {&tmW, &tmX, &a};
    if (int e = launch_pdl(reinterpret_cast<const void*>(sf), dim3(static_cast<unsigned>(a.tiles * kSplitK),
                                                                   static_cast<unsigned>(p.shots)),
                           dim3(kSplitThreads), static_cast<size_t>(ssmem), stream, sargs, kSplitK,
                           "gmm_nodes_split_kernel"))
      return e;
    return 0;
  }
  const int nkb = p.Ci / 64;
  const int stage_bytes = nkb * kNodeRows * 128 + nkb * p.Co * 128;
  const int fixed = 1024 + kNodeRows * p.Co * 2 + ((kNodeRows * p.K * 4 + 15) & ~15) + 16;
  int stages = std::min(p.K, 8);
  while (stages > 1 && fixed + stages * stage_bytes + (2 * stages + 2) * 8 > kNodeSmemLimit) --stages;
  a.stages = stages;
  const int smem = fixed + stages * stage_bytes + (2 * stages + 2) * 8;
  NodeFn fn = select_node_kernel(p.Ci, p.Co, p.epi, p.head.head_w != nullptr);
  if (!fn) return fail(BPC_ERR_ARG, "node-tiled path: unsupported epilogue");
  if (int e = allow_smem(reinterpret_cast<const void*>(fn), kNodeSmemLimit)) return e;
  void* args[] = {&tmW, &tmX, &tmY, &a};
  if (int e = launch_pdl(reinterpret_cast<const void*>(fn), dim3(a.tiles, static_cast<unsigned>(p.shots)),
                         dim3(kNodeThreads), static_cast<size_t>(smem), stream, args, 1, "gmm_nodes_kernel"))
    return e;
  return 0;
}

}  // namespace bpc
