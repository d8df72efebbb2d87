// Bipartite-conv step on the 5th-generation tensor cores (sm_100a): one persistent, warp-specialised kernel.
//
//   y[s, n, :] (op)= sum_r x[s, idx[n, r], :] W_{type(n), r}^T            (cascade_triton.py:5,40 -- same arithmetic)
//
// Tile = one target node n x 128 MT shots.  The rows of the MMA are shots, so for a given relation r every row of
// the tile reads the same source node idx[n, r]: the neighbour "gather" is one block copy per (tile, relation,
// 64-channel block), and a pad slot (idx outside [0, NS)) is a relation the tile skips entirely (no load, no MMA).
// Two activation layouts:
//   rows     x of any row layout -- shot-major (B, NS, C), the reference op's, or node-major -- viewed as the 3D
//            tensor (channel, shot, node); one TMA box per stage into the 128-byte-swizzled K-major layout.
//   blocked  the pre-decoder's (node, shots / TM, C / 8, TM, 8) layout, TM = 128 MT: a tile's activations are one
//            contiguous block, so a stage is one 1D bulk copy (8 channel groups x TM shots x 16 bytes) straight into
//            the canonical no-swizzle K-major layout (8-row x 16-byte core matrices), and the epilogue's loads and
//            stores cover 512 contiguous bytes per warp instruction.
// W_r (Co x 64 channels per stage) always comes by TMA in the 128-byte-swizzled K-major layout.
//
// Roles (320 threads, one CTA per SM):
//   warp 0     producer: A block(s) + W box per stage, completion counted in bytes on the stage's mbarrier
//   warp 1     TMEM owner and MMA issuer: per 16-channel step MT tcgen05.mma M=128 N=Co K=16 sharing the W stage,
//              fp32 accumulators in TMEM, double-buffered (2 x MT x Co columns) so the epilogue of tile i overlaps
//              the MMAs of tile i + 1
//   warps 2-9  epilogue, one shot (TMEM lane) per thread: tcgen05.ld of 32 columns at a time, GELU / residual add
//              (the residual rows are loaded before the accumulator is waited for), bf16 store, and for the
//              pre-decoder's last check -> data step the X / Z head, the threshold and the XOR of the predicted flips
//              into the bit-packed residual syndrome (one ballot + atomicXor per warp and check)
// Every wait is bounded (mbar_wait); a timeout sets the status word and the CTA drains and returns.
#include <algorithm>
#include <cstdio>
#include <map>
#include <mutex>
#include <string>
#include <set>
#include <utility>

#include <cudaTypedefs.h>

#include "bpc_common.cuh"
#include "bpc_internal.h"

namespace bpc {

namespace {

constexpr int kThreads = 320;         // warp 0 producer, warp 1 MMA, warps 2-9 epilogue
constexpr int kEpiWarps = 8;
constexpr int kBlockM = 128;          // rows of one MMA (shots)
constexpr int kKBlock = 64;           // channels per stage
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
  const int32_t* order;                   // target processing order (null: node order)
  const __nv_bfloat16* x;                 // blocked loader only
  int64_t x_node_stride;                  // blocked loader only (elements)
  void* y;
  int64_t y_shot_stride, y_node_stride, y_cg_stride;
  int epi;
  const float* epi_scale;
  const float* epi_shift;
  HeadEpilogue head;
  const void* res_h;                      // kEpiGeluStream: residual stream in (null: none), out, bf16 copy out
  int res_f32;
  void* res_out;
  void* res_out16;
  int64_t res_shot_stride, res_node_stride;
  int* status;
  uint64_t timeout_ns;
  uint32_t tmem_cols;
  unsigned long long* tile_counter;       // dynamic scheduling (zero at launch), or null
};

__device__ __forceinline__ int target_of(const TcArgs& a, int64_t tile) {
  const int i = static_cast<int>(tile % a.NT);
  return a.order ? __ldg(a.order + i) : i;
}

constexpr int kMaxK = 16;   // relations per target on the tensor-core path

// A tile's target node and index row.  The loads are independent (unrolled, predicated) and every role issues the
// next tile's loads one tile ahead; the valid mask is formed only when the tile starts (finish_row), so no role
// stalls on table loads in the middle of its pipeline.
struct TileRow {
  int n;
  uint32_t vm;              // relations whose source is in [0, NS)
  int src[kMaxK];
};

__device__ __forceinline__ void issue_row(const TcArgs& a, int64_t tile, TileRow& t) {
  t.n = target_of(a, tile);
  const int32_t* row = a.idx + static_cast<int64_t>(t.n) * a.K;
#pragma unroll
  for (int r = 0; r < kMaxK; ++r) t.src[r] = r < a.K ? __ldg(row + r) : -1;
}

__device__ __forceinline__ void finish_row(const TcArgs& a, TileRow& t) {
  t.vm = 0;
#pragma unroll
  for (int r = 0; r < kMaxK; ++r)
    if (t.src[r] >= 0 && t.src[r] < a.NS) t.vm |= 1u << r;
}


// the 4 channel groups (32 channels) of chunk c of one shot's row
__device__ __forceinline__ void ld_chunk(const __nv_bfloat16* base, int64_t cg_stride, int c, uint4 (&r)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) r[j] = *reinterpret_cast<const uint4*>(base + (4 * c + j) * cg_stride);
}

// Tiles reach the MMA and epilogue warps through a small ring in shared memory written by the producer thread,
// which is the only role that picks tiles: from a global counter (dynamic scheduling: all CTAs stay within a
// window of consecutive tiles, so the sources they share stay in L2) or, without a counter, by striding.
constexpr int kRing = 4;
struct RingEntry {
  long long tile;           // -1: no more tiles
  int n;                    // target node
  uint32_t vm;              // relations with a source in [0, NS)
};

template <int MT, int NCH, bool BLOCKED, int EPI, bool HEAD>
__global__ void __launch_bounds__(kThreads, 1)
    gmm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW, const TcArgs a) {
  constexpr int Co = NCH * 32;
  constexpr int kTileM = kBlockM * MT;
  constexpr uint32_t kABytes = kSubBytes * MT;
  constexpr uint32_t kItemBytes = kABytes + Co * 128;  // one (relation, 64-channel block) item: A block + W block
  constexpr uint32_t kCgBytes = kTileM * 16;        // blocked layout: one channel group of the tile's shots
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  constexpr uint32_t stage_bytes = kItemBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * stage_bytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* accf = bars + 2 * S;
  uint64_t* acce = bars + 2 * S + 2;
  uint64_t* drain = bars + 2 * S + 4;
  uint64_t* tfull = bars + 2 * S + 5;
  uint64_t* tempty = bars + 2 * S + 5 + kRing;
  volatile RingEntry* ring = reinterpret_cast<volatile RingEntry*>(bars + 2 * S + 5 + 2 * kRing);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5 + 2 * kRing + 2 * kRing);
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
    for (int i = 0; i < kRing; ++i) {
      mbar_init(smem_u32(&tfull[i]), 1);
      mbar_init(smem_u32(&tempty[i]), 1 + kEpiWarps);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_mbar_init();
    if (!BLOCKED) tma_prefetch_desc(&tmA);
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
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_parity = 0;   // stages with a load in flight and the parity it completes
      int rslot = 0;
      uint32_t rphase = 0;
      bool ok = true;
      long long next = a.tile_counter ? atomicAdd(a.tile_counter, 1ull) : static_cast<long long>(blockIdx.x);
      TileRow nrow;
      issue_row(a, next < a.num_tiles ? next : 0, nrow);
      while (ok) {
        const long long tile = next;
        finish_row(a, nrow);
        const TileRow cur = nrow;
        // publish the tile (or the end) to the MMA and epilogue warps
        if (!mbar_wait(smem_u32(&tempty[rslot]), rphase ^ 1u, abort_flag, a.status, a.timeout_ns)) break;
        ring[rslot].tile = tile < a.num_tiles ? tile : -1;
        ring[rslot].n = cur.n;
        ring[rslot].vm = cur.vm;
        mbar_arrive(smem_u32(&tfull[rslot]));
        if (++rslot == kRing) {
          rslot = 0;
          rphase ^= 1u;
        }
        if (tile >= a.num_tiles) break;
        // the next tile: picked now so its index row is on its way while this tile is loaded
        next = a.tile_counter ? atomicAdd(a.tile_counter, 1ull) : tile + gridDim.x;
        issue_row(a, next < a.num_tiles ? next : tile, nrow);
        const int n = cur.n;
        const int64_t s0 = (tile / a.NT) * kTileM;
        const int wrow = (n >= a.type_split) ? Co : 0;
#pragma unroll 1
        for (int r = 0; r < a.K && ok; ++r) {
          if (!(cur.vm & (1u << r))) continue;
          const int src = cur.src[r];
#pragma unroll 1
          for (int kb = 0; kb < a.n_kb; ++kb) {
            if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, a.status, a.timeout_ns)) {
              ok = false;
              break;
            }
            const uint32_t sa = smem_u32(smem + stage * stage_bytes);
            const uint32_t fb = smem_u32(&full[stage]);
            if (BLOCKED) {
              const int ncg = min(8, (a.Ci - kb * kKBlock) / 8);
              mbar_arrive_expect_tx(fb, ncg * kCgBytes + Co * 128);
              bulk_load(sa, a.x + static_cast<int64_t>(src) * a.x_node_stride + s0 * a.Ci + kb * 8 * (kTileM * 8),
                        ncg * kCgBytes, fb);
            } else {
              mbar_arrive_expect_tx(fb, kItemBytes);
              tma_load_3d(sa, &tmA, kb * kKBlock, static_cast<int32_t>(s0), src, fb);   // kTileM shots x 64 ch
            }
            tma_load_3d(sa + kABytes, &tmW, kb * kKBlock, r, wrow, fb);               // Co rows x 64 ch of W_r
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
      int rslot = 0;
      uint32_t rphase = 0;
      bool ok = true;
      while (ok) {
        if (!mbar_wait(smem_u32(&tfull[rslot]), rphase, abort_flag, a.status, a.timeout_ns)) break;
        const long long tile = ring[rslot].tile;
        const uint32_t vm = ring[rslot].vm;
        mbar_arrive(smem_u32(&tempty[rslot]));
        if (++rslot == kRing) {
          rslot = 0;
          rphase ^= 1u;
        }
        if (tile < 0) break;
        if (!mbar_wait(smem_u32(&acce[acc]), acc_phase ^ 1u, abort_flag, a.status, a.timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * MT * Co);
        uint32_t accumulate = 0;
#pragma unroll 1
        for (int r = 0; r < a.K && ok; ++r) {
          if (!(vm & (1u << r))) continue;
#pragma unroll 1
          for (int kb = 0; kb < a.n_kb; ++kb) {
            if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, a.status, a.timeout_ns)) {
              ok = false;
              break;
            }
            // descriptors built once per stage, advanced by constants (the address field counts 16-byte units)
            const uint32_t sa = smem_u32(smem + stage * stage_bytes);
            const uint64_t ad0 = BLOCKED ? sdesc_k_none(sa, kCgBytes, 128) : sdesc_k_sw128(sa);
            const uint64_t bd0 = sdesc_k_sw128(sa + kABytes);
            const bool full_kb = (kb + 1) * kKBlock <= a.Ci;
            const int ksteps = full_kb ? 4 : (a.Ci - kb * kKBlock + 15) / 16;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              if (k < ksteps) {
                const uint64_t bd = bd0 + static_cast<uint64_t>((k * 32) >> 4);
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                  const uint32_t aoff = BLOCKED ? (2 * k * kCgBytes + m * kBlockM * 16) : (m * kSubBytes + k * 32);
                  tc_mma_ss(d_tmem + m * Co, ad0 + static_cast<uint64_t>(aoff >> 4), bd, idesc, accumulate);
                }
                accumulate = 1;
              }
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
    // One shot (TMEM lane) per thread.  Element math runs on packed fp32 pairs (f32x2); the residual row is loaded
    // before the accumulator wait (whole row up to 128 channels, then two 32-channel chunks ahead).
    constexpr bool kResid = EPI == kEpiGeluResid || EPI == kEpiAdd;
    constexpr int kPre = NCH <= 4 ? NCH : 2;          // chunks loaded before the accumulator wait
    const int q = warp & 3;                   // TMEM lane quarter this warp may access
    const int m = (warp - 2) >> 2;            // which 128-shot sub-tile
    const int row = q * 32 + lane;
    const bool active = m < MT;
    const int64_t cgs = BLOCKED ? kTileM * 8 : a.y_cg_stride;
    int acc = 0;
    uint32_t acc_phase = 0;
    int rslot = 0;
    uint32_t rphase = 0;
    while (true) {
      if (!mbar_wait(smem_u32(&tfull[rslot]), rphase, abort_flag, a.status, a.timeout_ns)) break;
      const long long tile = ring[rslot].tile;
      const int n = ring[rslot].n;
      const uint32_t vm = active ? ring[rslot].vm : 0u;
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&tempty[rslot]));
      if (++rslot == kRing) {
        rslot = 0;
        rphase ^= 1u;
      }
      if (tile < 0) break;
      const int64_t s0 = (tile / a.NT) * kTileM + m * kBlockM;
      const int64_t shot = s0 + row;
      const bool ok = active && shot < a.shots;
      __nv_bfloat16* yrow = reinterpret_cast<__nv_bfloat16*>(a.y) + static_cast<int64_t>(n) * a.y_node_stride +
                            (BLOCKED ? (s0 - m * kBlockM) * Co + (m * kBlockM + row) * 8 : shot * a.y_shot_stride);
      // the residual rows do not depend on the MMAs: load them before waiting for the accumulator
      uint4 rbuf[kResid ? kPre : 1][4];
      if (kResid && ok) {
#pragma unroll
        for (int c = 0; c < kPre; ++c) ld_chunk(yrow, cgs, c, rbuf[c]);
      }
      if (!mbar_wait(smem_u32(&accf[acc]), acc_phase, abort_flag, a.status, a.timeout_ns)) break;
      tc_fence_after();
      uint64_t lg0 = 0, lg1 = 0;              // packed partial head sums (two columns each)
      if (active) {
        const uint32_t taddr =
            tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * MT * Co + m * Co);
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          float v[32];
          if (vm) {
            tmem_ld32(taddr + c * 32, v);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0.f;
          }
          uint4 cur[4];
          if (kResid) {
#pragma unroll
            for (int j = 0; j < 4; ++j) cur[j] = rbuf[c % kPre][j];
            if (ok && c + kPre < NCH) ld_chunk(yrow, cgs, c + kPre, rbuf[c % kPre]);
          }
          if (ok) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint4 u;
              uint32_t* o = reinterpret_cast<uint32_t*>(&u);
              const uint32_t* h = reinterpret_cast<const uint32_t*>(&cur[j]);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                uint64_t x = f2_pack(v[j * 8 + 2 * e], v[j * 8 + 2 * e + 1]);
                if (EPI == kEpiAffineSilu) {
                  const int colp = c * 32 + j * 8 + 2 * e;
                  x = silu_tanh_fast2(f2_fma(x, *reinterpret_cast<const uint64_t*>(a.epi_scale + colp),
                                             *reinterpret_cast<const uint64_t*>(a.epi_shift + colp)));
                } else if (EPI == kEpiGeluInit || EPI == kEpiGeluResid) {
                  x = gelu_tanh_fast2(x);
                }
                if (kResid) x = f2_add(x, bf2_to_f2(h[e]));
                o[e] = f2_to_bf2(x);
                if (HEAD) {
                  const uint64_t f = bf2_to_f2(o[e]);   // the stored (rounded) value feeds the head
                  const int col = c * 32 + j * 8 + 2 * e;
                  lg0 = f2_fma(f, *reinterpret_cast<const uint64_t*>(a.head.head_w + col), lg0);
                  lg1 = f2_fma(f, *reinterpret_cast<const uint64_t*>(a.head.head_w + Co + col), lg1);
                }
              }
              *reinterpret_cast<uint4*>(yrow + (4 * c + j) * cgs) = u;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&acce[acc]));
      if (HEAD && active) {
        const float l0 = f2_lo(lg0) + f2_hi(lg0) + __ldg(a.head.head_b);
        const float l1 = f2_lo(lg1) + f2_hi(lg1) + __ldg(a.head.head_b + 1);
        if (ok) {
          float2* lp = reinterpret_cast<float2*>(a.head.logits + shot * a.head.lg_shot_stride +
                                                 static_cast<int64_t>(n) * a.head.lg_node_stride);
          *lp = make_float2(l0, l1);
        }
        if (a.head.res_bits) {
          const uint32_t m0 = __ballot_sync(0xffffffffu, ok && l0 > 0.f);
          const uint32_t m1 = __ballot_sync(0xffffffffu, ok && l1 > 0.f);
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

// ---------------------------------------------------------------------------------------------------------------
// Wide-tile kernel: C_out in {64, 96, 128}, C_in <= 128, both layouts.
//
// The MMA rows are the output channels (M = 128; rows past C_out compute values nobody reads) and its columns the
// tile's 256 shots: one tcgen05.mma M=128 N=256 K=16 per 16 input channels, W_r's 64-channel stage (the same TMA box
// as above) as the K-major 128-byte-swizzled A operand and the activation stage as the B operand: the blocked
// stage (one bulk copy) in the K-major no-swizzle layout, or the row layout's TMA box (64 channels x 256 shots) in
// the K-major 128-byte-swizzled layout.  The tensor pipe takes a 256-column MMA at its full rate, while 128-column
// MMAs cost more than their share per instruction (measured on B200 with one issuing thread: M128 N128 K16 80-100
// cycles each against 64 ideal, M128 N256 K16 at the ideal 128).  Each stage is freed by a commit after its MMAs.
//
// The accumulator rows are channels.  Each epilogue warp owns one TMEM lane quarter (32 channels) and one half of
// the tile's shots; it reads 16 shot columns at a time (tcgen05.ld 32x32b.x16), turns them around through a 2 KB
// scratch of its own (row = channel, 16-byte chunks swizzled: conflict-free stores and loads) so that each thread
// holds 16 channels of one shot, and then runs the row kernel's element arithmetic (same bits).  Quarters past
// C_out only keep the barriers.  With the head (blocked layout), the logits of a shot need all its channels: after
// every warp has stored its part of the tile (an mbarrier of 256 arrivals, waited with the watchdog), each warp
// reads 32 shots' rows back and forms the logits, threshold and residual XOR exactly as the row kernel does.
constexpr int kWideShots = 256;                       // tile shots = MMA N
constexpr int kWideM = 128;                           // MMA M (output channels, padded)
constexpr uint32_t kWideXBytes = kWideShots * 64 * 2;   // one 64-channel activation stage
constexpr uint32_t kWideWBytes = kWideM * 128;          // W_r rows x 64 channels
constexpr uint32_t kWideStageBytes = kWideXBytes + kWideWBytes;
constexpr int kWideStages = 4;
constexpr int kWideScratch = 2048;                    // per epilogue warp: 32 channels x 16 shots fp32
constexpr int kWideBars = 2 * kWideStages + 2 + 2 + 1 + 2 * kRing + 2;

__host__ __device__ constexpr int wide_smem_bytes() {
  return 1024 + kWideStages * kWideStageBytes + kEpiWarps * kWideScratch + kWideBars * 8 + kRing * 16 + 16;
}

// fp32 scratch element (channel row c of the warp's quarter, shot column s of the 16-shot piece), in bytes
__device__ __forceinline__ uint32_t wide_scr_off(int c, int s) {
  return static_cast<uint32_t>((c ^ ((c >> 4) & 1)) * 64 + (((s >> 2) ^ ((c >> 1) & 3)) << 4) + (s & 3) * 4);
}

// NKB 64-channel blocks of C_in, KLAST 16-channel MMA steps in the last one (C_in = 64 (NKB - 1) + 16 KLAST): the MMA
// issue sequence is unrolled at compile time.  Blocked layout: C_out = C_in.
template <bool BLOCKED, int EPI, bool HEAD, int NKB, int KLAST>
__global__ void __launch_bounds__(kThreads, 1)
    gmm_wide_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW, const TcArgs a) {
  constexpr int kCgElems = kWideShots * 8;            // blocked: one channel group of a tile (elements)
  constexpr int kCi = 64 * (NKB - 1) + 16 * KLAST;
  constexpr bool kLoadY = EPI == kEpiGeluResid || EPI == kEpiAdd;     // the epilogue reads y before writing it
  constexpr bool kGelu = EPI == kEpiGeluInit || EPI == kEpiGeluResid;
  constexpr bool kAffine = EPI == kEpiAffineSilu;                    // SiLU(scale acc + shift) per output channel
  constexpr bool kStream = EPI == kEpiGeluStream;                    // y = acc, and the GELU residual stream
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* scratch = smem + kWideStages * kWideStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(scratch + kEpiWarps * kWideScratch);
  uint64_t* full = bars;                              // per stage
  uint64_t* empty = bars + kWideStages;               // per stage
  uint64_t* accf = empty + kWideStages;
  uint64_t* acce = accf + 2;
  uint64_t* drain = acce + 2;
  uint64_t* tfull = drain + 1;
  uint64_t* tempty = tfull + kRing;
  uint64_t* stored = tempty + kRing;                  // head: the tile's outputs are all stored (per accumulator)
  volatile RingEntry* ring = reinterpret_cast<volatile RingEntry*>(bars + kWideBars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(bars + kWideBars) + kRing * 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int Co = BLOCKED ? kCi : a.Co;                // blocked layout: C_out = C_in, known at compile time

  if (threadIdx.x == 0) {
    for (int i = 0; i < kWideStages; ++i) {
      mbar_init(smem_u32(&full[i]), 1);
      mbar_init(smem_u32(&empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&accf[i]), 1);
      mbar_init(smem_u32(&acce[i]), kEpiWarps);
      mbar_init(smem_u32(&stored[i]), kEpiWarps * 32);
    }
    for (int i = 0; i < kRing; ++i) {
      mbar_init(smem_u32(&tfull[i]), 1);
      mbar_init(smem_u32(&tempty[i]), 1 + kEpiWarps);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_mbar_init();
    if (!BLOCKED) tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_parity = 0;
      int rslot = 0;
      uint32_t rphase = 0;
      bool ok = true;
      const uint32_t stage_tx = kWideXBytes + static_cast<uint32_t>(Co) * 128;
      long long next = a.tile_counter ? atomicAdd(a.tile_counter, 1ull) : static_cast<long long>(blockIdx.x);
      TileRow nrow;
      issue_row(a, next < a.num_tiles ? next : 0, nrow);
      while (ok) {
        const long long tile = next;
        finish_row(a, nrow);
        const TileRow cur = nrow;
        if (!mbar_wait(smem_u32(&tempty[rslot]), rphase ^ 1u, abort_flag, a.status, a.timeout_ns)) break;
        ring[rslot].tile = tile < a.num_tiles ? tile : -1;
        ring[rslot].n = cur.n;
        ring[rslot].vm = cur.vm;
        mbar_arrive(smem_u32(&tfull[rslot]));
        if (++rslot == kRing) {
          rslot = 0;
          rphase ^= 1u;
        }
        if (tile >= a.num_tiles) break;
        next = a.tile_counter ? atomicAdd(a.tile_counter, 1ull) : tile + gridDim.x;
        issue_row(a, next < a.num_tiles ? next : tile, nrow);
        const int64_t s0 = (tile / a.NT) * kWideShots;
        const int wrow = (cur.n >= a.type_split) ? Co : 0;
#pragma unroll 1
        for (int r = 0; r < a.K && ok; ++r) {
          if (!(cur.vm & (1u << r))) continue;
#pragma unroll
          for (int kb = 0; kb < NKB; ++kb) {
            if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, a.status, a.timeout_ns)) {
              ok = false;
              break;
            }
            const uint32_t sa = smem_u32(smem + stage * kWideStageBytes);
            const uint32_t fb = smem_u32(&full[stage]);
            if (BLOCKED) {
              const int ncg = kb + 1 < NKB ? 8 : 2 * KLAST;
              mbar_arrive_expect_tx(fb, ncg * kCgElems * 2 + static_cast<uint32_t>(Co) * 128);
              bulk_load(sa, a.x + static_cast<int64_t>(cur.src[r]) * a.x_node_stride + s0 * kCi + kb * 8 * kCgElems,
                        ncg * kCgElems * 2, fb);
            } else {
              mbar_arrive_expect_tx(fb, stage_tx);
              tma_load_3d(sa, &tmA, kb * kKBlock, static_cast<int32_t>(s0), cur.src[r], fb);
            }
            tma_load_3d(sa + kWideXBytes, &tmW, kb * kKBlock, r, wrow, fb);
            armed |= 1u << stage;
            armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
            if (++stage == kWideStages) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
      if (!ok) {
        for (int i = 0; i < kWideStages; ++i)
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
      constexpr uint32_t idesc = idesc_bf16_f32(kWideM, kWideShots);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      int rslot = 0;
      uint32_t rphase = 0;
      bool ok = true;
      while (ok) {
        if (!mbar_wait(smem_u32(&tfull[rslot]), rphase, abort_flag, a.status, a.timeout_ns)) break;
        const long long tile = ring[rslot].tile;
        const uint32_t vm = ring[rslot].vm;
        mbar_arrive(smem_u32(&tempty[rslot]));
        if (++rslot == kRing) {
          rslot = 0;
          rphase ^= 1u;
        }
        if (tile < 0) break;
        if (!mbar_wait(smem_u32(&acce[acc]), acc_phase ^ 1u, abort_flag, a.status, a.timeout_ns)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kWideShots);
        uint32_t accumulate = 0;
#pragma unroll 1
        for (int r = 0; r < a.K && ok; ++r) {
          if (!(vm & (1u << r))) continue;
#pragma unroll
          for (int kb = 0; kb < NKB; ++kb) {
            if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, a.status, a.timeout_ns)) {
              ok = false;
              break;
            }
            const uint32_t sa = smem_u32(smem + stage * kWideStageBytes);
            const uint64_t ad0 = sdesc_k_sw128(sa + kWideXBytes);
            const uint64_t bd0 = BLOCKED ? sdesc_k_none(sa, kCgElems * 2, 128) : sdesc_k_sw128(sa);
            const int ksteps = kb + 1 < NKB ? 4 : KLAST;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              if (k < ksteps) {
                const uint32_t boff = BLOCKED ? 2 * k * kCgElems * 2 : k * 32;
                tc_mma_ss(d_tmem, ad0 + static_cast<uint64_t>((k * 32) >> 4), bd0 + static_cast<uint64_t>(boff >> 4),
                          idesc, accumulate);
                accumulate = 1;
              }
            }
            tc_commit(smem_u32(&empty[stage]));   // the stage is free once its MMAs have read it
            if (++stage == kWideStages) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
        if (!ok) break;
        tc_commit(smem_u32(&accf[acc]));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      tc_commit(smem_u32(drain));
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(smem_u32(drain), 0) && globaltimer_ns() - t0 < a.timeout_ns) {
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..9)
    const int q = warp & 3;                   // TMEM lane quarter: channels 32 q .. 32 q + 31
    const bool live = 32 * q < Co;            // quarters past C_out only keep the barriers
    const int e = warp - 2;
    const int half = e >> 2;                  // tile shots 128 half .. 128 half + 127
    const int s = lane & 15;                  // after the turn-around: shot s of the 16-shot piece ...
    const int h = lane >> 4;                  // ... channels 32 q + 16 h .. + 15 (channel groups 4 q + 2 h, + 1)
    const int cg0 = 4 * q + 2 * h;
    const uint32_t scr_u = smem_u32(scratch + e * kWideScratch);
    int acc = 0;
    uint32_t acc_phase = 0;
    int rslot = 0;
    uint32_t rphase = 0;
    // every wait is decided for the whole warp (a watchdog timeout seen by some lanes ends the loop for all, so no
    // lane is left in a warp-collective instruction)
    while (true) {
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&tfull[rslot]), rphase, abort_flag, a.status, a.timeout_ns)))
        break;
      const long long tile = ring[rslot].tile;
      const int n = ring[rslot].n;
      const uint32_t vm = ring[rslot].vm;
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&tempty[rslot]));
      if (++rslot == kRing) {
        rslot = 0;
        rphase ^= 1u;
      }
      if (tile < 0) break;
      const int64_t s0 = (tile / a.NT) * kWideShots;
      __nv_bfloat16* const y = reinterpret_cast<__nv_bfloat16*>(a.y);
      __nv_bfloat16* const yt = y + static_cast<int64_t>(n) * a.y_node_stride + (BLOCKED ? s0 * kCi : 0);
      // this thread's two 16-byte chunks of piece j (shot 128 half + 16 j + s of the tile, channels 32 q + 16 h ..):
      // blocked: channel groups cg0 and cg0 + 1 of the tile block; rows: 32 contiguous bytes of the shot's row
      const int64_t step_j = BLOCKED ? 128 : 16 * a.y_shot_stride;
      const int64_t step_g = BLOCKED ? kCgElems : 8;
      __nv_bfloat16* const yc = BLOCKED ? yt + cg0 * kCgElems + (128 * half + s) * 8
                                        : yt + (s0 + 128 * half + s) * a.y_shot_stride + 32 * q + 16 * h;
      uint4 rb[kLoadY ? 8 : 1][2];
      if (kLoadY && live) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (s0 + 128 * half + 16 * j + s < a.shots) {
            rb[j][0] = *reinterpret_cast<const uint4*>(yc + j * step_j);
            rb[j][1] = *reinterpret_cast<const uint4*>(yc + j * step_j + step_g);
          }
      }
      // kStream: this thread's 16 channels (32 q + 16 h ..) of the residual stream row of its shot in each piece,
      // loaded one piece ahead
      const int64_t rbase = kStream ? static_cast<int64_t>(n) * a.res_node_stride + 32 * q + 16 * h : 0;
      float4 hf[4], hfn[4];
      uint4 hb[2], hbn[2];
      auto load_res = [&](int j, float4 (&f)[4], uint4 (&b)[2]) {
        const int64_t sj = s0 + 128 * half + 16 * j + s;
        if (!live || sj >= a.shots || !a.res_h) return;
        const int64_t off = sj * a.res_shot_stride + rbase;
        if (a.res_f32) {
          const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(a.res_h) + off);
#pragma unroll
          for (int i = 0; i < 4; ++i) f[i] = p[i];
        } else {
          const uint4* p = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.res_h) + off);
          b[0] = p[0];
          b[1] = p[1];
        }
      };
      if (kStream) load_res(0, hf, hb);
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&accf[acc]), acc_phase, abort_flag, a.status, a.timeout_ns)))
        break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                             static_cast<uint32_t>(acc * kWideShots + 128 * half);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (kStream && j + 1 < 8) load_res(j + 1, hfn, hbn);
        float v[16];
        if (vm && live) {
          tmem_ld16(taddr + 16 * j, v);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = 0.f;
        }
        if (j == 7) {                         // the accumulator buffer is free for the next tile's MMAs
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&acce[acc]));
        }
        if (!live) continue;
        // turn around: row = channel (this lane), 16 shot columns -> this thread: shot s, 16 channels
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4)
          asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(scr_u + wide_scr_off(lane, 4 * c4)),
                       "f"(v[4 * c4]), "f"(v[4 * c4 + 1]), "f"(v[4 * c4 + 2]), "f"(v[4 * c4 + 3])
                       : "memory");
        __syncwarp();
        float x[16];
#pragma unroll
        for (int k = 0; k < 16; ++k)
          asm volatile("ld.shared.f32 %0, [%1];" : "=f"(x[k]) : "r"(scr_u + wide_scr_off(16 * h + k, s)) : "memory");
        __syncwarp();
        const bool ok = s0 + 128 * half + 16 * j + s < a.shots;
        if (ok) {
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            uint4 u;
            uint32_t* o = reinterpret_cast<uint32_t*>(&u);
            const uint32_t* hr = reinterpret_cast<const uint32_t*>(&rb[kLoadY ? j : 0][g]);
#pragma unroll
            for (int e4 = 0; e4 < 4; ++e4) {
              uint64_t xx = f2_pack(x[8 * g + 2 * e4], x[8 * g + 2 * e4 + 1]);
              if (kGelu) xx = gelu_tanh_fast2(xx);
              if (kAffine) {
                const int colp = 32 * q + 16 * h + 8 * g + 2 * e4;
                xx = silu_tanh_fast2(f2_fma(xx, *reinterpret_cast<const uint64_t*>(a.epi_scale + colp),
                                            *reinterpret_cast<const uint64_t*>(a.epi_shift + colp)));
              }
              if (kLoadY) xx = f2_add(xx, bf2_to_f2(hr[e4]));
              o[e4] = f2_to_bf2(xx);
            }
            *reinterpret_cast<uint4*>(yc + j * step_j + g * step_g) = u;
            if (kStream) {
              // the residual step of the training network on the stored (bf16) pre-activation, the arithmetic of
              // the GELU / residual pass: g = bf16(GELU(a)); fp32 stream: out = h + g and its bf16 copy; bf16
              // stream: out = bf16(g + h); no stream: out = g
              float gv[8];
#pragma unroll
              for (int e4 = 0; e4 < 4; ++e4) {
                gv[2 * e4] = __bfloat162float(__float2bfloat16_rn(gelu_tanh_pass(__uint_as_float(o[e4] << 16))));
                gv[2 * e4 + 1] =
                    __bfloat162float(__float2bfloat16_rn(gelu_tanh_pass(__uint_as_float(o[e4] & 0xFFFF0000u))));
              }
              const int64_t off = (s0 + 128 * half + 16 * j + s) * a.res_shot_stride + rbase + 8 * g;
              uint4 w16;
              uint32_t* w16w = reinterpret_cast<uint32_t*>(&w16);
              if (a.res_h && a.res_f32) {
                const float4 h0 = hf[2 * g], h1 = hf[2 * g + 1];
                const float vv[8] = {h0.x + gv[0], h0.y + gv[1], h0.z + gv[2], h0.w + gv[3],
                                     h1.x + gv[4], h1.y + gv[5], h1.z + gv[6], h1.w + gv[7]};
                float4* op = reinterpret_cast<float4*>(static_cast<float*>(a.res_out) + off);
                op[0] = make_float4(vv[0], vv[1], vv[2], vv[3]);
                op[1] = make_float4(vv[4], vv[5], vv[6], vv[7]);
#pragma unroll
                for (int e4 = 0; e4 < 4; ++e4) w16w[e4] = f2_to_bf2(f2_pack(vv[2 * e4], vv[2 * e4 + 1]));
                *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.res_out16) + off) = w16;
              } else {
                const uint32_t* hw = reinterpret_cast<const uint32_t*>(&hb[g]);
#pragma unroll
                for (int e4 = 0; e4 < 4; ++e4) {
                  float v0 = gv[2 * e4], v1 = gv[2 * e4 + 1];
                  if (a.res_h) {
                    v0 += __uint_as_float(hw[e4] << 16);
                    v1 += __uint_as_float(hw[e4] & 0xFFFF0000u);
                  }
                  w16w[e4] = f2_to_bf2(f2_pack(v0, v1));
                }
                *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.res_out) + off) = w16;
              }
            }
          }
        }
        if (kStream) {
#pragma unroll
          for (int i = 0; i < 4; ++i) hf[i] = hfn[i];
          hb[0] = hbn[0];
          hb[1] = hbn[1];
        }
      }
      if (HEAD) {
        // every warp's part of the tile is stored: read 32 shots' rows back and form the logits in the row kernel's
        // order (channel pairs, 32-channel chunks in order, stored bf16 values)
        mbar_arrive(smem_u32(&stored[acc]));
        if (!__all_sync(0xffffffffu,
                        mbar_wait(smem_u32(&stored[acc]), acc_phase, abort_flag, a.status, a.timeout_ns)))
          break;
        const int sl = 32 * e + lane;
        const bool ok = s0 + sl < a.shots;
        uint64_t lg0 = 0, lg1 = 0;
#pragma unroll
        for (int cg = 0; cg < kCi / 8; ++cg) {
          const uint4 u = *reinterpret_cast<const uint4*>(yt + cg * kCgElems + sl * 8);
          const uint32_t* o = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
          for (int e4 = 0; e4 < 4; ++e4) {
            const uint64_t f = bf2_to_f2(o[e4]);
            const int col = cg * 8 + 2 * e4;
            lg0 = f2_fma(f, *reinterpret_cast<const uint64_t*>(a.head.head_w + col), lg0);
            lg1 = f2_fma(f, *reinterpret_cast<const uint64_t*>(a.head.head_w + kCi + col), lg1);
          }
        }
        const float l0 = f2_lo(lg0) + f2_hi(lg0) + __ldg(a.head.head_b);
        const float l1 = f2_lo(lg1) + f2_hi(lg1) + __ldg(a.head.head_b + 1);
        if (ok) {
          float2* lp = reinterpret_cast<float2*>(a.head.logits + (s0 + sl) * a.head.lg_shot_stride +
                                                 static_cast<int64_t>(n) * a.head.lg_node_stride);
          *lp = make_float2(l0, l1);
        }
        if (a.head.res_bits) {
          const uint32_t m0 = __ballot_sync(0xffffffffu, ok && l0 > 0.f);
          const uint32_t m1 = __ballot_sync(0xffffffffu, ok && l1 > 0.f);
          if (lane < 4) {
            const int32_t c = __ldg(a.head.xor_nbr + static_cast<int64_t>(n) * 4 + lane);
            const uint32_t msk = (lane >> 1) ? m1 : m0;
            if (c >= 0 && msk)
              atomicXor(a.head.res_bits + static_cast<int64_t>(c) * a.head.res_words + (s0 >> 5) + e, msk);
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
    tmem_dealloc(tmem_base, 512);
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

int item_bytes_for(int Co) { return kSubBytes * mt_for(Co) + Co * 128; }

int smem_bytes_for(int Co, int stages) {
  return 1024 + stages * item_bytes_for(Co) + (2 * stages + 5 + 2 * kRing) * 8 + kRing * 16 + 8;
}

int stages_for(int Co) {
  int s = kMaxStages;
  while (s > 2 && smem_bytes_for(Co, s) > kSmemLimit) --s;
  return s;
}

using KernelFn = void (*)(CUtensorMap, CUtensorMap, TcArgs);

// rows layout: the plain op (store); blocked layout: the pre-decoder's steps (GELU first / GELU + residual, with or
// without the head)
template <int NCH>
KernelFn kernel_for(bool blocked, int epi, bool head) {
  constexpr int MT = mt_for(NCH * 32);
  if (!blocked) {
    if (head) return nullptr;
    if (epi == kEpiStore) return &gmm_tc_kernel<MT, NCH, false, kEpiStore, false>;
    if (epi == kEpiAffineSilu) return &gmm_tc_kernel<MT, NCH, false, kEpiAffineSilu, false>;
    if (epi == kEpiAdd) return &gmm_tc_kernel<MT, NCH, false, kEpiAdd, false>;
    return nullptr;
  }
  if (epi == kEpiGeluInit)
    return head ? &gmm_tc_kernel<MT, NCH, true, kEpiGeluInit, true> : &gmm_tc_kernel<MT, NCH, true, kEpiGeluInit, false>;
  if (epi == kEpiGeluResid)
    return head ? &gmm_tc_kernel<MT, NCH, true, kEpiGeluResid, true>
                : &gmm_tc_kernel<MT, NCH, true, kEpiGeluResid, false>;
  return nullptr;
}

KernelFn select_kernel(int Co, bool blocked, int epi, bool head) {
  switch (Co / 32) {
    case 1: return kernel_for<1>(blocked, epi, head);
    case 2: return kernel_for<2>(blocked, epi, head);
    case 3: return kernel_for<3>(blocked, epi, head);
    case 4: return kernel_for<4>(blocked, epi, head);
    case 5: return kernel_for<5>(blocked, epi, head);
    case 6: return kernel_for<6>(blocked, epi, head);
    case 7: return kernel_for<7>(blocked, epi, head);
    case 8: return kernel_for<8>(blocked, epi, head);
    default: return nullptr;
  }
}

// wide-tile kernel for (layout, epilogue, head, C_in in {64, 96, 128})
template <bool BLOCKED, int EPI, bool HEAD>
const void* wide_for_ci(int Ci) {
  switch (Ci) {
    case 64: return reinterpret_cast<const void*>(&gmm_wide_kernel<BLOCKED, EPI, HEAD, 1, 4>);
    case 96: return reinterpret_cast<const void*>(&gmm_wide_kernel<BLOCKED, EPI, HEAD, 2, 2>);
    case 128: return reinterpret_cast<const void*>(&gmm_wide_kernel<BLOCKED, EPI, HEAD, 2, 4>);
    default: return nullptr;
  }
}

const void* wide_kernel_for(bool blocked, int epi, bool head, int Ci) {
  if (blocked) {
    if (epi == kEpiGeluInit)
      return head ? wide_for_ci<true, kEpiGeluInit, true>(Ci) : wide_for_ci<true, kEpiGeluInit, false>(Ci);
    if (epi == kEpiGeluResid)
      return head ? wide_for_ci<true, kEpiGeluResid, true>(Ci) : wide_for_ci<true, kEpiGeluResid, false>(Ci);
    return nullptr;
  }
  if (head) return nullptr;
  if (epi == kEpiStore) return wide_for_ci<false, kEpiStore, false>(Ci);
  if (epi == kEpiAdd) return wide_for_ci<false, kEpiAdd, false>(Ci);
  if (epi == kEpiAffineSilu) return wide_for_ci<false, kEpiAffineSilu, false>(Ci);
  if (epi == kEpiGeluStream) return wide_for_ci<false, kEpiGeluStream, false>(Ci);
  return nullptr;
}

}  // namespace

int allow_smem(const void* fn, int bytes) {
  // the attribute is per device and kernel: remember the size set for each (device, kernel) pair and raise it when
  // a launch needs more
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> configured;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  auto it = configured.find({dev, fn});
  if (it != configured.end() && it->second >= bytes) return 0;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return fail(4, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  configured[{dev, fn}] = bytes;
  return 0;
}

int launch_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, void** args, int cluster_x,
               const char* what) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.dynamicSmemBytes = smem;
  lc.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = static_cast<unsigned>(cluster_x);
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  lc.attrs = attr;
  lc.numAttrs = n;
  cudaError_t e = cudaLaunchKernelExC(&lc, fn, args);
  if (e != cudaSuccess) return fail(4, std::string(what) + " launch: " + cudaGetErrorString(e));
  return 0;
}

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
  if (p.K < 1 || p.K > kMaxK) return fail(2, "tcgen05 path supports 1..16 relations per target");
  if (p.NT < 1 || p.NS < 1) return fail(2, "empty node set");
  if (p.n_wtypes < 1 || p.n_wtypes > 2) return fail(2, "one or two weight sets");
  const uintptr_t xa = reinterpret_cast<uintptr_t>(p.x), wa = reinterpret_cast<uintptr_t>(p.w),
                  ya = reinterpret_cast<uintptr_t>(p.y);
  if ((xa | wa | ya) & 15) return fail(2, "x, w and y must be 16-byte aligned");
  if ((p.x_shot_stride | p.x_node_stride | p.x_cg_stride | p.y_shot_stride | p.y_node_stride | p.y_cg_stride) & 7)
    return fail(2, "strides must be multiples of 8 elements");
  if (p.blocked) {
    const int64_t tile_m = kBlockM * mt_for(p.Co);
    if (p.Ci != p.Co || p.x_node_stride % (static_cast<int64_t>(p.Ci) * tile_m) != 0 ||
        p.y_node_stride % (static_cast<int64_t>(p.Co) * tile_m) != 0 || p.x_node_stride / p.Ci < p.shots ||
        p.y_node_stride / p.Co < p.shots)
      return fail(2, "blocked layout needs C_in == C_out and a shot capacity that is a multiple of the tile");
  }
  if (p.head.head_w && (!p.head.logits || (reinterpret_cast<uintptr_t>(p.head.logits) & 7) ||
                        ((p.head.lg_shot_stride | p.head.lg_node_stride) & 1)))
    return fail(2, "head logits must be 8-byte aligned with even strides");
  if (p.epi == kEpiGeluStream) {
    if (p.blocked || p.head.head_w || !p.res_out || (p.res_h && p.res_f32 && !p.res_out16))
      return fail(2, "the GELU stream epilogue takes row layouts, an output stream and (fp32 stream) its bf16 copy");
    if ((reinterpret_cast<uintptr_t>(p.res_h) | reinterpret_cast<uintptr_t>(p.res_out) |
         reinterpret_cast<uintptr_t>(p.res_out16)) & 15 || (p.res_shot_stride | p.res_node_stride) & 7)
      return fail(2, "the residual stream must be 16-byte aligned with strides that are multiples of 8 elements");
  }
  if (p.epi == kEpiAffineSilu && (!p.epi_scale || !p.epi_shift ||
                                  ((reinterpret_cast<uintptr_t>(p.epi_scale) | reinterpret_cast<uintptr_t>(p.epi_shift)) & 7)))
    return fail(2, "the affine + SiLU epilogue needs 8-byte aligned scale and shift vectors");
  return 0;
}

int gmm_tc_make_maps(const GmmProblem& p, GmmMaps* maps) {
  auto enc = get_encode();
  if (!enc) return fail(3, "cuTensorMapEncodeTiled is not available from the CUDA driver");
  if (!p.blocked) {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(p.Ci), static_cast<cuuint64_t>(p.shots),
                          static_cast<cuuint64_t>(p.NS)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(p.x_shot_stride) * 2, static_cast<cuuint64_t>(p.x_node_stride) * 2};
    cuuint32_t box[3] = {kKBlock, static_cast<cuuint32_t>(kBlockM * mt_for(p.Co)), 1};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = enc(&maps->x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(p.x), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(3, "cuTensorMapEncodeTiled(x) failed: " + std::to_string(int(r)));
  } else {
    maps->x = CUtensorMap{};
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
  a.order = p.order;
  a.x = static_cast<const __nv_bfloat16*>(p.x);
  a.x_node_stride = p.x_node_stride;
  a.y = p.y;
  a.y_shot_stride = p.y_shot_stride;
  a.y_node_stride = p.y_node_stride;
  a.y_cg_stride = p.y_cg_stride;
  a.epi = p.epi;
  a.epi_scale = p.epi_scale;
  a.epi_shift = p.epi_shift;
  a.head = p.head;
  a.res_h = p.res_h;
  a.res_f32 = p.res_f32 ? 1 : 0;
  a.res_out = p.res_out;
  a.res_out16 = p.res_out16;
  a.res_shot_stride = p.res_shot_stride;
  a.res_node_stride = p.res_node_stride;
  a.status = status;
  a.timeout_ns = timeout_ns;
  a.tile_counter = p.tile_counter;
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(2 * mt_for(p.Co) * p.Co)) cols <<= 1;
  a.tmem_cols = cols;
  const bool head = p.head.head_w != nullptr;
  // wide tiles: C_out in {64, 96, 128} and C_in <= 128; blocked layout (C_in = C_out) with the GELU epilogues and
  // the head, row layouts with contiguous channels and the store / add / affine + SiLU epilogues
  const bool wide_shape = p.Co >= 64 && p.Co <= kWideM && p.Co % 32 == 0 && (p.Ci == 64 || p.Ci == 96 || p.Ci == 128);
  const bool wide_blocked = p.blocked && p.Ci == p.Co && (p.epi == kEpiGeluInit || p.epi == kEpiGeluResid);
  const bool wide_rows = !p.blocked && !head && p.y_cg_stride == 8 &&
                         (p.epi == kEpiStore || p.epi == kEpiAdd || p.epi == kEpiAffineSilu ||
                          p.epi == kEpiGeluStream);
  if (p.epi == kEpiGeluStream && !(wide_shape && wide_rows))
    return fail(2, "the GELU stream epilogue runs on the wide-tile kernel: C_in, C_out in {64, 96, 128}, row layouts");
  if (wide_shape && (wide_blocked || wide_rows)) {
    const void* wf = wide_kernel_for(p.blocked, p.epi, head, p.Ci);
    if (!wf) return fail(2, "unsupported wide-tile configuration");
    constexpr int wsmem = wide_smem_bytes();
    static_assert(wsmem <= kSmemLimit, "wide-tile kernel exceeds the shared memory per CTA");
    if (int e = allow_smem(wf, wsmem)) return e;
    const int64_t grid = std::min<int64_t>(a.num_tiles, num_sms());
    void* args[] = {const_cast<CUtensorMap*>(&maps.x), const_cast<CUtensorMap*>(&maps.w), &a};
    cudaError_t le = cudaLaunchKernel(wf, dim3(static_cast<unsigned>(grid)),
                                      dim3(kThreads), args, static_cast<size_t>(wsmem), stream);
    if (le != cudaSuccess) return fail(4, std::string("gmm_wide_kernel launch: ") + cudaGetErrorString(le));
    return 0;
  }
  const int smem = smem_bytes_for(p.Co, a.stages);
  KernelFn fn = select_kernel(p.Co, p.blocked, p.epi, head);
  if (!fn) return fail(2, "unsupported C_out / layout / epilogue combination for the tcgen05 path");
  if (int e = allow_smem(reinterpret_cast<const void*>(fn), kSmemLimit)) return e;
  const int64_t grid = std::min<int64_t>(a.num_tiles, num_sms());
  void* args[] = {const_cast<CUtensorMap*>(&maps.x), const_cast<CUtensorMap*>(&maps.w), &a};
  cudaError_t le = cudaLaunchKernel(reinterpret_cast<const void*>(fn), dim3(static_cast<unsigned>(grid)),
                                    dim3(kThreads), args, static_cast<size_t>(smem), stream);
  if (le != cudaSuccess) return fail(4, std::string("gmm_tc_kernel launch: ") + cudaGetErrorString(le));
  return 0;
}

int gmm_tc_tile_shots(int Co) { return kBlockM * mt_for(Co); }

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() { return get_encode(); }

}  // namespace bpc
