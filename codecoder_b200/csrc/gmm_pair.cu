// Bipartite-conv step on CTA pairs (tcgen05 cta_group::2) for the pre-decoder's hidden-128 steps, with the step's
// relation matrices resident in shared memory for the whole launch.
//
//   y[s, n, :] = (y[s, n, :] +) GELU(sum_r x[s, idx[n, r], :] W_{type(n), r}^T)     (cascade_triton.py:5,40 -- the
//                                                                                   same contraction, in the pre-
//                                                                                   decoder's blocked layout)
//
// A cluster of two CTAs is one pair; the pair's tile is one target node x 256 shots.  Each MMA is M = 256 shots x
// N = 128 output channels x K = 16 input channels: the even CTA ("leader") holds shots 0-127 of the tile and output
// channels 0-63 of every W_r, the odd CTA ("peer") shots 128-255 and output channels 64-127, and each CTA's tensor
// memory receives its 128 shots x all 128 channels.  The halves of W (8 relations x 64 x 128 bf16 = 128 KB per CTA)
// are loaded once at launch and never again, so only activations stream: 32 KB per CTA per relation for 4.2 MFLOP
// per SM (131 FLOP/B), against 96 KB for 8.4 MFLOP (87 FLOP/B) when a CTA streams the whole W_r with its tile.  The
// pairs of a data -> check step are split between the two check types (X, Z), each type with its own tile counter
// and its own resident W; a check -> data step has one type.
//
// Activations use the blocked layout with 128-shot blocks: element (s, n, c) at n node_stride + (s / 128) 128 C +
// (c / 8) 1024 + (s % 128) 8 + c % 8, so the 64-channel stage of one CTA's 128 shots is one contiguous 16 KB block,
// loaded by one 2D TMA box (rows of 256 elements) straight into the canonical no-swizzle K-major operand layout
// (8-shot x 16-byte core matrices, SBO = 128 B, LBO = 2 KB).  W halves are loaded as 64-row x 64-channel boxes with
// the 128-byte swizzle (the K-major SW128 layout).
//
// Roles (320 threads per CTA):
//   warp 0     producer.  Leader: takes tiles from its type's counter, publishes each (tile, node, valid relations,
//              sources) to both CTAs' tile rings (the peer's by shared::cluster stores and a remote arrive), and loads
//              its 128 shots' stages.  Peer: reads its ring and loads its stages; its TMA loads count their bytes on
//              the leader's stage barrier (cta_group::2 copies), so one barrier covers both halves of a stage.
//   warp 1     leader: TMEM owner and MMA issuer (cta_group::2 MMAs, commits multicast to both CTAs' stage and
//              accumulator barriers); peer: TMEM owner only.  Accumulators: 2 x 128 fp32 columns per CTA.
//   warps 2-9  epilogue, one shot (TMEM lane) per thread, 64 channels per warp: GELU, residual, bf16 store; in the
//              last check -> data step the X / Z head, the threshold and the XOR into the bit-packed residual (the
//              second channel half finishes the logits in the order the other step kernels use: same bits).
// Every wait is bounded: a timeout sets the status word and the abort flags of both CTAs, and the pair drains and
// leaves.  No copy uses cluster multicast.
//
// Measured on B200 (d = 13, 262,144 shots): 79k syndromes/s against 111k for gmm_wide_kernel, the same bits.  With
// half of the shared memory holding W, 96 KB of activation stages are in flight per SM against 192 KB, and under
// load that does not cover the loads' latency: each SM draws 20 B/clk where the MMAs need 57 and the tensor pipe is
// 32 % busy (54 % for the wide kernel).  The pre-decoder runs it only when BPC_STEP_KERNEL=pair.
//
// The streaming variant (template flag SW, BPC_STEP_KERNEL=pair_stream) keeps no W resident: each of 5 stages holds
// this CTA's two 128-shot blocks of a 512-shot pair tile and its half of the stage's W block (40 KB), 200 KB in
// flight per SM and a sixth fewer bytes per FLOP than the wide kernel (each CTA streams half of W for twice the
// shots).  Measured on the same workload: 92.1k syndromes/s against 109.2k for the wide kernel on the same box, the
// same bits; every stage waits for the slower of the two CTAs' loads, and the partner's loads start only after the
// tile reaches its ring.
#include <algorithm>
#include <cstdio>
#include <string>

#include <cudaTypedefs.h>

#include "bpc_common.cuh"
#include "bpc_internal.h"

namespace bpc {

namespace {

constexpr int kPThreads = 320;
constexpr int kPEpiWarps = 8;
constexpr int kPC = 128;                                // channels in and out
constexpr int kPHalfShots = 128;                        // shots per CTA (the pair's tile: 256)
constexpr int kPTileShots = 2 * kPHalfShots;
constexpr int kPMaxK = 8;                               // relations whose W halves stay resident
constexpr uint32_t kPStageBytes = kPHalfShots * 64 * 2; // one 64-channel block of 128 shots: 16 KB
constexpr int kPStages = 6;
constexpr uint32_t kPWBlock = 64 * 64 * 2;              // 64 output channels x 64 input channels: 8 KB
constexpr uint32_t kPWBytes = kPMaxK * 2 * kPWBlock;    // 128 KB
constexpr int kPRing = 4;
constexpr int kPBlockElems = kPHalfShots * kPC;         // one 128-shot block of one node: 16,384 elements
constexpr int kPCgElems = kPHalfShots * 8;              // one channel group of a block: 1,024 elements
constexpr int kPRowElems = 256;                         // TMA rows of the activation map
constexpr int kPStageRows = static_cast<int>(kPStageBytes / (kPRowElems * 2));   // 32
constexpr uint32_t kPAccCols = kPC;                     // one accumulator: 128 fp32 columns

struct PairRing {
  long long tile;      // -1: no more tiles
  int n;
  uint32_t vm;         // relations with a source in [0, NS)
  int src[kPMaxK];
};
static_assert(sizeof(PairRing) == 48, "ring entry layout");

// Shared memory of one CTA (offsets from a 1024-byte aligned base).  Resident-W variant: the W halves, then 6 stages
// of one 128-shot activation block.  Streaming variant (STREAMW): no resident W; 5 stages, each this CTA's two
// 128-shot activation blocks (the pair's tile is 512 shots: two M = 256 MMAs per K step, one per block pair) and its
// half of the step's W block for that stage (64 output channels x 64 input channels), 40 KB.
constexpr uint32_t kPOffW = 0;                          // resident variant: the W halves
constexpr int kSSub = 2;
constexpr int kSStages = 5;
constexpr uint32_t kSStageBytes = kSSub * kPStageBytes + kPWBlock;
template <bool SW>
struct PairLayout {
  static constexpr int sub = SW ? kSSub : 1;                        // 128-shot blocks per CTA per tile
  static constexpr int stages = SW ? kSStages : kPStages;
  static constexpr uint32_t stage_bytes = SW ? kSStageBytes : kPStageBytes;
  static constexpr uint32_t off_stages = SW ? 0 : kPWBytes;
  static constexpr uint32_t off_bars = off_stages + stages * stage_bytes;
  static constexpr int num_bars = 2 * stages + 2 + 2 + 2 * kPRing + 1 + 1 + 16;   // full, empty, accf, acce, tfull,
                                                                                   // tempty, drain, wfull, hstore
                                                                                   // (quarter x acc x block)
  static constexpr uint32_t off_ring = off_bars + 512;
  static constexpr uint32_t off_misc = off_ring + kPRing * sizeof(PairRing);
  static constexpr uint32_t smem_bytes = 1024 + off_misc + 64;
  static constexpr uint32_t tmem_cols = 2 * sub * kPAccCols;        // two accumulator sets
  static constexpr int tile_shots = sub * kPTileShots;
  static_assert(num_bars * 8 <= 512, "barrier area");
  static_assert(smem_bytes <= 232448, "pair kernel exceeds the shared memory per CTA");
};

struct PairArgs {
  const int32_t* idx;        // (NT, K) sources
  int NT, NS, K;
  const int32_t* order;      // type-major processing order: n_type0 targets of type 0, then the others (null:
                             // identity, one type)
  int n_type0;
  int pairs_type0;           // pairs serving type 0; the rest serve type 1
  int64_t shots;             // valid shots of the pass
  int64_t sblocks;           // 256-shot blocks of the pass
  int64_t x_node_rows;       // activation rows (of 256 elements) per source node
  __nv_bfloat16* y;
  int64_t y_node_stride;     // elements
  HeadEpilogue head;
  int* status;
  uint64_t timeout_ns;
  unsigned long long* counters;   // [2] tile counters (zero at launch)
};

// A ring entry as published (volatile reads: the entry may have been written by the other CTA of the pair).
__device__ __forceinline__ PairRing load_ring(const PairRing* p) {
  const volatile PairRing* v = p;
  PairRing e;
  e.tile = v->tile;
  e.n = v->n;
  e.vm = v->vm;
#pragma unroll
  for (int r = 0; r < kPMaxK; ++r) e.src[r] = v->src[r];
  return e;
}

// One epilogue warp of either CTA is done with an accumulator (the count is on the leader's barrier).
__device__ __forceinline__ void release_acc(bool leader, uint64_t* bar) {
  if (leader) mbar_arrive(smem_u32(bar));
  else mbar_arrive_remote(map_to_cta(smem_u32(bar), 0));
}

__device__ __forceinline__ void pair_abort(volatile int* abort_flag, uint32_t peer_abort_cluster) {
  *abort_flag = 1;
  st_cluster_u32(peer_abort_cluster, 1u);
}

template <int EPI, bool HEAD, bool SW>
__global__ void __launch_bounds__(kPThreads, 1)
    gmm_pair_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, const PairArgs a) {
  using Lay = PairLayout<SW>;
  constexpr int kSub = Lay::sub;
  constexpr int kStages = Lay::stages;
  constexpr bool kLoadY = EPI == kEpiGeluResid;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Lay::off_bars);
  uint64_t* full = bars;                          // leader: both halves of a stage landed
  uint64_t* empty = bars + kStages;               // both CTAs: the MMAs that read a stage are done
  uint64_t* accf = empty + kStages;               // both CTAs: an accumulator is complete
  uint64_t* acce = accf + 2;                      // leader: both CTAs' epilogues drained an accumulator
  uint64_t* tfull = acce + 2;                     // both CTAs: a ring entry is published
  uint64_t* tempty = tfull + kPRing;              // leader: every consumer of both CTAs released a ring entry
  uint64_t* drain = tempty + kPRing;
  uint64_t* wfull = drain + 1;
  uint64_t* hstore = wfull + 1;                   // head: quarter q's first channel half is stored (per acc, block)
  PairRing* ring = reinterpret_cast<PairRing*>(smem + Lay::off_ring);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Lay::off_misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Lay::off_misc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const uint32_t peer = rank ^ 1u;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int type = pair < a.pairs_type0 ? 0 : 1;
  const int n_t = type == 0 ? a.n_type0 : a.NT - a.n_type0;
  const int t_base = type == 0 ? 0 : a.n_type0;
  const long long num_tiles = static_cast<long long>(n_t) * a.sblocks;
  const uint32_t peer_abort = map_to_cta(smem_u32(const_cast<int*>(abort_flag)), peer);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(smem_u32(&full[i]), 1);
      mbar_init(smem_u32(&empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&accf[i]), 1);
      mbar_init(smem_u32(&acce[i]), 2 * kPEpiWarps);
    }
    for (int i = 0; i < kPRing; ++i) {
      mbar_init(smem_u32(&tfull[i]), 1);
      mbar_init(smem_u32(&tempty[i]), 1 + kPEpiWarps + 1 + kPEpiWarps);
    }
    mbar_init(smem_u32(drain), 1);
    mbar_init(smem_u32(wfull), 1);
    for (int i = 0; i < 16; ++i) mbar_init(smem_u32(&hstore[i]), 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
    // this CTA's half of every W_r of its type, resident for the launch: block (r, kb) = output channels
    // 64 rank .. + 63 of W_{type, r}, input channels 64 kb .. + 63 (the streaming variant loads them per stage)
    if (!SW && n_t > 0) {
      mbar_arrive_expect_tx(smem_u32(wfull), static_cast<uint32_t>(a.K) * 2 * kPWBlock);
      for (int r = 0; r < a.K; ++r)
        for (int kb = 0; kb < 2; ++kb)
          tma_load_3d(smem_u32(smem + kPOffW + (2 * r + kb) * kPWBlock), &tmW, kb * 64, r,
                      type * kPC + static_cast<int>(rank) * 64, smem_u32(wfull));
    } else {
      mbar_arrive(smem_u32(wfull));
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), Lay::tmem_cols);
    tmem_relinquish_pair();
  }
  bool ok = true;
  if (threadIdx.x == 0) ok = mbar_wait(smem_u32(wfull), 0, abort_flag, a.status, a.timeout_ns);
  if (!__syncthreads_and(ok)) *abort_flag = 1;
  tc_fence_before();
  // both CTAs: barriers initialised, W resident, TMEM allocated before any remote arrive or pair MMA
  cluster_arrive_release();
  cluster_wait_acquire();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  {
    // either CTA's failure before the loop stops both
    uint32_t pv;
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(pv) : "r"(peer_abort) : "memory");
    if (pv) *abort_flag = 1;
  }
  __syncthreads();


  if (warp == 0) {
    // ------------------------------------------------------------------ producers
    if (lane == 0 && !*abort_flag) {
      int stage = 0;
      uint32_t phase = 0;
      int rslot = 0;
      uint32_t rphase = 0;
      uint32_t armed = 0, armed_parity = 0;
      bool good = true;
      if (leader) {
        unsigned long long* counter = a.counters + type;
        // tiles are taken two ahead, so the index rows of the next tile have arrived by the time it starts
        auto take = [&]() -> PairRing {
          PairRing e;
          const long long t = n_t > 0 ? static_cast<long long>(atomicAdd(counter, 1ull)) : num_tiles;
          e.tile = t < num_tiles ? t : -1;
          e.n = 0;
          e.vm = 0;
          const int i = t_base + static_cast<int>((e.tile >= 0 ? e.tile : 0) % (n_t > 0 ? n_t : 1));
          e.n = e.tile >= 0 ? (a.order ? __ldg(a.order + i) : i) : 0;
          const int32_t* row = a.idx + static_cast<int64_t>(e.n) * a.K;
#pragma unroll
          for (int r = 0; r < kPMaxK; ++r) e.src[r] = (e.tile >= 0 && r < a.K) ? __ldg(row + r) : -1;
          return e;
        };
        auto finish = [&](PairRing& e) {
          e.vm = 0;
#pragma unroll
          for (int r = 0; r < kPMaxK; ++r)
            if (e.src[r] >= 0 && e.src[r] < a.NS) e.vm |= 1u << r;
        };
        PairRing nxt1 = take();
        PairRing nxt2 = nxt1.tile >= 0 ? take() : nxt1;
        while (good) {
          PairRing e = nxt1;
          finish(e);
          if (!mbar_wait_cl(smem_u32(&tempty[rslot]), rphase ^ 1u, abort_flag, a.status, a.timeout_ns)) {
            pair_abort(abort_flag, peer_abort);
            break;
          }
          // publish to both CTAs: own ring, then the peer's by shared::cluster stores and a release arrive
          ring[rslot] = e;
          const uint32_t pr = map_to_cta(smem_u32(&ring[rslot]), peer);
          const uint32_t* ew = reinterpret_cast<const uint32_t*>(&e);
#pragma unroll
          for (int w = 0; w < 12; ++w) st_cluster_u32(pr + 4 * w, ew[w]);
          mbar_arrive(smem_u32(&tfull[rslot]));
          mbar_arrive_remote(map_to_cta(smem_u32(&tfull[rslot]), peer));
          if (++rslot == kPRing) {
            rslot = 0;
            rphase ^= 1u;
          }
          if (e.tile < 0) break;
          nxt1 = nxt2;
          if (nxt2.tile >= 0) nxt2 = take();
          const int64_t sb = e.tile / n_t;
          for (int r = 0; r < a.K && good; ++r) {
            if (!(e.vm & (1u << r))) continue;
            for (int kb = 0; kb < 2; ++kb) {
              if (!mbar_wait_cl(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, a.status, a.timeout_ns)) {
                pair_abort(abort_flag, peer_abort);
                good = false;
                break;
              }
              const uint32_t fb = smem_u32(&full[stage]);
              mbar_arrive_expect_tx(fb, 2 * Lay::stage_bytes);      // both CTAs' halves
              uint8_t* sdst = smem + Lay::off_stages + stage * Lay::stage_bytes;
#pragma unroll
              for (int u = 0; u < kSub; ++u) {
                // this CTA's 128-shot block u of the tile: block 2 (sub sb + u) + rank of the node
                const int64_t row = e.src[r] * a.x_node_rows +
                                    (2 * (kSub * sb + u)) * (kPBlockElems / kPRowElems) + kb * kPStageRows;
                tma_load_2d(smem_u32(sdst + u * kPStageBytes), &tmX, 0, static_cast<int32_t>(row), fb);
              }
              if (SW) tma_load_3d(smem_u32(sdst + kSub * kPStageBytes), &tmW, kb * 64, r, type * kPC, fb);
              armed |= 1u << stage;
              armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
              if (++stage == kStages) {
                stage = 0;
                phase ^= 1u;
              }
            }
          }
        }
        if (!good || *abort_flag) {
          // drain: the stages armed last may still be landing (both halves count on these barriers)
          for (int i = 0; i < kStages; ++i)
            if (armed & (1u << i)) {
              const uint32_t par = (armed_parity >> i) & 1u;
              const uint64_t t0 = globaltimer_ns();
              while (!mbar_try_wait(smem_u32(&full[i]), par) && globaltimer_ns() - t0 < a.timeout_ns) {
              }
            }
        }
      } else {
        bool issued = false;
        while (good) {
          if (!mbar_wait_cl(smem_u32(&tfull[rslot]), rphase, abort_flag, a.status, a.timeout_ns)) {
            pair_abort(abort_flag, peer_abort);
            break;
          }
          const PairRing e = load_ring(&ring[rslot]);
          mbar_arrive_remote(map_to_cta(smem_u32(&tempty[rslot]), 0));
          if (++rslot == kPRing) {
            rslot = 0;
            rphase ^= 1u;
          }
          if (e.tile < 0) break;
          const int64_t sb = e.tile / n_t;
          for (int r = 0; r < a.K && good; ++r) {
            if (!(e.vm & (1u << r))) continue;
            for (int kb = 0; kb < 2; ++kb) {
              if (!mbar_wait_cl(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, a.status, a.timeout_ns)) {
                pair_abort(abort_flag, peer_abort);
                good = false;
                break;
              }
              const uint32_t fb = map_to_cta(smem_u32(&full[stage]), 0);
              uint8_t* sdst = smem + Lay::off_stages + stage * Lay::stage_bytes;
#pragma unroll
              for (int u = 0; u < kSub; ++u) {
                const int64_t row = e.src[r] * a.x_node_rows +
                                    (2 * (kSub * sb + u) + 1) * (kPBlockElems / kPRowElems) + kb * kPStageRows;
                tma_load_2d_pair(smem_u32(sdst + u * kPStageBytes), &tmX, 0, static_cast<int32_t>(row), fb);
              }
              if (SW) tma_load_3d_pair(smem_u32(sdst + kSub * kPStageBytes), &tmW, kb * 64, r, type * kPC + 64, fb);
              issued = true;
              if (++stage == kStages) {
                stage = 0;
                phase ^= 1u;
              }
            }
          }
        }
        if ((!good || *abort_flag) && issued) {
          // the peer's copies count on the leader's barriers: give any still in flight time to land
          const uint64_t t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 200000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (leader)
    if (leader && lane == 0 && !*abort_flag) {
      constexpr uint32_t idesc = idesc_bf16_f32(2 * kPHalfShots, kPC);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      int rslot = 0;
      uint32_t rphase = 0;
      bool good = true;
      const uint32_t w_base = smem_u32(smem + kPOffW);   // resident variant only
      while (good) {
        if (!mbar_wait(smem_u32(&tfull[rslot]), rphase, abort_flag, a.status, a.timeout_ns)) {
          pair_abort(abort_flag, peer_abort);
          break;
        }
        const PairRing en = load_ring(&ring[rslot]);
        const long long tile = en.tile;
        const uint32_t vm = en.vm;
        mbar_arrive(smem_u32(&tempty[rslot]));
        if (++rslot == kPRing) {
          rslot = 0;
          rphase ^= 1u;
        }
        if (tile < 0) break;
        if (!mbar_wait_cl(smem_u32(&acce[acc]), acc_phase ^ 1u, abort_flag, a.status, a.timeout_ns)) {
          pair_abort(abort_flag, peer_abort);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc) * kSub * kPAccCols;
        uint32_t accumulate = 0;
        for (int r = 0; r < a.K && good; ++r) {
          if (!(vm & (1u << r))) continue;
#pragma unroll
          for (int kb = 0; kb < 2; ++kb) {
            if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, a.status, a.timeout_ns)) {
              pair_abort(abort_flag, peer_abort);
              good = false;
              break;
            }
            tc_fence_after();
            const uint32_t sbase = smem_u32(smem + Lay::off_stages + stage * Lay::stage_bytes);
            const uint64_t bd = SW ? sdesc_k_sw128(sbase + kSub * kPStageBytes)
                                   : sdesc_k_sw128(w_base + (2 * r + kb) * kPWBlock);
            // each block's accumulator takes the same MMA sequence (relations, k-blocks, 16-channel steps in order)
#pragma unroll
            for (int u = 0; u < kSub; ++u) {
              const uint64_t ad = sdesc_k_none(sbase + u * kPStageBytes, 2 * kPCgElems, 128);
#pragma unroll
              for (int k = 0; k < 4; ++k)
                tc_mma_ss_pair(d_tmem + u * kPAccCols, ad + static_cast<uint64_t>((k * 2 * 2 * kPCgElems) >> 4),
                               bd + static_cast<uint64_t>((k * 32) >> 4), idesc, (accumulate | k) ? 1u : 0u);
            }
            accumulate = 1;
            tc_commit_pair(smem_u32(&empty[stage]), 3);   // the stage is free in both CTAs
            if (++stage == kStages) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
        if (!good) break;
        tc_commit_pair(smem_u32(&accf[acc]), 3);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      tc_commit_pair(smem_u32(drain), 1);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(smem_u32(drain), 0) && globaltimer_ns() - t0 < a.timeout_ns) {
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..9, both CTAs)
    const int q = warp & 3;                   // TMEM lane quarter: shots 32 q .. 32 q + 31 of this CTA's half
    const int e = warp - 2;
    const int h = e >> 2;                     // channels 64 h .. 64 h + 63
    int acc = 0;
    uint32_t acc_phase = 0;
    int rslot = 0;
    uint32_t rphase = 0;
    // in the head step the second channel half keeps its accumulator until the logits are done, so the first half
    // is never more than one tile (the other accumulator) ahead of it on the hand-over barriers
    const bool late_release = HEAD && h == 1;
    while (!*abort_flag) {
      if (!__all_sync(0xffffffffu, mbar_wait_cl(smem_u32(&tfull[rslot]), rphase, abort_flag, a.status, a.timeout_ns))) {
        if (lane == 0) pair_abort(abort_flag, peer_abort);
        break;
      }
      const PairRing en = load_ring(&ring[rslot]);
      const long long tile = en.tile;
      const int n = en.n;
      const uint32_t vm = en.vm;
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(smem_u32(&tempty[rslot]));
        else mbar_arrive_remote(map_to_cta(smem_u32(&tempty[rslot]), 0));
      }
      if (++rslot == kPRing) {
        rslot = 0;
        rphase ^= 1u;
      }
      if (tile < 0) break;
      bool bail = false;
#pragma unroll 1
      for (int u = 0; u < kSub; ++u) {
        // this CTA's 128-shot block u of the tile (kSub blocks per CTA, interleaved with the partner's)
        const int64_t s_half = (tile / n_t) * Lay::tile_shots + u * kPTileShots + static_cast<int64_t>(rank) * kPHalfShots;
        const int sl = 32 * q + lane;           // this thread's shot within the CTA's half
        const bool ok = s_half + sl < a.shots;
        __nv_bfloat16* const yb = a.y + static_cast<int64_t>(n) * a.y_node_stride + (s_half / kPHalfShots) * kPBlockElems;
        __nv_bfloat16* const yc = yb + (8 * h) * kPCgElems + sl * 8;   // channel group 8 h of this shot; + g kPCgElems
        uint4 rb[kLoadY ? 8 : 1];
        if (kLoadY && ok) {
  #pragma unroll
          for (int g = 0; g < 8; ++g) rb[g] = *reinterpret_cast<const uint4*>(yc + g * kPCgElems);
        }
        if (u == 0 &&
            !__all_sync(0xffffffffu, mbar_wait_cl(smem_u32(&accf[acc]), acc_phase, abort_flag, a.status, a.timeout_ns))) {
          if (lane == 0) pair_abort(abort_flag, peer_abort);
          bail = true;
          break;
        }
        tc_fence_after();
        float v[64];
        {
          const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                 static_cast<uint32_t>(acc * kSub + u) * kPAccCols + 64 * h;
          float* v0 = v;
          float* v1 = v + 32;
          if (vm) {
            tmem_ld32(taddr, *reinterpret_cast<float(*)[32]>(v0));
            tmem_ld32(taddr + 32, *reinterpret_cast<float(*)[32]>(v1));
          } else {
  #pragma unroll
            for (int i = 0; i < 64; ++i) v[i] = 0.f;
          }
        }
        // the accumulator is free for the pair's next tile once both CTAs' eight warps have read it
        tc_fence_before();
        __syncwarp();
        if (lane == 0 && !late_release && u == kSub - 1) release_acc(leader, &acce[acc]);
        uint32_t outw[32];
  #pragma unroll
        for (int g = 0; g < 8; ++g) {
          uint4 u;
          uint32_t* o = reinterpret_cast<uint32_t*>(&u);
          const uint32_t* hr = reinterpret_cast<const uint32_t*>(&rb[kLoadY ? g : 0]);
  #pragma unroll
          for (int e4 = 0; e4 < 4; ++e4) {
            uint64_t xx = gelu_tanh_fast2(f2_pack(v[8 * g + 2 * e4], v[8 * g + 2 * e4 + 1]));
            if (kLoadY) xx = f2_add(xx, bf2_to_f2(hr[e4]));
            o[e4] = f2_to_bf2(xx);
            outw[4 * g + e4] = o[e4];
          }
          if (ok) *reinterpret_cast<uint4*>(yc + g * kPCgElems) = u;
        }
        if (HEAD) {
          // logits over the 128 stored channels in order (channel pairs, groups 0 .. 15): the first channel half is
          // read back once its warp has stored it, the second is this warp's own
          if (h == 0) {
            __threadfence_block();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&hstore[(2 * q + acc) * kSub + u]));
          } else {
            if (!__all_sync(0xffffffffu,
                            mbar_wait(smem_u32(&hstore[(2 * q + acc) * kSub + u]), acc_phase, abort_flag, a.status,
                                      a.timeout_ns))) {
              if (lane == 0) pair_abort(abort_flag, peer_abort);
              bail = true;
              break;
            }
            uint64_t lg0 = 0, lg1 = 0;
            const __nv_bfloat16* y0 = yb + sl * 8;
  #pragma unroll
            for (int g = 0; g < 8; ++g) {
              uint4 u = make_uint4(0, 0, 0, 0);
              if (ok) u = __ldcg(reinterpret_cast<const uint4*>(y0 + g * kPCgElems));   // through L2
              const uint32_t* o = reinterpret_cast<const uint32_t*>(&u);
  #pragma unroll
              for (int e4 = 0; e4 < 4; ++e4) {
                const uint64_t f = bf2_to_f2(o[e4]);
                const int col = g * 8 + 2 * e4;
                lg0 = f2_fma(f, *reinterpret_cast<const uint64_t*>(a.head.head_w + col), lg0);
                lg1 = f2_fma(f, *reinterpret_cast<const uint64_t*>(a.head.head_w + kPC + col), lg1);
              }
            }
  #pragma unroll
            for (int g = 0; g < 8; ++g)
  #pragma unroll
              for (int e4 = 0; e4 < 4; ++e4) {
                const uint64_t f = bf2_to_f2(outw[4 * g + e4]);
                const int col = 64 + g * 8 + 2 * e4;
                lg0 = f2_fma(f, *reinterpret_cast<const uint64_t*>(a.head.head_w + col), lg0);
                lg1 = f2_fma(f, *reinterpret_cast<const uint64_t*>(a.head.head_w + kPC + col), lg1);
              }
            const float l0 = f2_lo(lg0) + f2_hi(lg0) + __ldg(a.head.head_b);
            const float l1 = f2_lo(lg1) + f2_hi(lg1) + __ldg(a.head.head_b + 1);
            if (ok) {
              float2* lp = reinterpret_cast<float2*>(a.head.logits + (s_half + sl) * a.head.lg_shot_stride +
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
                  atomicXor(a.head.res_bits + static_cast<int64_t>(c) * a.head.res_words + ((s_half + 32 * q) >> 5), msk);
              }
            }
            __syncwarp();
            if (lane == 0 && u == kSub - 1) release_acc(leader, &acce[acc]);
          }
        }
      }
      if (bail) break;
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  // every remote access between the two CTAs is done, and the leader has seen its last MMA complete, before either
  // CTA frees its tensor memory or leaves
  tc_fence_before();
  __syncthreads();
  cluster_arrive_release();
  cluster_wait_acquire();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Lay::tmem_cols);
  }
}

using PairFn = void (*)(CUtensorMap, CUtensorMap, PairArgs);

template <bool SW>
PairFn pair_kernel_for(int epi, bool head) {
  if (epi == kEpiGeluInit)
    return head ? &gmm_pair_kernel<kEpiGeluInit, true, SW> : &gmm_pair_kernel<kEpiGeluInit, false, SW>;
  if (epi == kEpiGeluResid)
    return head ? &gmm_pair_kernel<kEpiGeluResid, true, SW> : &gmm_pair_kernel<kEpiGeluResid, false, SW>;
  return nullptr;
}

bool pair_shape_ok(const GmmProblem& p) {
  return p.blocked && p.Ci == kPC && p.Co == kPC && p.K >= 1 && p.K <= kPMaxK && p.n_wtypes >= 1 && p.n_wtypes <= 2;
}

}  // namespace

bool gmm_pair_supported(const GmmProblem& p) {
  return pair_shape_ok(p) && (p.epi == kEpiGeluInit || p.epi == kEpiGeluResid);
}

int gmm_pair_make_maps(const GmmProblem& p, GmmMaps* maps) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(3, "cuTensorMapEncodeTiled is not available from the CUDA driver");
  if (!pair_shape_ok(p)) return fail(2, "the pair kernel takes blocked hidden-128 steps with at most 8 relations");
  if (p.x_node_stride % kPRowElems != 0) return fail(2, "pair kernel: node stride is not a multiple of 256 elements");
  {
    const cuuint64_t rows = static_cast<cuuint64_t>(p.NS) * static_cast<cuuint64_t>(p.x_node_stride / kPRowElems);
    if (rows > 0x7fffffffull) return fail(2, "pair kernel: activation buffer too large for 32-bit TMA rows");
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(kPRowElems), rows};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(kPRowElems) * 2};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(kPRowElems), static_cast<cuuint32_t>(kPStageRows)};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(&maps->x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(p.x), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(3, "cuTensorMapEncodeTiled(pair x) failed: " + std::to_string(int(r)));
  }
  {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(p.Ci), static_cast<cuuint64_t>(p.K),
                          static_cast<cuuint64_t>(p.Co) * p.n_wtypes};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(p.Ci) * 2, static_cast<cuuint64_t>(p.K) * p.Ci * 2};
    cuuint32_t box[3] = {64, 1, 64};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = enc(&maps->w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(p.w), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(3, "cuTensorMapEncodeTiled(pair w) failed: " + std::to_string(int(r)));
  }
  return 0;
}

int gmm_pair_launch(const GmmProblem& p, const GmmMaps& maps, const int32_t* type_order, int n_type0,
                    unsigned long long* counters, int* status, uint64_t timeout_ns, cudaStream_t stream,
                    bool stream_w) {
  if (!gmm_pair_supported(p)) return fail(2, "the pair kernel takes blocked hidden-128 steps with at most 8 relations");
  if (p.shots <= 0) return 0;
  if (!counters) return fail(2, "the pair kernel needs two tile counters");
  const uintptr_t xa = reinterpret_cast<uintptr_t>(p.x), ya = reinterpret_cast<uintptr_t>(p.y);
  if ((xa | ya) & 15) return fail(2, "pair kernel: activation buffers must be 16-byte aligned");
  if (p.x_node_stride % (2 * kPBlockElems) || p.y_node_stride % (2 * kPBlockElems) ||
      p.x_node_stride / kPC < p.shots || p.y_node_stride / kPC < p.shots)
    return fail(2, "pair kernel: the shot capacity must be a multiple of 256 and hold the pass");
  if (p.head.head_w && (!p.head.logits || (reinterpret_cast<uintptr_t>(p.head.logits) & 7) ||
                        ((p.head.lg_shot_stride | p.head.lg_node_stride) & 1)))
    return fail(2, "head logits must be 8-byte aligned with even strides");
  const int n0 = p.n_wtypes > 1 ? n_type0 : p.NT;
  if (n0 < 0 || n0 > p.NT) return fail(2, "pair kernel: invalid type split");
  const int sms = num_sms();
  int pairs = std::max(1, sms / 2);
  // pairs per type in proportion to the type's targets (every type that has targets gets at least one pair)
  int pairs0 = pairs;
  if (p.n_wtypes > 1) {
    if (pairs < 2) pairs = 2;
    pairs0 = static_cast<int>((static_cast<int64_t>(pairs) * n0 + p.NT / 2) / p.NT);
    pairs0 = std::min(std::max(pairs0, n0 > 0 ? 1 : 0), pairs - (n0 < p.NT ? 1 : 0));
  }
  PairArgs a;
  a.idx = p.idx;
  a.NT = p.NT;
  a.NS = p.NS;
  a.K = p.K;
  a.order = p.n_wtypes > 1 ? type_order : p.order;
  a.n_type0 = n0;
  a.pairs_type0 = pairs0;
  a.shots = p.shots;
  const int tile_shots = stream_w ? PairLayout<true>::tile_shots : PairLayout<false>::tile_shots;
  a.sblocks = (p.shots + tile_shots - 1) / tile_shots;
  a.x_node_rows = p.x_node_stride / kPRowElems;
  a.y = static_cast<__nv_bfloat16*>(p.y);
  a.y_node_stride = p.y_node_stride;
  a.head = p.head;
  a.status = status;
  a.timeout_ns = timeout_ns;
  a.counters = counters;
  PairFn fn = stream_w ? pair_kernel_for<true>(p.epi, p.head.head_w != nullptr)
                       : pair_kernel_for<false>(p.epi, p.head.head_w != nullptr);
  if (!fn) return fail(2, "unsupported pair-kernel epilogue");
  const uint32_t smem_bytes = stream_w ? PairLayout<true>::smem_bytes : PairLayout<false>::smem_bytes;
  if (int e = allow_smem(reinterpret_cast<const void*>(fn), static_cast<int>(smem_bytes))) return e;
  cudaError_t me = cudaMemsetAsync(counters, 0, 2 * sizeof(unsigned long long), stream);
  if (me != cudaSuccess) return fail(4, std::string("cudaMemsetAsync: ") + cudaGetErrorString(me));
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(static_cast<unsigned>(2 * pairs));
  lc.blockDim = dim3(kPThreads);
  lc.dynamicSmemBytes = smem_bytes;
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  void* args[] = {const_cast<CUtensorMap*>(&maps.x), const_cast<CUtensorMap*>(&maps.w), &a};
  cudaError_t le = cudaLaunchKernelExC(&lc, reinterpret_cast<const void*>(fn), args);
  if (le != cudaSuccess) return fail(4, std::string("gmm_pair_kernel launch: ") + cudaGetErrorString(le));
  return 0;
}

int gmm_pair_tile_shots() { return kPHalfShots; }

}  // namespace bpc
