// The boundary between two Cascade bottleneck blocks in one pass (eval, H = 512, bottleneck 128): what the reference
// computes from the end of one Block's bipartite convolution to the input of the next Block's convolution
// (training/bb/ising_compare/bb/cascade_net.py:236-259, `branch` and the residual of `forward`):
//
//   u  = bf16(x3 W_up^T)                       the block's up projection (bf16 output, as under autocast)
//   h' = scale_h h + scale_u u                 the residual stream (fp32)
//   x1 = bf16(SiLU(a1 h' + b1))                the next block's BN1 (folded to scale and shift) + SiLU
//   x2 = bf16(SiLU(a2 (x1 W_down^T) + b2))     the next block's down projection + BN2 (folded) + SiLU
//
// Unfused these are four launches that move ~8.5 KB per node row through HBM (u and x1 are written and read back);
// here one kernel reads x3 (256 B) and h (2 KB) and writes h' (2 KB) and x2 (256 B) per row.  After the last block
// the same kernel writes x1 (the stream after bn_out + SiLU) instead of running a down projection.  For the first
// block of a network (token mode) h is not read at all: it is the embedding table's row for each node's detector
// token (CascadeBB.tokens, cascade_net.py:310-312), and cascade_stem_kernel below writes that block's BN1 + SiLU.
//
// The arithmetic is the unfused path's, in the same order: the MMAs accumulate in K order; u is rounded to bf16
// before the residual; h' = fmaf(scale_u, u, scale_h h); x1 = SiLU, rounded to bf16; x2 = the op
// kernel's affine + SiLU epilogue.  SiLU is x/2 + x/2 tanh(x/2) on the hardware tanh wherever its result is
// rounded to bf16 right after (here and in bpc_residual_affine_silu alike).
//
// One CTA per SM, persistent over 128-row tiles.  Roles (480 threads):
//   warp 0      TMA: the x3 tile (128 rows x 128 channels), W_up in quarters of 128 output channels, W_down in
//               chunks of 64 input channels
//   warp 1      TMEM (512 columns: two 128-column up accumulators, two down accumulators) and the MMAs, one thread:
//               per tile up(q) for the 4 quarters (8 MMAs of M128 N128 K16 each) interleaved with down(kc) for the 8
//               chunks (4 MMAs each) in the order the middle stage produces x1
//   warps 2-9   the middle stage, two warps per TMEM lane quarter (one row per thread, one 32-channel half of every
//               64-channel chunk per warp): h arrives by TMA in 128-row x 32-channel fp32 boxes (128-byte swizzle,
//               three chunks in flight), u comes from TMEM, h' goes back into the same box, x1 goes into the swizzled
//               K-major operand of the down MMA (after the last block: a box for the TMA store); each warp signals
//               its part of a chunk on mbarriers (no CTA barrier), so the warps run ahead of one another
//   warps 10-13 the down epilogue: TMEM -> BN2 + SiLU -> bf16 rows of x2
//   warp 14     the stores and the h loads: once the middle stage has finished a chunk it stores h' (and x1 after the
//               last block) by TMA and, once the stores have read the boxes, refills the slot with the chunk three ahead
//               (token mode: hands the slot back to the middle stage without a load)
// Every wait is bounded (mbar_wait); on a timeout the status word is set, each role leaves its loop, waits (bounded)
// for the copies and MMAs it issued, and the CTA returns.
#include <algorithm>
#include <string>

#include <cudaTypedefs.h>

#include "bpc.h"
#include "bpc_common.cuh"
#include "bpc_internal.h"

namespace bpc {
namespace {

constexpr int kBH = 512;                // residual stream channels
constexpr int kBB = 128;                // bottleneck channels
constexpr int kBRows = 128;             // rows per tile (MMA M)
constexpr int kBThreads = 480;
constexpr int kMidWarp0 = 2, kMidWarps = 8, kEpiWarp0 = 10, kStoreWarp = 14;
constexpr int kHSlots = 3;              // h chunks in flight
constexpr uint32_t kBox = kBRows * 128;                 // one 128-row box of 128-byte rows: 16 KB
constexpr uint32_t kOffX3 = 0;                          // 2 boxes: the tile's 128 channels of x3
constexpr uint32_t kOffWup = kOffX3 + 2 * kBox;         // 2 boxes: one quarter of W_up (128 outputs x 128 inputs)
constexpr uint32_t kOffWdn = kOffWup + 2 * kBox;        // 2 slots: a chunk of W_down (128 outputs x 64 inputs)
constexpr uint32_t kOffX1 = kOffWdn + 2 * kBox;         // 2 slots: a chunk of x1 (128 rows x 64 channels)
constexpr uint32_t kOffH = kOffX1 + 2 * kBox;           // 3 slots x 2 boxes: a chunk of h (128 rows x 64 fp32)
constexpr uint32_t kOffBar = kOffH + kHSlots * 2 * kBox;
constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;   // + barriers, + slack for the 1024-byte alignment
static_assert(kSmemBytes <= 232448, "boundary kernel exceeds the shared memory per CTA");

// mbarrier slots
enum : int {
  kX3F = 0, kX3E = 1, kWuF = 2, kWuE = 3, kWdF = 4, kWdE = 6, kDuF = 8, kDuE = 10, kX1F = 12, kX1E = 14, kHF = 16,
  kDdF = 19, kDdE = 21, kDrain = 23, kDone = 24, kNumBars = 27
};
// kX1E: the x1 slot is free again -- after the down MMAs read it, or (last block) after its store read it
// kDone: the middle stage has finished the chunk in an h slot (h' and x1 written; one arrival per middle warp)

struct BoundaryArgs {
  float scale_h, scale_u;
  const float* a1;
  const float* b1;
  const float* a2;
  const float* b2;
  __nv_bfloat16* y;             // down mode: x2 (rows, 128)
  int64_t rows;
  int num_tiles;
  int store_h;                  // write h' (through the h_out map)
  int store_x1;                 // x1 mode: write x1 (through the y map)
  // token mode (the first block of a network): h is the embedding of each row's detector token, h[row] =
  // E[tbase[node] + det[shot, gidx[node]]] (gidx = D: no detector), row = shot N + node; no h is read from memory
  int tokens;
  const uint8_t* det;           // (B, D)
  const int32_t* gidx;          // (N)
  const int32_t* tbase;         // (N)
  const float* E;               // (5, 512)
  int D, N;
  int* status;
  uint64_t timeout_ns;
};

// Token of a row of the network's stream (token mode); rows past the batch take the absent token.
__device__ __forceinline__ int row_token(const BoundaryArgs& a, int64_t row) {
  if (row >= a.rows) return 4;
  const int64_t shot = row / a.N;
  const int node = static_cast<int>(row - shot * a.N);
  const int g = __ldg(a.gidx + node);
  return __ldg(a.tbase + node) + (g < a.D ? (__ldg(a.det + shot * a.D + g) & 1) : 0);
}

// Bounded wait used while leaving: every copy or MMA this thread issued signals its barrier; give up after the limit.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, uint64_t limit) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity) && globaltimer_ns() - t0 < limit) {
  }
}

template <bool DOWN>
__global__ void __launch_bounds__(kBThreads, 1)
    cascade_boundary_kernel(const __grid_constant__ CUtensorMap tmX3, const __grid_constant__ CUtensorMap tmWup,
                            const __grid_constant__ CUtensorMap tmWdn, const __grid_constant__ CUtensorMap tmH,
                            const __grid_constant__ CUtensorMap tmHo, const __grid_constant__ CUtensorMap tmY,
                            const BoundaryArgs a) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned by offsetting within the shared array (so the compiler keeps these accesses in the shared
  // space and knows they do not alias the global BatchNorm vectors)
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sb = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto bar = [&](int i) { return smem_u32(bars + i); };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = (a.num_tiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                 static_cast<int>(gridDim.x);                  // tiles of this CTA (grid <= num_tiles)

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i) {
      uint32_t count = 1;
      if (i == kDuE || i == kDuE + 1 || i >= kDone) count = kMidWarps;
      if (DOWN && (i == kX1F || i == kX1F + 1)) count = kMidWarps;
      if (i == kDdE || i == kDdE + 1) count = 4;
      mbar_init(bar(i), count);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmX3);
    tma_prefetch_desc(&tmWup);
    tma_prefetch_desc(&tmH);
    if (DOWN) tma_prefetch_desc(&tmWdn);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- TMA producer
      uint32_t n_x3 = 0, n_wu = 0, n_wd[2] = {0, 0};
      bool ok = true;
      for (int i = 0; i < nt && ok; ++i) {
        const int tile = static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x);
        if (!mbar_wait(bar(kX3E), (n_x3 & 1u) ^ 1u, abort_flag, a.status, a.timeout_ns)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(bar(kX3F), 2 * kBox);
        for (int kb = 0; kb < 2; ++kb) tma_load_2d(sb + kOffX3 + kb * kBox, &tmX3, kb * 64, tile * kBRows, bar(kX3F));
        ++n_x3;
        for (int q = 0; q < 4 && ok; ++q) {
          if (!mbar_wait(bar(kWuE), (n_wu & 1u) ^ 1u, abort_flag, a.status, a.timeout_ns)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(bar(kWuF), 2 * kBox);
          for (int kb = 0; kb < 2; ++kb) tma_load_2d(sb + kOffWup + kb * kBox, &tmWup, kb * 64, q * kBB, bar(kWuF));
          ++n_wu;
          if (DOWN)
            for (int c = 0; c < 2; ++c) {
              const int kc = 2 * q + c, s = kc & 1;
              if (!mbar_wait(bar(kWdE + s), (n_wd[s] & 1u) ^ 1u, abort_flag, a.status, a.timeout_ns)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(bar(kWdF + s), kBox);
              tma_load_2d(sb + kOffWdn + s * kBox, &tmWdn, kc * 64, 0, bar(kWdF + s));
              ++n_wd[s];
            }
        }
      }
      // the last copy of every buffer has landed before the CTA may leave
      if (n_x3) drain_wait(bar(kX3F), (n_x3 - 1) & 1u, a.timeout_ns);
      if (n_wu) drain_wait(bar(kWuF), (n_wu - 1) & 1u, a.timeout_ns);
      for (int s = 0; s < 2; ++s)
        if (n_wd[s]) drain_wait(bar(kWdF + s), (n_wd[s] - 1) & 1u, a.timeout_ns);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc = idesc_bf16_f32(kBRows, kBB);
      uint32_t n_x3 = 0, n_wu = 0, n_wd[2] = {0, 0}, n_du[2] = {0, 0}, n_x1[2] = {0, 0}, n_dd[2] = {0, 0};
      auto up = [&](int q) -> bool {
        const int b = static_cast<int>(n_du[0] + n_du[1]) & 1;   // quarters alternate between the two accumulators
        if (q == 0 && !mbar_wait(bar(kX3F), n_x3 & 1u, abort_flag, a.status, a.timeout_ns)) return false;
        if (!mbar_wait(bar(kWuF), n_wu & 1u, abort_flag, a.status, a.timeout_ns)) return false;
        if (!mbar_wait(bar(kDuE + b), (n_du[b] & 1u) ^ 1u, abort_flag, a.status, a.timeout_ns)) return false;
        tc_fence_after();
        const uint32_t d = tbase + static_cast<uint32_t>(b * kBB);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          const uint64_t ad = sdesc_k_sw128(sb + kOffX3 + kb * kBox);
          const uint64_t bd = sdesc_k_sw128(sb + kOffWup + kb * kBox);
#pragma unroll
          for (int k = 0; k < 4; ++k) tc_mma_ss(d, ad + ((k * 32) >> 4), bd + ((k * 32) >> 4), idesc, (kb | k) ? 1u : 0u);
        }
        tc_commit(bar(kWuE));
        ++n_wu;
        tc_commit(bar(kDuF + b));
        ++n_du[b];
        if (q == 3) {
          tc_commit(bar(kX3E));
          ++n_x3;
        }
        return true;
      };
      auto down = [&](int i, int kc) -> bool {
        const int s = kc & 1, e = i & 1;
        if (kc == 0 && !mbar_wait(bar(kDdE + e), (n_dd[e] & 1u) ^ 1u, abort_flag, a.status, a.timeout_ns)) return false;
        if (!mbar_wait(bar(kX1F + s), n_x1[s] & 1u, abort_flag, a.status, a.timeout_ns)) return false;
        if (!mbar_wait(bar(kWdF + s), n_wd[s] & 1u, abort_flag, a.status, a.timeout_ns)) return false;
        tc_fence_after();
        const uint32_t d = tbase + static_cast<uint32_t>(2 * kBB + e * kBB);
        const uint64_t ad = sdesc_k_sw128(sb + kOffX1 + s * kBox);
        const uint64_t bd = sdesc_k_sw128(sb + kOffWdn + s * kBox);
#pragma unroll
        for (int k = 0; k < 4; ++k) tc_mma_ss(d, ad + ((k * 32) >> 4), bd + ((k * 32) >> 4), idesc, (kc | k) ? 1u : 0u);
        tc_commit(bar(kX1E + s));
        ++n_x1[s];
        tc_commit(bar(kWdE + s));
        ++n_wd[s];
        if (kc == 7) {
          tc_commit(bar(kDdF + e));
          ++n_dd[e];
        }
        return true;
      };
      bool ok = true;
      for (int i = 0; i < nt && ok; ++i) {
        if (DOWN)
          ok = up(0) && up(1) && down(i, 0) && down(i, 1) && up(2) && down(i, 2) && down(i, 3) && up(3) &&
               down(i, 4) && down(i, 5) && down(i, 6) && down(i, 7);
        else
          ok = up(0) && up(1) && up(2) && up(3);
      }
      // every MMA issued so far has completed before TMEM is released
      tc_commit(bar(kDrain));
      drain_wait(bar(kDrain), 0, a.timeout_ns);
    }
    __syncwarp();
  } else if (warp < kEpiWarp0) {
    // ------------------------------------------------------------------ middle stage: residual, BN1 + SiLU -> x1
    const int quarter = warp & 3;
    const int half = (warp - kMidWarp0) >> 2;
    const int m = quarter * 32 + lane;                         // row of the tile = TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const bool x1_out = DOWN || a.store_x1;
    const uint64_t sh2 = f2_pack(a.scale_h, a.scale_h), su2 = f2_pack(a.scale_u, a.scale_u);
    bool ok = true;
    for (int i = 0; i < nt && ok; ++i) {
      const float* erow = a.tokens ? a.E + static_cast<int64_t>(row_token(
                                             a, static_cast<int64_t>(blockIdx.x + i * gridDim.x) * kBRows + m)) * kBH
                                   : nullptr;
      for (int q = 0; q < 4 && ok; ++q) {
        const int gq = 4 * i + q, b = gq & 1;
        for (int c = 0; c < 2; ++c) {
          const int kc = 2 * q + c, g = 8 * i + kc, hs = g % kHSlots, s = g & 1;
          // every wait is decided for the whole warp, so no lane is left behind in a warp-collective instruction
          bool good = true;
          if (c == 0) good = mbar_wait(bar(kDuF + b), (gq >> 1) & 1, abort_flag, a.status, a.timeout_ns);
          good = good && mbar_wait(bar(kHF + hs), (g / kHSlots) & 1, abort_flag, a.status, a.timeout_ns);
          if (x1_out) good = good && mbar_wait(bar(kX1E + s), ((g >> 1) & 1) ^ 1, abort_flag, a.status, a.timeout_ns);
          if (!__all_sync(0xffffffffu, good)) {
            ok = false;
            break;
          }
          {
            tc_fence_after();
            float acc[32];
            tmem_ld32(tbase + lane_base + static_cast<uint32_t>(b * kBB + c * 64 + half * 32), acc);
            uint8_t* hrow = smem + kOffH + (hs * 2 + half) * kBox + m * 128;
            const int ch0 = kc * 64 + half * 32;
            uint32_t xw[16];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float4* p = reinterpret_cast<float4*>(hrow + ((j ^ (m & 7)) << 4));
              const float4 hv = erow ? __ldg(reinterpret_cast<const float4*>(erow + ch0) + j) : *p;
              // u = bf16(acc); v = fmaf(scale_u, u, scale_h h), as packed pairs
              const uint64_t u0 = bf2_to_f2(f2_to_bf2(f2_pack(acc[4 * j], acc[4 * j + 1])));
              const uint64_t u1 = bf2_to_f2(f2_to_bf2(f2_pack(acc[4 * j + 2], acc[4 * j + 3])));
              const uint64_t v0 = f2_fma(su2, u0, f2_mul(f2_pack(hv.x, hv.y), sh2));
              const uint64_t v1 = f2_fma(su2, u1, f2_mul(f2_pack(hv.z, hv.w), sh2));
              if (a.store_h) *p = make_float4(f2_lo(v0), f2_hi(v0), f2_lo(v1), f2_hi(v1));
              if (x1_out) {
                const uint64_t* ap = reinterpret_cast<const uint64_t*>(a.a1 + ch0 + 4 * j);
                const uint64_t* bp = reinterpret_cast<const uint64_t*>(a.b1 + ch0 + 4 * j);
                xw[2 * j] = f2_to_bf2(silu_tanh_fast2(f2_fma(ap[0], v0, bp[0])));
                xw[2 * j + 1] = f2_to_bf2(silu_tanh_fast2(f2_fma(ap[1], v1, bp[1])));
              }
            }
            if (x1_out) {
              uint8_t* xrow = smem + kOffX1 + s * kBox + m * 128;
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int unit = half * 4 + u;
                *reinterpret_cast<uint4*>(xrow + ((unit ^ (m & 7)) << 4)) =
                    make_uint4(xw[4 * u], xw[4 * u + 1], xw[4 * u + 2], xw[4 * u + 3]);
              }
            }
            fence_proxy_async_smem();                   // the TMA stores and the MMAs read what was written here
          }
          if (c == 1) tc_fence_before();                // the quarter's accumulator reads are done
          __syncwarp();
          if (lane == 0) {                              // this warp's rows of the chunk are written
            if (DOWN) mbar_arrive(bar(kX1F + s));
            mbar_arrive(bar(kDone + hs));
            if (c == 1) mbar_arrive(bar(kDuE + b));
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == kStoreWarp) {
    if (lane == 0) {
      // ---------------------------------------------------------------- stores of finished chunks, h loads ahead
      const int total = nt * 8;                                 // 64-channel chunks of this CTA
      uint32_t n_h[kHSlots] = {0, 0, 0};
      auto h_load = [&](int g) {
        const int tile = static_cast<int>(blockIdx.x) + (g >> 3) * static_cast<int>(gridDim.x), kc = g & 7,
                  slot = g % kHSlots;
        if (a.tokens) {                                 // nothing to load: the slot is free for the middle stage
          mbar_arrive(bar(kHF + slot));
          return;
        }
        mbar_arrive_expect_tx(bar(kHF + slot), 2 * kBox);
        for (int bx = 0; bx < 2; ++bx)
          tma_load_2d(sb + kOffH + (slot * 2 + bx) * kBox, &tmH, kc * 64 + 32 * bx, tile * kBRows, bar(kHF + slot));
        ++n_h[slot];
      };
      for (int g = 0; g < kHSlots && g < total; ++g) h_load(g);
      for (int g = 0; g < total; ++g) {
        const int tile = static_cast<int>(blockIdx.x) + (g >> 3) * static_cast<int>(gridDim.x), kc = g & 7,
                  hs = g % kHSlots, s = g & 1;
        if (!mbar_wait(bar(kDone + hs), (g / kHSlots) & 1, abort_flag, a.status, a.timeout_ns)) break;
        if (a.store_h)
          for (int bx = 0; bx < 2; ++bx)
            tma_store_2d(&tmHo, kc * 64 + 32 * bx, tile * kBRows, sb + kOffH + (hs * 2 + bx) * kBox);
        if (!DOWN && a.store_x1) tma_store_2d(&tmY, kc * 64, tile * kBRows, sb + kOffX1 + s * kBox);
        bulk_commit();
        bulk_wait_read();                               // the boxes have been read: the slots may be reused
        if (!DOWN && a.store_x1) mbar_arrive(bar(kX1E + s));
        if (g + kHSlots < total) h_load(g + kHSlots);
      }
      bulk_wait_all();
      for (int sl = 0; sl < kHSlots; ++sl)
        if (n_h[sl]) drain_wait(bar(kHF + sl), (n_h[sl] - 1) & 1u, a.timeout_ns);
    }
    __syncwarp();
  } else if (DOWN) {
    // ------------------------------------------------------------------ down epilogue: BN2 + SiLU -> x2 rows
    const int m = (warp & 3) * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    for (int i = 0; i < nt; ++i) {
      const int tile = static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x), e = i & 1;
      if (!mbar_wait(bar(kDdF + e), (i >> 1) & 1, abort_flag, a.status, a.timeout_ns)) break;
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(tile) * kBRows + m;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(tbase + lane_base + static_cast<uint32_t>(2 * kBB + e * kBB + c * 32), v);
        uint32_t o[16];
#pragma unroll
        for (int p = 0; p < 16; ++p) {
          const int col = c * 32 + 2 * p;
          const uint64_t x = silu_tanh_fast2(f2_fma(f2_pack(v[2 * p], v[2 * p + 1]),
                                                    *reinterpret_cast<const uint64_t*>(a.a2 + col),
                                                    *reinterpret_cast<const uint64_t*>(a.b2 + col)));
          o[p] = f2_to_bf2(x);
        }
        if (row < a.rows) {
          uint4* dst = reinterpret_cast<uint4*>(a.y + row * kBB + c * 32);
#pragma unroll
          for (int w = 0; w < 4; ++w) dst[w] = make_uint4(o[4 * w], o[4 * w + 1], o[4 * w + 2], o[4 * w + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kDdE + e));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

int encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
              uint64_t row_bytes, uint32_t box_inner, const char* what) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(BPC_ERR_LAUNCH, "cuTensorMapEncodeTiled is not available from the CUDA driver");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, static_cast<cuuint32_t>(kBRows)};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(BPC_ERR_LAUNCH, std::string("cuTensorMapEncodeTiled(") + what + ") failed: " +
                                                         std::to_string(static_cast<int>(r)));
  return 0;
}

}  // namespace
}  // namespace bpc

using namespace bpc;

namespace bpc {
namespace {

struct TokenSource {
  const uint8_t* det = nullptr;
  const int32_t* gidx = nullptr;
  const int32_t* tbase = nullptr;
  const float* E = nullptr;
  int D = 0, N = 0;
};

int launch_boundary(const void* x3, const void* w_up, const float* h, const TokenSource* tok, float* h_out,
                    float scale_h, float scale_u, const float* a1, const float* b1, const void* w_down,
                    const float* a2, const float* b2, void* y, int64_t rows, int32_t H, int32_t Hb,
                    bpc_stream_t stream) {
  if (H != kBH || Hb != kBB) return fail(BPC_ERR_ARG, "the block boundary supports H = 512 with a 128-channel bottleneck");
  if (rows < 0 || rows > (static_cast<int64_t>(1) << 30)) return fail(BPC_ERR_ARG, "rows must be in [0, 2^30]");
  if (rows == 0) return 0;                      // nothing to do (empty buffers may be null)
  const bool down = w_down != nullptr;
  if (down && (!a1 || !b1 || !a2 || !b2 || !y)) return fail(BPC_ERR_ARG, "the down projection needs a1, b1, a2, b2 and y");
  if (!down && y && (!a1 || !b1)) return fail(BPC_ERR_ARG, "x1 needs a1 and b1");
  if (!x3 || !w_up || (!h && !tok)) return fail(BPC_ERR_ARG, "null buffer");
  const uintptr_t al16 = reinterpret_cast<uintptr_t>(x3) | reinterpret_cast<uintptr_t>(w_up) |
                         reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(h_out) |
                         reinterpret_cast<uintptr_t>(w_down) | reinterpret_cast<uintptr_t>(y) |
                         reinterpret_cast<uintptr_t>(a1) | reinterpret_cast<uintptr_t>(b1) |
                         reinterpret_cast<uintptr_t>(tok ? tok->E : nullptr);
  const uintptr_t al8 = reinterpret_cast<uintptr_t>(a2) | reinterpret_cast<uintptr_t>(b2);
  if ((al16 & 15) || (al8 & 7)) return fail(BPC_ERR_ARG, "buffers must be 16-byte aligned (a2, b2: 8-byte)");

  CUtensorMap mX3, mWup, mWdn{}, mH{}, mHo{}, mY{};
  const uint64_t R = static_cast<uint64_t>(rows);
  if (int e = encode_2d(&mX3, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x3, kBB, R, kBB * 2, 64, "x3")) return e;
  if (int e = encode_2d(&mWup, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, w_up, kBB, kBH, kBB * 2, 64, "w_up")) return e;
  if (!tok)
    if (int e = encode_2d(&mH, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, h, kBH, R, kBH * 4, 32, "h")) return e;
  if (h_out)
    if (int e = encode_2d(&mHo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, h_out, kBH, R, kBH * 4, 32, "h_out")) return e;
  if (down) {
    if (int e = encode_2d(&mWdn, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, w_down, kBH, kBB, kBH * 2, 64, "w_down")) return e;
  } else if (y) {
    if (int e = encode_2d(&mY, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, y, kBH, R, kBH * 2, 64, "x1")) return e;
  }
  BoundaryArgs a{};
  a.scale_h = scale_h;
  a.scale_u = scale_u;
  a.a1 = a1;
  a.b1 = b1;
  a.a2 = a2;
  a.b2 = b2;
  a.y = static_cast<__nv_bfloat16*>(y);
  a.rows = rows;
  a.num_tiles = static_cast<int>((rows + kBRows - 1) / kBRows);
  a.store_h = h_out != nullptr;
  a.store_x1 = !down && y != nullptr;
  if (tok) {
    a.tokens = 1;
    a.det = tok->det;
    a.gidx = tok->gidx;
    a.tbase = tok->tbase;
    a.E = tok->E;
    a.D = tok->D;
    a.N = tok->N;
  }
  a.status = op_status_ptr();
  a.timeout_ns = 2000000000ull;
  const void* fn = down ? reinterpret_cast<const void*>(&cascade_boundary_kernel<true>)
                        : reinterpret_cast<const void*>(&cascade_boundary_kernel<false>);
  if (int e = allow_smem(fn, static_cast<int>(kSmemBytes))) return e;
  const int grid = std::min(a.num_tiles, num_sms());
  void* args[] = {&mX3, &mWup, &mWdn, &mH, &mHo, &mY, &a};
  cudaError_t le = cudaLaunchKernel(fn, dim3(static_cast<unsigned>(grid)), dim3(kBThreads), args, kSmemBytes,
                                    reinterpret_cast<cudaStream_t>(stream));
  if (le != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("cascade_boundary_kernel launch: ") + cudaGetErrorString(le));
  return 0;
}

// The network's stem and the first block's BN1 + SiLU in one pass, 8 channels per thread:
// x1[shot, node, c] = bf16(SiLU(a1[c] E[token, c] + b1[c])), token = tbase[node] + det[shot, gidx[node]] (gidx = D: none)
__global__ void __launch_bounds__(256) cascade_stem_kernel(const uint8_t* __restrict__ det,
                                                           const int32_t* __restrict__ gidx,
                                                           const int32_t* __restrict__ tbase,
                                                           const float* __restrict__ E, const float* __restrict__ a,
                                                           const float* __restrict__ b, __nv_bfloat16* __restrict__ x,
                                                           int64_t groups, int D, int N, int H8) {
  for (int64_t gi = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; gi < groups;
       gi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = gi / H8;
    const int c0 = static_cast<int>(gi - row * H8) * 8;
    const int64_t shot = row / N;
    const int node = static_cast<int>(row - shot * N);
    const int g = __ldg(gidx + node);
    const int tok = __ldg(tbase + node) + (g < D ? (__ldg(det + shot * D + g) & 1) : 0);
    const float* e = E + static_cast<int64_t>(tok) * (8 * H8) + c0;
    uint4 o;
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      // v = 1 * h, as the residual pass computes it; SiLU on the hardware tanh, rounded to bf16
      const uint64_t v = f2_mul(f2_pack(__ldg(e + 2 * k), __ldg(e + 2 * k + 1)), f2_pack(1.f, 1.f));
      const uint64_t av = f2_pack(__ldg(a + c0 + 2 * k), __ldg(a + c0 + 2 * k + 1));
      const uint64_t bv = f2_pack(__ldg(b + c0 + 2 * k), __ldg(b + c0 + 2 * k + 1));
      op[k] = f2_to_bf2(silu_tanh_fast2(f2_fma(av, v, bv)));
    }
    reinterpret_cast<uint4*>(x)[gi] = o;
  }
}

}  // namespace
}  // namespace bpc

extern "C" int bpc_cascade_boundary(const void* x3, const void* w_up, const float* h, float* h_out, float scale_h,
                                    float scale_u, const float* a1, const float* b1, const void* w_down,
                                    const float* a2, const float* b2, void* y, int64_t rows, int32_t H, int32_t Hb,
                                    bpc_stream_t stream) {
  return launch_boundary(x3, w_up, h, nullptr, h_out, scale_h, scale_u, a1, b1, w_down, a2, b2, y, rows, H, Hb,
                         stream);
}

extern "C" int bpc_cascade_boundary_tokens(const void* x3, const void* w_up, const uint8_t* det, const int32_t* gidx,
                                           const int32_t* tbase, const float* E, int32_t D, int32_t N, float* h_out,
                                           float scale_h, float scale_u, const float* a1, const float* b1,
                                           const void* w_down, const float* a2, const float* b2, void* y, int64_t B,
                                           int32_t H, int32_t Hb, bpc_stream_t stream) {
  if (B < 0 || D < 0 || N < 1) return fail(BPC_ERR_ARG, "B >= 0, D >= 0, N >= 1");
  if (B > 0 && (!det && D > 0)) return fail(BPC_ERR_ARG, "null det");
  if (B > 0 && (!gidx || !tbase || !E)) return fail(BPC_ERR_ARG, "null token tables");
  TokenSource t;
  t.det = det;
  t.gidx = gidx;
  t.tbase = tbase;
  t.E = E;
  t.D = D;
  t.N = N;
  return launch_boundary(x3, w_up, nullptr, &t, h_out, scale_h, scale_u, a1, b1, w_down, a2, b2, y, B * N, H, Hb,
                         stream);
}

extern "C" int bpc_cascade_stem(const uint8_t* det, const int32_t* gidx, const int32_t* tbase, const float* E,
                                int32_t D, int32_t N, const float* a1, const float* b1, void* x1, int64_t B, int32_t H,
                                bpc_stream_t stream) {
  if (B < 0 || D < 0 || N < 1 || H < 8 || H % 8) return fail(BPC_ERR_ARG, "B >= 0, D >= 0, N >= 1, H a multiple of 8");
  if (B == 0) return 0;
  if ((!det && D > 0) || !gidx || !tbase || !E || !a1 || !b1 || !x1) return fail(BPC_ERR_ARG, "null buffer");
  if (reinterpret_cast<uintptr_t>(x1) & 15) return fail(BPC_ERR_ARG, "x1 must be 16-byte aligned");
  const int64_t groups = B * N * (H / 8);
  const int blocks = static_cast<int>(std::min<int64_t>((groups + 255) / 256, static_cast<int64_t>(num_sms()) * 16));
  cascade_stem_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      det, gidx, tbase, E, a1, b1, static_cast<__nv_bfloat16*>(x1), groups, D, N, H / 8);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("cascade_stem_kernel: ") + cudaGetErrorString(e));
  return 0;
}
