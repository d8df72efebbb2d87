// Persistent streaming pre-decoder (sliding window of W rounds, batch 1, C = 64, K = 8): one resident kernel that
// serves rounds through a request line in mapped host memory, the protocol of the reference's persistent kernel
// (evaluation/timing/d7/kernel.cu:310-369,440-527; router.cc:170-223,576-650): the host writes a round's detectors
// and a tag, the kernel publishes the round's residual syndrome and the newest round's X/Z logits with the same tag,
// a stop command or an idle watchdog ends the kernel, and a step watchdog turns any wait that never completes into
// an error status instead of a hang.
//
// Grid: 8 clusters x 8 CTAs (cooperative).  Cluster c owns target tile c (128 nodes) of every step; CTA r of the
// cluster owns relation r: it keeps W_r of every layer resident in shared memory (the check -> data step's and, for
// its tile's check type, the data -> check step's: 16 KB per layer), gathers relation r's 128 source rows of the
// step by TMA (tile::gather4), runs 4 MMAs into its TMEM accumulator and sends the fp32 partial rows to their owner
// CTAs by bulk shared -> distributed-shared copies; the owner adds the 8 partials in relation order and runs the
// epilogue (GELU, residual, head, XOR) for its 16 rows -- the arithmetic of gmm_nodes_split_kernel.  Activations live
// in device memory (L2); a bounded grid barrier separates the steps.
//
// A round: wait for the request; embed the window's check nodes (a device ring holds the W - 1 older rounds, the
// new round comes from the request line); L check -> data steps and L - 1 data -> check steps (the last layer's
// data -> check step does not reach the outputs); the last check -> data step writes the newest round's logits to
// the response and XORs the predicted flips into the residual; CTA 0 copies the residual to the response and
// releases the tag.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstring>
#include <string>
#include <thread>

#include <cudaTypedefs.h>

#include "bpc.h"
#include "bpc_common.cuh"
#include "bpc_internal.h"

namespace bpc {
namespace {

constexpr int kSThreads = 128;
constexpr int kSClusters = 8;
constexpr int kSRel = 8;
constexpr int kSRows = 128;
constexpr int kSC = 64;
constexpr int kSMaxLayers = 8;
constexpr uint32_t kSWBytes = kSC * 128;             // one W_r block: 64 rows x 64 channels bf16
constexpr uint32_t kSABytes = kSRows * 128;          // gathered rows
constexpr uint32_t kSSlot = 16 * kSC * 4;            // one owner's block of a partial (16 rows x 64 fp32)
constexpr uint32_t kSPart = kSRel * kSSlot;          // 32 KB

// Request / response lines in mapped host memory.
constexpr int kReqDets = 64;                         // request: u64 tag, u32 cmd, then the detectors at byte 64
constexpr int kRespOff = 4096;                       // response: u64 tag, u32 status, then residual, logits
constexpr int kRespData = 64;

enum : uint32_t { kCmdRound = 0, kCmdStop = 1 };
constexpr unsigned long long kStopFlag = ~0ull;
enum : uint32_t { kStStarting = 0, kStReady = 1, kStStopped = 2, kStWatchdog = 3, kStIdle = 4 };

struct StreamArgs {
  // model
  const __nv_bfloat16* embed;   // (4, 64)
  const float* head_w;          // (2, 64)
  const float* head_b;          // (2)
  const int32_t* c2d;           // (N_d, 8)
  const int32_t* d2c;           // (N_c, 8)
  const int32_t* xor_nbr;       // (N_d, 4)
  int layers, W, nh, nq, N_c, N_d;
  int tiles_c2d, tiles_x;       // check -> data tiles; X-check tiles of a data -> check step (then Z)
  // state
  __nv_bfloat16* hc;            // (N_c, 64)
  __nv_bfloat16* hd;            // (N_d, 64)
  uint8_t* ring;                // (2, W, nh): the W - 1 older rounds
  uint32_t* res;                // (N_c / 4 rounded up): residual bytes of the current round
  unsigned long long* bar;      // grid barrier counter
  int* abort_flag;              // any CTA gave up a wait
  unsigned long long* round_flag;  // the tag of the accepted request (kStopFlag: stop), released by CTA 0
  uint8_t* dev_req;             // the accepted request's detectors, copied by CTA 0
  uint8_t* dev_out;             // the round's results: residual bytes (N_c, rounded to 16), then the newest logits
  // host lines (device pointers of mapped host memory)
  volatile uint8_t* req;
  volatile uint8_t* resp;
  uint64_t idle_ns, step_ns;
};

__device__ __forceinline__ uint64_t ld_volatile_u64(volatile const uint8_t* p) {
  return *reinterpret_cast<volatile const unsigned long long*>(p);
}
// 16-byte accesses of mapped host memory that the compiler neither caches nor merges
__device__ __forceinline__ uint4 ld_volatile_u4(volatile const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(const_cast<const void*>(p))
               : "memory");
  return v;
}
__device__ __forceinline__ void st_volatile_u4(volatile void* p, uint4 v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(const_cast<void*>(p)), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// Bounded grid barrier over every CTA of the grid: `n` is the number of barriers passed so far (the counter only
// grows).  Returns false after the step watchdog or when another CTA gave up.
__device__ bool grid_sync(const StreamArgs& a, unsigned long long n, volatile int* cta_abort) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(a.bar, 1ull);
    const unsigned long long target = (n + 1) * gridDim.x;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
      unsigned long long v;
      asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(a.bar) : "memory");
      if (v >= target) break;
      if (*reinterpret_cast<volatile int*>(a.abort_flag) || globaltimer_ns() - t0 > a.step_ns) {
        atomicExch(a.abort_flag, 1);
        *cta_abort = 1;
        break;
      }
    }
  }
  __syncthreads();
  return !*cta_abort;
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__global__ void __launch_bounds__(kSThreads, 1)
    stream_kernel(const __grid_constant__ CUtensorMap tmWc, const __grid_constant__ CUtensorMap tmWd,
                  const __grid_constant__ CUtensorMap tmHc, const __grid_constant__ CUtensorMap tmHd,
                  const StreamArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int L = a.layers;
  uint8_t* sWc = smem;                                  // L blocks: W_c2d[l]_r
  uint8_t* sWd = smem + L * kSWBytes;                   // L blocks: W_d2c[l, type]_r
  uint8_t* sA = smem + 2 * L * kSWBytes;
  uint8_t* sO = sA + kSABytes;
  uint8_t* sR = sO + kSPart;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sR + kSPart);
  uint64_t* wfull = bars;
  uint64_t* full = bars + 1;
  uint64_t* accf = bars + 2;
  uint64_t* recv = bars + 3;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  volatile int* cta_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile uint32_t* s_cmd = reinterpret_cast<volatile uint32_t*>(tmem_slot + 2);
  uint8_t* s_new = reinterpret_cast<uint8_t*>(bars + 8);   // the new round's detectors (2 nh bytes)

  const int t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31;
  const int r = static_cast<int>(cluster_ctarank());
  const int cl = blockIdx.x / kSRel;                    // tile index of every step
  // this cluster's tiles: check -> data (data nodes), data -> check (X checks, then Z checks)
  const bool has_c2d = cl < a.tiles_c2d;
  const int c2d_begin = cl * kSRows, c2d_end = min(a.N_d, c2d_begin + kSRows);
  const int nx = a.W * a.nh;
  const bool zt = cl >= a.tiles_x;
  const bool has_d2c = cl < 2 * a.tiles_x;
  const int d2c_begin = zt ? nx + (cl - a.tiles_x) * kSRows : cl * kSRows;
  const int d2c_end = zt ? min(a.N_c, d2c_begin + kSRows) : min(nx, d2c_begin + kSRows);
  // gather rows (thread t = row t) and owned output rows (16 r + t / 8, channels 8 (t % 8) .. + 7)
  const int src_c2d = (has_c2d && c2d_begin + t < c2d_end) ? __ldg(a.c2d + static_cast<int64_t>(c2d_begin + t) * kSRel + r) : -1;
  const int src_d2c = (has_d2c && d2c_begin + t < d2c_end) ? __ldg(a.d2c + static_cast<int64_t>(d2c_begin + t) * kSRel + r) : -1;
  const int orow = t >> 3;

  if (t == 0) {
    mbar_init(smem_u32(wfull), 1);
    mbar_init(smem_u32(full), 4);
    mbar_init(smem_u32(accf), 1);
    mbar_init(smem_u32(recv), 1);
    mbar_arrive_expect_tx(smem_u32(recv), kSPart);     // armed for the first step; peers send after the barrier
    *cta_abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmWc);
    tma_prefetch_desc(&tmWd);
    tma_prefetch_desc(&tmHc);
    tma_prefetch_desc(&tmHd);
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), 64);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  cluster_arrive_release();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (t == 0) {
    // every layer's W_r, resident for the kernel's lifetime
    mbar_arrive_expect_tx(smem_u32(wfull), 2 * L * kSWBytes);
    for (int l = 0; l < L; ++l) {
      tma_load_3d(smem_u32(sWc + l * kSWBytes), &tmWc, 0, r, l * kSC, smem_u32(wfull));
      tma_load_3d(smem_u32(sWd + l * kSWBytes), &tmWd, 0, r, (2 * l + (zt ? 1 : 0)) * kSC, smem_u32(wfull));
    }
  }
  cluster_wait_acquire();
  bool ok = true;
  if (t == 0) ok = mbar_wait(smem_u32(wfull), 0, cta_abort, nullptr, a.step_ns);
  if (!__syncthreads_and(ok)) *cta_abort = 1;
  unsigned long long nbar = 0;
  uint32_t ph_full = 0, ph_acc = 0, ph_recv = 0;
  uint64_t tag = 0;
  int head = 0;                                         // ring slot of the oldest round
  const uint32_t idesc = idesc_bf16_f32(kSRows, kSC);
  if (blockIdx.x == 0 && t == 0 && !*cta_abort) {
    *reinterpret_cast<volatile uint32_t*>(a.resp + 8) = kStReady;
    __threadfence_system();
  }

  while (!*cta_abort) {
    // ------------------------------------------------------------------ the next request (idle watchdog)
    // CTA 0 polls the host line, copies the detectors into device memory and releases the round on a device flag;
    // the other CTAs poll that flag in L2 (one reader of host memory instead of 64)
    if (blockIdx.x == 0) {
      if (t == 0) {
        const uint64_t t0 = globaltimer_ns();
        uint32_t cmd = kCmdStop;
        while (true) {
          const uint64_t v = ld_volatile_u64(a.req);
          if (v == tag + 1) {
            __threadfence_system();
            cmd = *reinterpret_cast<volatile const uint32_t*>(a.req + 8);
            break;
          }
          if (*reinterpret_cast<volatile int*>(a.abort_flag)) break;
          if (globaltimer_ns() - t0 > a.idle_ns) {
            *reinterpret_cast<volatile uint32_t*>(a.resp + 8) = kStIdle;
            break;
          }
        }
        *s_cmd = cmd;
      }
      __syncthreads();
      if (*s_cmd == kCmdRound)
        for (int e = t; e < (2 * a.nh + 15) / 16; e += kSThreads)
          reinterpret_cast<uint4*>(a.dev_req)[e] = ld_volatile_u4(a.req + kReqDets + 16 * e);
      __syncthreads();
      if (t == 0) {
        __threadfence();
        const unsigned long long f = *s_cmd == kCmdRound ? tag + 1 : kStopFlag;
        asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(a.round_flag), "l"(f) : "memory");
      }
    } else if (t == 0) {
      const uint64_t t0 = globaltimer_ns();
      uint32_t cmd = kCmdStop;
      while (true) {
        unsigned long long v;
        asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(a.round_flag) : "memory");
        if (v == tag + 1) {
          cmd = kCmdRound;
          break;
        }
        if (v == kStopFlag || *reinterpret_cast<volatile int*>(a.abort_flag)) break;
        if (globaltimer_ns() - t0 > a.idle_ns + 1000000000ull) break;   // CTA 0 gives up first
      }
      *s_cmd = cmd;
    }
    __syncthreads();
    if (*s_cmd != kCmdRound) break;
    ++tag;
    for (int e = t; e < 2 * a.nh; e += kSThreads) s_new[e] = __ldcg(a.dev_req + e) & 1;
    __syncthreads();
    // ------------------------------------------------------------------ embed the window and reset the residual
    {
      const int g = blockIdx.x * kSThreads + t;         // node g / 8, 16-byte chunk g % 8
      const int n = g >> 3, j = g & 7;
      if (n < a.N_c) {
        const int ty = n / nx, tt = (n / a.nh) % a.W, s = n % a.nh;
        const uint8_t det = tt == a.W - 1 ? s_new[ty * a.nh + s]
                                          : (__ldcg(a.ring + (ty * a.W + (head + tt) % a.W) * a.nh + s) & 1);
        reinterpret_cast<uint4*>(a.hc + static_cast<int64_t>(n) * kSC)[j] =
            __ldg(reinterpret_cast<const uint4*>(a.embed + (2 * ty + det) * kSC) + j);
        if (j == 0 && (n & 3) == 0) {
          uint32_t w = 0;
          for (int k = 0; k < 4 && n + k < a.N_c; ++k) {
            const int m = n + k;
            const int tym = m / nx, ttm = (m / a.nh) % a.W, sm = m % a.nh;
            const uint8_t dm = ttm == a.W - 1 ? s_new[tym * a.nh + sm]
                                              : (__ldcg(a.ring + (tym * a.W + (head + ttm) % a.W) * a.nh + sm) & 1);
            w |= static_cast<uint32_t>(dm) << (8 * k);
          }
          a.res[n >> 2] = w;
        }
      }
      // the new round enters the ring (its slot is the newest in this window; no CTA reads it this round)
      if (blockIdx.x == 0)
        for (int e = t; e < 2 * a.nh; e += kSThreads) {
          const int ty = e / a.nh, s = e % a.nh;
          a.ring[(ty * a.W + (head + a.W - 1) % a.W) * a.nh + s] = s_new[e];
        }
    }
    if (!grid_sync(a, nbar++, cta_abort)) break;
    // ------------------------------------------------------------------ L check -> data and L - 1 data -> check steps
    bool failed = false;
    for (int step = 0; step < 2 * L - 1 && !failed; ++step) {
      const int l = step >> 1;
      const bool c2d = (step & 1) == 0;
      const bool active = c2d ? has_c2d : has_d2c;
      const bool last = step == 2 * L - 2;
      if (active) {
        const CUtensorMap* tm = c2d ? &tmHc : &tmHd;
        const int src = c2d ? src_c2d : src_d2c;
        const int nsrc = c2d ? a.N_c : a.N_d;
        fence_proxy_async_global();                    // the gathers read what earlier steps stored
        const int32_t xr = (src >= 0 && src < nsrc) ? src : nsrc;
        const int q4 = lane & ~3;
        const int32_t i0 = __shfl_sync(0xffffffffu, xr, q4), i1 = __shfl_sync(0xffffffffu, xr, q4 + 1),
                      i2 = __shfl_sync(0xffffffffu, xr, q4 + 2), i3 = __shfl_sync(0xffffffffu, xr, q4 + 3);
        if (lane == 0) mbar_arrive_expect_tx(smem_u32(full), 32 * 128);
        __syncwarp();
        if ((lane & 3) == 0) tma_gather4(smem_u32(sA + t * 128), tm, 0, i0, i1, i2, i3, smem_u32(full));
        // the residual rows this thread owns (outputs of earlier steps)
        const int ob = c2d ? c2d_begin : d2c_begin, oe = c2d ? c2d_end : d2c_end;
        const int on = ob + r * 16 + orow;
        const bool o_ok = on < oe;
        __nv_bfloat16* y = c2d ? a.hd : a.hc;
        const bool resid = !(c2d && l == 0);
        uint4 res = make_uint4(0, 0, 0, 0);
        // (through L2: other CTAs of this kernel wrote these rows; L1 is not coherent)
        if (resid && o_ok) res = __ldcg(reinterpret_cast<const uint4*>(y + static_cast<int64_t>(on) * kSC + (t & 7) * 8));
        bool good = true;
        if (t == 0) {
          good = mbar_wait(smem_u32(full), ph_full, cta_abort, nullptr, a.step_ns);
          if (good) {
            tc_fence_after();
            const uint64_t ad = sdesc_k_sw128(smem_u32(sA));
            const uint64_t bd = sdesc_k_sw128(smem_u32((c2d ? sWc : sWd) + l * kSWBytes));
#pragma unroll
            for (int k = 0; k < 4; ++k)
              tc_mma_ss(tmem_base, ad + ((k * 32) >> 4), bd + ((k * 32) >> 4), idesc, k ? 1u : 0u);
          }
          tc_commit(smem_u32(accf));
        }
        ph_full ^= 1u;
        good = mbar_wait(smem_u32(accf), ph_acc, cta_abort, nullptr, a.step_ns) && good && !*cta_abort;
        ph_acc ^= 1u;
        if (good) {
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
        tc_fence_before();
        fence_proxy_async_smem();
        __syncthreads();
        if (t == 0) {
          for (int jj = 0; jj < kSRel; ++jj)
            bulk_s2cluster(map_to_cta(smem_u32(sR + r * kSSlot), jj), smem_u32(sO + jj * kSSlot), kSSlot,
                           map_to_cta(smem_u32(recv), jj));
          bulk_commit();
        }
        // the 8 partials of this CTA's rows
        bool rec = true;
        {
          const uint32_t rb = smem_u32(recv);
          if (!mbar_try_wait_cluster(rb, ph_recv)) {
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait_cluster(rb, ph_recv)) {
              if (globaltimer_ns() - t0 > a.step_ns) {
                rec = false;
                break;
              }
            }
          }
        }
        ph_recv ^= 1u;
        float sum[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) sum[e] = 0.f;
#pragma unroll
        for (int jj = 0; jj < kSRel; ++jj)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float4 v = *reinterpret_cast<const float4*>(sR + recv_off(jj, orow, 2 * (t & 7) + h));
            sum[4 * h] += v.x;
            sum[4 * h + 1] += v.y;
            sum[4 * h + 2] += v.z;
            sum[4 * h + 3] += v.w;
          }
        uint64_t lg0 = 0, lg1 = 0;
        if (o_ok && rec) {
          uint4 u;
          uint32_t* o = reinterpret_cast<uint32_t*>(&u);
          const uint32_t* hres = reinterpret_cast<const uint32_t*>(&res);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            uint64_t xv = gelu_tanh_fast2(f2_pack(sum[2 * e], sum[2 * e + 1]));
            if (resid) xv = f2_add(xv, bf2_to_f2(hres[e]));
            o[e] = f2_to_bf2(xv);
            if (last) {
              const uint64_t f = bf2_to_f2(o[e]);
              const int col = (t & 7) * 8 + 2 * e;
              lg0 = f2_fma(f, *reinterpret_cast<const uint64_t*>(a.head_w + col), lg0);
              lg1 = f2_fma(f, *reinterpret_cast<const uint64_t*>(a.head_w + kSC + col), lg1);
            }
          }
          *reinterpret_cast<uint4*>(y + static_cast<int64_t>(on) * kSC + (t & 7) * 8) = u;
        }
        if (last) {
          float l0 = f2_lo(lg0) + f2_hi(lg0), l1 = f2_lo(lg1) + f2_hi(lg1);
#pragma unroll
          for (int m = 1; m < 8; m <<= 1) {
            l0 += __shfl_xor_sync(0xffffffffu, l0, m);
            l1 += __shfl_xor_sync(0xffffffffu, l1, m);
          }
          if (o_ok && rec && (t & 7) == 0) {
            l0 += __ldg(a.head_b);
            l1 += __ldg(a.head_b + 1);
            const int newest = (a.W - 1) * a.nq;
            if (on >= newest)
              *reinterpret_cast<float2*>(a.dev_out + ((a.N_c + 15) & ~15) + static_cast<int64_t>(on - newest) * 8) =
                  make_float2(l0, l1);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const bool flip = (k >> 1) ? (l1 > 0.f) : (l0 > 0.f);
              const int32_t cidx = __ldg(a.xor_nbr + static_cast<int64_t>(on) * 4 + k);
              if (flip && cidx >= 0) atomicXor(a.res + (cidx >> 2), 1u << (8 * (cidx & 3)));
            }
          }
        }
        if (t == 0) bulk_wait_read();                  // sO is free for the next step
        if (t == 0) mbar_arrive_expect_tx(smem_u32(recv), kSPart);   // re-armed before the peers' next copies
        if (!rec || !good) {
          if (t == 0) atomicExch(a.abort_flag, 1);
          *cta_abort = 1;
        }
      }
      if (!grid_sync(a, nbar++, cta_abort)) failed = true;
    }
    if (failed || *cta_abort) break;
    // ------------------------------------------------------------------ publish: results in 16-byte stores, then the tag
    if (blockIdx.x == 0) {
      const int nres = (a.N_c + 15) / 16, nlg = (a.nq * 8 + 15) / 16;
      volatile uint8_t* rp = a.resp + kRespData;
      for (int e = t; e < nres + nlg; e += kSThreads) {
        // the residual bytes are the bytes of the residual words; the logits were staged in device memory
        const uint4 v = e < nres ? __ldcg(reinterpret_cast<const uint4*>(a.res) + e)
                                 : __ldcg(reinterpret_cast<const uint4*>(a.dev_out + ((a.N_c + 15) & ~15)) + (e - nres));
        st_volatile_u4(rp + 16 * e, v);
      }
      __threadfence_system();
      __syncthreads();
      if (t == 0) {
        *reinterpret_cast<volatile unsigned long long*>(a.resp) = tag;
        __threadfence_system();
      }
    }
    head = (head + 1) % a.W;
  }
  if (blockIdx.x == 0 && t == 0) {
    const int ab = *reinterpret_cast<volatile int*>(a.abort_flag);
    volatile uint32_t* st = reinterpret_cast<volatile uint32_t*>(a.resp + 8);
    if (ab) *st = kStWatchdog;
    else if (*st != kStIdle) *st = kStStopped;
    __threadfence_system();
  }
  // every CTA of the cluster is done with its peers' shared memory before any leaves
  cluster_arrive_release();
  cluster_wait_acquire();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 64);
  }
}

}  // namespace
}  // namespace bpc

using namespace bpc;

struct bpc_stream {
  const bpc_predecoder* pd = nullptr;
  StreamArgs args{};
  CUtensorMap maps[4];
  uint8_t* host = nullptr;      // mapped: request at 0, response at kRespOff
  uint8_t* host_dev = nullptr;
  void* dev = nullptr;          // hc, hd, ring, res, barrier, abort
  cudaStream_t stream = nullptr;
  bool running = false;
  bool desynced = false;        // a round was given up before its response: later rounds fail until stop / start
  uint64_t tag = 0;
  int smem = 0;
};

namespace {

int map3(CUtensorMap* m, const void* base, cuuint64_t d0, cuuint64_t d1, cuuint64_t d2, uint32_t b2) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return fail(BPC_ERR_DRIVER, "cuTensorMapEncodeTiled is not available from the CUDA driver");
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {d0 * 2, d0 * d1 * 2};
  cuuint32_t box[3] = {64, 1, b2};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : fail(BPC_ERR_DRIVER, "cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
}

int rows2(CUtensorMap* m, const void* base, int64_t rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return fail(BPC_ERR_DRIVER, "cuTensorMapEncodeTiled is not available from the CUDA driver");
  cuuint64_t dims[2] = {64, static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {128};
  cuuint32_t box[2] = {64, 1};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : fail(BPC_ERR_DRIVER, "cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
}

volatile uint64_t* req_tag(bpc_stream* s) { return reinterpret_cast<volatile uint64_t*>(s->host); }
volatile uint64_t* resp_tag(bpc_stream* s) { return reinterpret_cast<volatile uint64_t*>(s->host + kRespOff); }
volatile uint32_t* resp_status(bpc_stream* s) { return reinterpret_cast<volatile uint32_t*>(s->host + kRespOff + 8); }

}  // namespace

extern "C" int bpc_stream_create(const bpc_predecoder* h, int32_t window, int32_t nh, int32_t nq,
                                 int32_t idle_timeout_ms, bpc_stream** out) {
  if (!h || !out) return fail(BPC_ERR_ARG, "null argument");
  *out = nullptr;
  bpc_predecoder_config c{};
  const void *embed, *wc, *wd;
  const float *hw, *hb;
  const int32_t *c2d, *d2c, *xr;
  if (int e = predecoder_internals(h, &c, &embed, &wc, &wd, &hw, &hb, &c2d, &d2c, &xr)) return e;
  if (c.dtype != BPC_DTYPE_BF16 || c.channels != kSC || c.K != kSRel || c.layers < 1 || c.layers > kSMaxLayers)
    return fail(BPC_ERR_ARG, "the persistent kernel serves bf16 networks with C = 64, K = 8 and at most 8 layers");
  if (window < 1 || nh < 1 || nq < 1 || c.n_checks != 2 * window * nh || c.n_data != window * nq ||
      c.z_check_begin != window * nh)
    return fail(BPC_ERR_ARG, "window, checks and data qubits per round disagree with the pre-decoder");
  const int tiles_c2d = (c.n_data + kSRows - 1) / kSRows, tiles_x = (window * nh + kSRows - 1) / kSRows;
  if (tiles_c2d > kSClusters || 2 * tiles_x > kSClusters)
    return fail(BPC_ERR_ARG, "the window is larger than 8 tiles of 128 nodes per step");
  if (2 * nh > 1024 || 2 * nh + kReqDets > kRespOff || kRespData + ((c.n_checks + 15) & ~15) + nq * 8 > 65536 - kRespOff)
    return fail(BPC_ERR_ARG, "the request or response does not fit its line");
  auto* s = new bpc_stream();
  s->pd = h;
  StreamArgs& a = s->args;
  a.embed = static_cast<const __nv_bfloat16*>(embed);
  a.head_w = hw;
  a.head_b = hb;
  a.c2d = c2d;
  a.d2c = d2c;
  a.xor_nbr = xr;
  a.layers = c.layers;
  a.W = window;
  a.nh = nh;
  a.nq = nq;
  a.N_c = c.n_checks;
  a.N_d = c.n_data;
  a.tiles_c2d = tiles_c2d;
  a.tiles_x = tiles_x;
  a.idle_ns = static_cast<uint64_t>(std::max(idle_timeout_ms, 1)) * 1000000ull;
  a.step_ns = 500000000ull;
  const size_t o_hd = static_cast<size_t>(a.N_c) * 128, o_ring = o_hd + static_cast<size_t>(a.N_d) * 128;
  const size_t o_res = (o_ring + 2 * window * nh + 255) & ~size_t(255);
  const size_t o_bar = (o_res + ((a.N_c + 15) / 16) * 16 + 255) & ~size_t(255);
  const size_t o_req = o_bar + 256;
  const size_t o_out = o_req + 1024;
  const size_t total = o_out + ((a.N_c + 15) & ~15) + static_cast<size_t>(nq) * 8 + 16;
  auto bail = [&](int code, const std::string& msg) {
    bpc_stream_destroy(s);
    return fail(code, msg);
  };
  if (cudaMalloc(&s->dev, total) != cudaSuccess) return bail(BPC_ERR_LAUNCH, "cudaMalloc of the stream state failed");
  if (cudaMemset(s->dev, 0, total) != cudaSuccess) return bail(BPC_ERR_LAUNCH, "cudaMemset failed");
  uint8_t* d = static_cast<uint8_t*>(s->dev);
  a.hc = reinterpret_cast<__nv_bfloat16*>(d);
  a.hd = reinterpret_cast<__nv_bfloat16*>(d + o_hd);
  a.ring = d + o_ring;
  a.res = reinterpret_cast<uint32_t*>(d + o_res);
  a.bar = reinterpret_cast<unsigned long long*>(d + o_bar);
  a.abort_flag = reinterpret_cast<int*>(d + o_bar + 64);
  a.round_flag = reinterpret_cast<unsigned long long*>(d + o_bar + 128);
  a.dev_req = d + o_req;
  a.dev_out = d + o_out;
  if (cudaHostAlloc(reinterpret_cast<void**>(&s->host), 65536, cudaHostAllocMapped) != cudaSuccess)
    return bail(BPC_ERR_LAUNCH, "cudaHostAlloc of the request / response lines failed");
  std::memset(s->host, 0, 65536);
  if (cudaHostGetDevicePointer(reinterpret_cast<void**>(&s->host_dev), s->host, 0) != cudaSuccess)
    return bail(BPC_ERR_LAUNCH, "cudaHostGetDevicePointer failed");
  a.req = s->host_dev;
  a.resp = s->host_dev + kRespOff;
  int e = 0;
  if ((e = map3(&s->maps[0], wc, kSC, kSRel, static_cast<cuuint64_t>(kSC) * c.layers, kSC)) ||
      (e = map3(&s->maps[1], wd, kSC, kSRel, static_cast<cuuint64_t>(kSC) * 2 * c.layers, kSC)) ||
      (e = rows2(&s->maps[2], a.hc, a.N_c)) || (e = rows2(&s->maps[3], a.hd, a.N_d))) {
    bpc_stream_destroy(s);
    return e;
  }
  s->smem = 1024 + 2 * c.layers * kSWBytes + kSABytes + 2 * kSPart + 64 + 1024;
  if (cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking) != cudaSuccess)
    return bail(BPC_ERR_LAUNCH, "cudaStreamCreate failed");
  *out = s;
  return 0;
}

extern "C" int bpc_stream_start(bpc_stream* s) {
  if (!s) return fail(BPC_ERR_ARG, "null stream");
  if (s->running) return fail(BPC_ERR_ARG, "the stream kernel already runs");
  if (int e = allow_smem(reinterpret_cast<const void*>(&stream_kernel), s->smem)) return e;
  std::memset(s->host, 0, 65536);
  s->tag = 0;
  s->desynced = false;
  if (cudaMemsetAsync(s->args.bar, 0, 256, s->stream) != cudaSuccess ||
      cudaMemsetAsync(s->args.ring, 0, 2 * s->args.W * s->args.nh, s->stream) != cudaSuccess)
    return fail(BPC_ERR_LAUNCH, "cudaMemsetAsync failed");
  // all 64 CTAs must be resident at once (the grid barrier waits for every one): a cooperative launch guarantees
  // it or fails
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(kSClusters * kSRel);
  lc.blockDim = dim3(kSThreads);
  lc.dynamicSmemBytes = static_cast<size_t>(s->smem);
  lc.stream = s->stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kSRel;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  lc.attrs = attr;
  lc.numAttrs = 2;
  void* args[] = {&s->maps[0], &s->maps[1], &s->maps[2], &s->maps[3], &s->args};
  cudaError_t le = cudaLaunchKernelExC(&lc, reinterpret_cast<const void*>(&stream_kernel), args);
  if (le != cudaSuccess) {
    // a cluster launch that cannot also be cooperative: launch plainly if the occupancy calculator confirms that
    // all 8 clusters fit at once
    cudaGetLastError();
    lc.numAttrs = 1;
    int max_clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&max_clusters, reinterpret_cast<const void*>(&stream_kernel), &lc) !=
            cudaSuccess ||
        max_clusters < kSClusters)
      return fail(BPC_ERR_LAUNCH, std::string("stream kernel: 8 resident clusters not available (") +
                                      cudaGetErrorString(le) + ")");
    le = cudaLaunchKernelExC(&lc, reinterpret_cast<const void*>(&stream_kernel), args);
    if (le != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("stream kernel launch: ") + cudaGetErrorString(le));
  }
  s->running = true;
  // wait (bounded) for the kernel to report READY
  const auto t0 = std::chrono::steady_clock::now();
  while (*resp_status(s) != kStReady) {
    if (*resp_status(s) == kStWatchdog || std::chrono::steady_clock::now() - t0 > std::chrono::seconds(10)) {
      return fail(BPC_ERR_DEVICE, "the stream kernel did not report ready");
    }
    cudaError_t q = cudaStreamQuery(s->stream);
    if (q != cudaErrorNotReady) {
      s->running = false;
      return fail(BPC_ERR_DEVICE, std::string("the stream kernel ended before ready: ") + cudaGetErrorString(q));
    }
  }
  return 0;
}

extern "C" int bpc_stream_round(bpc_stream* s, const uint8_t* round_dets, uint8_t* residual, float* logits,
                                int64_t timeout_us) {
  if (!s || !round_dets) return fail(BPC_ERR_ARG, "null argument");
  if (!s->running) return fail(BPC_ERR_ARG, "the stream kernel is not running");
  if (s->desynced)
    return fail(BPC_ERR_DEVICE, "an earlier round timed out before its response; stop and start the stream again");
  const StreamArgs& a = s->args;
  volatile uint8_t* dst = s->host + kReqDets;
  for (int i = 0; i < 2 * a.nh; ++i) dst[i] = round_dets[i];
  *reinterpret_cast<volatile uint32_t*>(s->host + 8) = kCmdRound;
  std::atomic_thread_fence(std::memory_order_release);
  const uint64_t tag = ++s->tag;
  *req_tag(s) = tag;
  const auto t0 = std::chrono::steady_clock::now();
  while (*resp_tag(s) != tag) {
    const uint32_t st = *resp_status(s);
    if (st == kStWatchdog || st == kStIdle || st == kStStopped) {
      s->running = false;
      return fail(BPC_ERR_DEVICE, "the stream kernel left (status " + std::to_string(st) + ")");
    }
    if (timeout_us > 0 && std::chrono::steady_clock::now() - t0 > std::chrono::microseconds(timeout_us)) {
      // the kernel may still answer this round later; a new request would overwrite the line it may be reading
      s->desynced = true;
      return fail(BPC_ERR_DEVICE, "no response within the timeout");
    }
  }
  std::atomic_thread_fence(std::memory_order_acquire);
  const uint8_t* src = s->host + kRespOff + kRespData;
  if (residual) std::memcpy(residual, src, a.N_c);
  if (logits) std::memcpy(logits, src + ((a.N_c + 15) & ~15), static_cast<size_t>(a.nq) * 8);
  return 0;
}

extern "C" int bpc_stream_run(bpc_stream* s, const uint8_t* rounds, int64_t n_rounds, uint8_t* residuals,
                              float* logits, int64_t* latency_ns, int64_t timeout_us) {
  if (!s || !rounds || n_rounds < 0) return fail(BPC_ERR_ARG, "invalid argument");
  const StreamArgs& a = s->args;
  for (int64_t i = 0; i < n_rounds; ++i) {
    const auto t0 = std::chrono::steady_clock::now();
    if (int e = bpc_stream_round(s, rounds + i * 2 * a.nh, residuals ? residuals + i * a.N_c : nullptr,
                                 logits ? logits + i * a.nq * 2 : nullptr, timeout_us))
      return e;
    if (latency_ns)
      latency_ns[i] = std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count();
  }
  return 0;
}

extern "C" int bpc_stream_stop(bpc_stream* s) {
  if (!s) return fail(BPC_ERR_ARG, "null stream");
  if (!s->running) return 0;
  *reinterpret_cast<volatile uint32_t*>(s->host + 8) = kCmdStop;
  std::atomic_thread_fence(std::memory_order_release);
  *req_tag(s) = ++s->tag;
  const auto t0 = std::chrono::steady_clock::now();
  cudaError_t q;
  while ((q = cudaStreamQuery(s->stream)) == cudaErrorNotReady) {
    if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(10))
      return fail(BPC_ERR_DEVICE, "the stream kernel did not stop");
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  s->running = false;
  if (q != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("stream kernel: ") + cudaGetErrorString(q));
  return *resp_status(s) == kStWatchdog ? fail(BPC_ERR_DEVICE, "the stream kernel's watchdog fired") : 0;
}

extern "C" int bpc_stream_status(const bpc_stream* s) {
  return s ? static_cast<int>(*reinterpret_cast<volatile const uint32_t*>(s->host + kRespOff + 8)) : -1;
}

extern "C" void bpc_stream_destroy(bpc_stream* s) {
  if (!s) return;
  if (s->running) bpc_stream_stop(s);
  if (s->stream) cudaStreamDestroy(s->stream);
  if (s->dev) cudaFree(s->dev);
  if (s->host) cudaFreeHost(s->host);
  delete s;
}
