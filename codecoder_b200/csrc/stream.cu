// Persistent streaming pre-decoder (sliding window of W rounds, batch 1, C = 64, K = 8): one resident kernel that
// serves rounds through a request line in mapped host memory, the protocol of the reference's persistent kernel
// (evaluation/timing/d7/kernel.cu:310-369,440-527; router.cc:170-223,576-650): the host writes a round's detectors
// tagged with its sequence number -- in every 8-byte word of the line, as the reference's request tags every word
// (poll_k) -- the kernel publishes the round's residual syndrome and the newest round's X/Z logits with the same tag,
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
// A round: CTA 0 takes the request and hands the detectors to the others through L2; every CTA keeps its own copy of
// the window's detectors in shared memory.  L check -> data steps and L - 1 data -> check steps follow (the last
// layer's data -> check step does not reach the outputs).  The first step gathers its source rows straight from the
// embedding table by detector token, while the CTAs store the window's embedding for the later steps.  The last
// check -> data step writes the newest round's logits and XORs the predicted flips into the residual; CTA 0 copies
// the residual and the logits to the response and releases the tag.  A one-cluster layout of the same arithmetic
// follows the grid kernel below.
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

// Request / response lines in mapped host memory.  Request: 8-byte words, word w = detectors 4w .. 4w + 3 (low half)
// and the round's sequence number (high half: 31 bits, bit 31 = stop), each word written and read whole, so that
// every word carries its own validity and one read of the line both finds a new round and delivers it.
// Response: u64 tag, u32 status, then residual, logits.
constexpr uint32_t kSeqMask = 0x7fffffffu, kSeqStop = 0x80000000u;
constexpr int kRespOff = 4096;
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
  unsigned long long* trace;    // phase stamps of the rounds served, or null (off)
};

// Tracing: thread 0 of every CTA stamps the global timer at the phase boundaries of each step into
// trace[CTA][step][k] (slot kTraceSlots - 1: the round's request, embedding and publication), overwritten round after
// round, so that after a run the buffer holds the last round served.  Off (no stores) when the pointer is null.
constexpr int kTraceCtas = 64, kTraceSlots = 16, kTraceK = 8;
__device__ __forceinline__ void trace_stamp(const StreamArgs& a, int cta, int slot, int k) {
  if (a.trace != nullptr && threadIdx.x == 0)
    a.trace[(static_cast<int64_t>(cta) * kTraceSlots + slot) * kTraceK + k] = globaltimer_ns();
}

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
// The arrival is a release reduction (it orders the CTA's earlier writes, seen through the CTA barrier, before the
// count); the poll is one acquire load per iteration, the abort flag read only every 32nd (an acquire load holds
// back every later load, so a flag read each time would add a second L2 round trip to each poll).
__device__ bool grid_sync(const StreamArgs& a, unsigned long long n, volatile int* cta_abort) {
  __syncthreads();
  if (threadIdx.x == 0) {
    asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(a.bar) : "memory");
    const unsigned long long target = (n + 1) * gridDim.x;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0;; ++i) {
      unsigned long long v;
      asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(a.bar) : "memory");
      if (v >= target) break;
      if (((i & 31) == 31 && *reinterpret_cast<volatile int*>(a.abort_flag)) || globaltimer_ns() - t0 > a.step_ns) {
        atomicExch(a.abort_flag, 1);
        *cta_abort = 1;
        break;
      }
    }
  }
  __syncthreads();
  return !*cta_abort;
}

// The next request, read by every thread of one CTA (each polls its words of the line, see above): the detector words
// go to dst (4 bytes each).  Returns kCmdRound, or kCmdStop on a stop command, once another CTA gave up, or after the
// idle limit (then the status word says idle).  Every thread of the CTA calls it; it ends past a CTA barrier.
__device__ uint32_t take_request(const StreamArgs& a, uint64_t tag, uint32_t* dst) {
  const uint32_t want = static_cast<uint32_t>(tag + 1) & kSeqMask;
  const int nw = (2 * a.nh + 3) / 4;
  int got = 1, stop = 0;
  const uint64_t t0 = globaltimer_ns();
  for (int w = threadIdx.x; w < nw; w += blockDim.x) {
    int ok = 0;
    while (true) {
      const uint64_t v = ld_volatile_u64(a.req + 8 * w);
      const uint32_t hi = static_cast<uint32_t>(v >> 32);
      if ((hi & kSeqMask) == want) {
        ok = 1;
        stop |= (hi & kSeqStop) ? 1 : 0;
        dst[w] = static_cast<uint32_t>(v);
        break;
      }
      if (*reinterpret_cast<volatile const int*>(a.abort_flag) || globaltimer_ns() - t0 > a.idle_ns) break;
    }
    got &= ok;
  }
  const int all = __syncthreads_and(got);
  const int any_stop = __syncthreads_or(stop);
  if (!all && threadIdx.x == 0 && !*reinterpret_cast<volatile const int*>(a.abort_flag))
    *reinterpret_cast<volatile uint32_t*>(a.resp + 8) = kStIdle;
  return all && !any_stop ? kCmdRound : kCmdStop;
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__global__ void __launch_bounds__(kSThreads, 1)
    stream_kernel(const __grid_constant__ CUtensorMap tmWc, const __grid_constant__ CUtensorMap tmWd,
                  const __grid_constant__ CUtensorMap tmHc, const __grid_constant__ CUtensorMap tmHd,
                  const __grid_constant__ CUtensorMap tmEmb, const StreamArgs a) {
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
  uint8_t* s_ring = reinterpret_cast<uint8_t*>(bars + 8);  // the window's detectors [type][ring slot][nh] (each CTA
                                                          // keeps its own copy: no L2 reads to embed a round)

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
  for (int e = t; e < 2 * a.W * a.nh; e += kSThreads) s_ring[e] = 0;

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
    tma_prefetch_desc(&tmEmb);
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
  // check node n of the window -> its detector (this CTA's copy of the window) and its embedding row 2 type + det
  auto window_det = [&](int n) -> uint32_t {
    const int ty = n / nx, tt = (n / a.nh) % a.W, sidx = n % a.nh;
    return s_ring[(ty * a.W + (head + tt) % a.W) * a.nh + sidx];
  };
  auto window_token = [&](int n) -> int32_t { return 2 * (n / nx) + static_cast<int32_t>(window_det(n)); };
  // this CTA's share of the stored window embedding (read by the data -> check steps' residuals and the later
  // check -> data gathers) and of the residual words
  auto embed_share = [&]() {
    const int g = blockIdx.x * kSThreads + t;           // node g / 8, 16-byte chunk g % 8
    const int n = g >> 3, j = g & 7;
    if (n < a.N_c) {
      reinterpret_cast<uint4*>(a.hc + static_cast<int64_t>(n) * kSC)[j] =
          __ldg(reinterpret_cast<const uint4*>(a.embed + window_token(n) * kSC) + j);
      if (j == 0 && (n & 3) == 0) {
        uint32_t w = 0;
        for (int k = 0; k < 4 && n + k < a.N_c; ++k) w |= window_det(n + k) << (8 * k);
        a.res[n >> 2] = w;
      }
    }
  };

  while (!*cta_abort) {
    trace_stamp(a, blockIdx.x, kTraceSlots - 1, 0);
    // ------------------------------------------------------------------ the next request (idle watchdog)
    // CTA 0 polls the host line, copies the detectors into device memory and releases the round on a device flag;
    // the other CTAs poll that flag in L2 (one reader of host memory instead of 64)
    if (blockIdx.x == 0) {
      const uint32_t cmd = take_request(a, tag, reinterpret_cast<uint32_t*>(a.dev_req));
      if (t == 0) *s_cmd = cmd;
      __syncthreads();
      if (t == 0) {
        __threadfence();
        const unsigned long long f = *s_cmd == kCmdRound ? tag + 1 : kStopFlag;
        asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(a.round_flag), "l"(f) : "memory");
      }
    } else if (t == 0) {
      const uint64_t t0 = globaltimer_ns();
      uint32_t cmd = kCmdStop;
      for (uint32_t i = 0;; ++i) {
        unsigned long long v;
        asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(a.round_flag) : "memory");
        if (v == tag + 1) {
          cmd = kCmdRound;
          break;
        }
        if (v == kStopFlag || ((i & 31) == 31 && *reinterpret_cast<volatile int*>(a.abort_flag))) break;
        if (globaltimer_ns() - t0 > a.idle_ns + 1000000000ull) break;   // CTA 0 gives up first
      }
      *s_cmd = cmd;
    }
    __syncthreads();
    if (*s_cmd != kCmdRound) break;
    trace_stamp(a, blockIdx.x, kTraceSlots - 1, 1);
    ++tag;
    // the new round enters this CTA's copy of the window (its newest slot; the oldest round leaves)
    for (int e = t; e < 2 * a.nh; e += kSThreads) {
      const int ty = e / a.nh, sidx = e % a.nh;
      s_ring[(ty * a.W + (head + a.W - 1) % a.W) * a.nh + sidx] = __ldcg(a.dev_req + e) & 1;
    }
    __syncthreads();
    trace_stamp(a, blockIdx.x, kTraceSlots - 1, 2);
    // ------------------------------------------------------------------ L check -> data and L - 1 data -> check steps
    bool failed = false;
    for (int step = 0; step < 2 * L - 1 && !failed; ++step) {
      const int l = step >> 1;
      const bool c2d = (step & 1) == 0;
      const bool active = c2d ? has_c2d : has_d2c;
      const bool last = step == 2 * L - 2;
      trace_stamp(a, blockIdx.x, step, 0);
      if (active) {
        // the first step reads the embedded check nodes straight from the embedding table: row 2 type + det of the
        // source node (a pad reads row 4, past the table: zeros); later steps read the stored features
        const CUtensorMap* tm = step == 0 ? &tmEmb : c2d ? &tmHc : &tmHd;
        const int src = c2d ? src_c2d : src_d2c;
        const int nsrc = c2d ? a.N_c : a.N_d;
        fence_proxy_async_global();                    // the gathers read what earlier steps stored
        const int32_t xr = (src < 0 || src >= nsrc) ? (step == 0 ? 4 : nsrc) : step == 0 ? window_token(src) : src;
        const int q4 = lane & ~3;
        const int32_t i0 = __shfl_sync(0xffffffffu, xr, q4), i1 = __shfl_sync(0xffffffffu, xr, q4 + 1),
                      i2 = __shfl_sync(0xffffffffu, xr, q4 + 2), i3 = __shfl_sync(0xffffffffu, xr, q4 + 3);
        if (lane == 0) mbar_arrive_expect_tx(smem_u32(full), 32 * 128);
        __syncwarp();
        if ((lane & 3) == 0) tma_gather4(smem_u32(sA + t * 128), tm, 0, i0, i1, i2, i3, smem_u32(full));
        if (step == 0) embed_share();                  // while the gathers run
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
          trace_stamp(a, blockIdx.x, step, 1);
          if (good) {
            tc_fence_after();
            const uint64_t ad = sdesc_k_sw128(smem_u32(sA));
            const uint64_t bd = sdesc_k_sw128(smem_u32((c2d ? sWc : sWd) + l * kSWBytes));
#pragma unroll
            for (int k = 0; k < 4; ++k)
              tc_mma_ss(tmem_base, ad + ((k * 32) >> 4), bd + ((k * 32) >> 4), idesc, k ? 1u : 0u);
          }
          tc_commit(smem_u32(accf));
          trace_stamp(a, blockIdx.x, step, 2);
        }
        ph_full ^= 1u;
        good = mbar_wait(smem_u32(accf), ph_acc, cta_abort, nullptr, a.step_ns) && good && !*cta_abort;
        ph_acc ^= 1u;
        trace_stamp(a, blockIdx.x, step, 3);
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
        __syncwarp();
        // warp w staged the rows of owners 2w and 2w + 1: it sends them at once, without waiting for the other warps
        if (lane == 0) {
          for (int jj = 2 * warp; jj < 2 * warp + 2; ++jj)
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
        trace_stamp(a, blockIdx.x, step, 4);
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
        if (lane == 0) bulk_wait_read();               // sO is free for the next step
        if (t == 0) mbar_arrive_expect_tx(smem_u32(recv), kSPart);   // re-armed before the peers' next copies
        if (!rec || !good) {
          if (t == 0) atomicExch(a.abort_flag, 1);
          *cta_abort = 1;
        }
      } else if (step == 0) {
        embed_share();
      }
      trace_stamp(a, blockIdx.x, step, 5);
      if (!grid_sync(a, nbar++, cta_abort)) failed = true;
      trace_stamp(a, blockIdx.x, step, 6);
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
      if (t == 0) *reinterpret_cast<volatile unsigned long long*>(a.resp) = tag;
    }
    trace_stamp(a, blockIdx.x, kTraceSlots - 1, 4);
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

// ---------------------------------------------------------------------------------------------------------------
// One-cluster layout: the whole round inside one thread-block cluster of 2 x (tiles per step) CTAs (16 at d = 17,
// window 3), so that no step hand-off goes through an L2 flag.  CTA pair (tile, half) splits a tile's relations:
// the low CTA gathers and multiplies relations 0-3, the high CTA relations 4-7, each into four TMEM accumulators (one
// per relation, as the per-relation partials of the grid layout).  The low CTA adds its four in relation order and
// pushes the 128 x 64 fp32 sum to the high CTA in one bulk shared -> distributed-shared copy; the high CTA adds its
// own four to it in order -- the same fp32 sum, in the same order, as the grid layout's owner -- and runs the
// epilogue (GELU, residual, head, XOR) for all 128 rows.  The relation matrices do not fit in shared memory for every
// layer, so each step's four are loaded into one of two buffers while the step before runs.  Steps are separated by
// a cluster barrier made of two alternating mbarriers that every CTA arrives on remotely (bounded waits, unlike the
// hardware cluster barrier, so a CTA that gives up cannot leave its peers waiting forever); CTA 0 hands each round's
// command and detectors to its peers with stores into their shared memory and one remote arrival each.
constexpr int kQThreads = 256;
constexpr int kQRel = 4;                                 // relations per CTA: a pair splits the 8
constexpr int kQMaxCtas = 16;
constexpr uint32_t kQWBuf = kQRel * kSWBytes;            // 32 KB: one step's four relation matrices
constexpr uint32_t kQA = kQRel * kSABytes;               // 64 KB: four relations' gathered rows
constexpr uint32_t kQX = kSRows * kSC * 4;               // 32 KB: fp32 sum of relations 0-3 for 128 rows
constexpr uint32_t kQoW = 0;
constexpr uint32_t kQoA = kQoW + 2 * kQWBuf;
constexpr uint32_t kQoX = kQoA + kQA;
constexpr uint32_t kQoIdx = kQoX + kQX;                  // int32 [step type][relation][row]
constexpr uint32_t kQoLg = kQoIdx + 2 * kQRel * kSRows * 4;
constexpr uint32_t kQoNew = kQoLg + kSRows * 8;          // the round's detectors (2 nh <= 1024 bytes)
constexpr uint32_t kQoBar = kQoNew + 1024;
constexpr int kQSmem = static_cast<int>(kQoBar) + 256 + 1024;

__device__ __forceinline__ void st_cluster_v4(uint32_t addr_cluster, uint4 v) {
  asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr_cluster), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void fence_acq_rel_cluster() { asm volatile("fence.acq_rel.cluster;" ::: "memory"); }

// Bounded wait (cluster-scope acquire) on an mbarrier that takes remote arrivals: false after `limit_ns` or once any
// CTA has set the kernel's abort flag.
__device__ bool cl_wait(uint32_t bar, uint32_t parity, const int* abort_flag, uint64_t limit_ns) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & 31) == 31 && *reinterpret_cast<volatile const int*>(abort_flag)) return false;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// Cluster barrier: every CTA arrives on barrier `k & 1` of every CTA (lane j of warp 0 on CTA j's, after a
// cluster-scope fence that orders this CTA's earlier writes, global and shared, before the peers' acquire), then
// waits (bounded) on its own.  Two barriers alternate so that an arrival for the next step can never land in the
// phase of this one.  False once this CTA or any other has given up.
__device__ bool cl_sync(uint32_t bars2, uint32_t& phases, int& k, int nct, const StreamArgs& a,
                        volatile int* cta_abort) {
  tc_fence_before();
  __syncthreads();
  const int t = threadIdx.x;
  const uint32_t bar = bars2 + 8 * (k & 1);
  if (t < nct) {
    fence_acq_rel_cluster();
    mbar_arrive_remote(map_to_cta(bar, t));
  }
  if (t == 0 && !*cta_abort && !cl_wait(bar, (phases >> (k & 1)) & 1, a.abort_flag, a.step_ns)) {
    atomicExch(a.abort_flag, 1);
    *cta_abort = 1;
  }
  phases ^= 1u << (k & 1);
  ++k;
  __syncthreads();
  tc_fence_after();
  return !*cta_abort;
}

__global__ void __launch_bounds__(kQThreads, 1)
    stream_cluster_kernel(const __grid_constant__ CUtensorMap tmWc, const __grid_constant__ CUtensorMap tmWd,
                          const __grid_constant__ CUtensorMap tmHc, const __grid_constant__ CUtensorMap tmHd,
                          const StreamArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sW = smem + kQoW;
  uint8_t* sA = smem + kQoA;
  uint8_t* sX = smem + kQoX;
  int32_t* sIdx = reinterpret_cast<int32_t*>(smem + kQoIdx);
  float2* sLg = reinterpret_cast<float2*>(smem + kQoLg);
  uint8_t* sNew = smem + kQoNew;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kQoBar);
  const uint32_t b_wfull = smem_u32(bars);               // 2: the two weight buffers
  const uint32_t b_full = smem_u32(bars + 2);            // 4: one per relation's gathered rows
  const uint32_t b_acc = smem_u32(bars + 6);
  const uint32_t b_recv = smem_u32(bars + 7);            // the high CTA's: the low CTA's sum arrived
  const uint32_t b_step = smem_u32(bars + 8);            // 2: the alternating cluster barriers
  const uint32_t b_go = smem_u32(bars + 10);             // CTA 0 handed over a command
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* cta_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile uint32_t* s_cmd = reinterpret_cast<volatile uint32_t*>(tmem_slot + 2);

  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int rank = static_cast<int>(cluster_ctarank());
  const int nct = static_cast<int>(gridDim.x);           // the grid is one cluster
  const int tile = rank >> 1, half = rank & 1;           // relations 4 half .. 4 half + 3 of tile `tile`
  const int L = a.layers, S = 2 * L - 1;
  const int nx = a.W * a.nh;
  const bool has_c2d = tile < a.tiles_c2d;
  const int c2d_begin = tile * kSRows, c2d_end = min(a.N_d, c2d_begin + kSRows);
  const bool zt = tile >= a.tiles_x;
  const bool has_d2c = tile < 2 * a.tiles_x;
  const int d2c_begin = zt ? nx + (tile - a.tiles_x) * kSRows : tile * kSRows;
  const int d2c_end = zt ? min(a.N_c, d2c_begin + kSRows) : min(nx, d2c_begin + kSRows);
  // the epilogue's rows and channels: TMEM lane quarter warp % 4 (rows 32 (warp % 4) + lane), channel half warp / 4
  const int row = 32 * (warp & 3) + lane, hh = warp >> 2;

  // source rows of this CTA's four relations for both step types (pads and rows past the tile read the zero row
  // past the map's end)
  for (int e = t; e < 2 * kQRel * kSRows; e += kQThreads) {
    const int ty = e / (kQRel * kSRows), j = (e / kSRows) % kQRel, rr = e % kSRows;
    const bool c2d = ty == 0;
    const int b = c2d ? c2d_begin : d2c_begin, en = c2d ? c2d_end : d2c_end, nsrc = c2d ? a.N_c : a.N_d;
    int src = -1;
    if ((c2d ? has_c2d : has_d2c) && b + rr < en)
      src = __ldg((c2d ? a.c2d : a.d2c) + static_cast<int64_t>(b + rr) * kSRel + kQRel * half + j);
    sIdx[e] = (src >= 0 && src < nsrc) ? src : nsrc;
  }
  if (t == 0) {
    mbar_init(b_wfull, 1);
    mbar_init(b_wfull + 8, 1);
    for (int j = 0; j < kQRel; ++j) mbar_init(b_full + 8 * j, 1);
    mbar_init(b_acc, 1);
    mbar_init(b_recv, 1);
    mbar_init(b_step, nct);
    mbar_init(b_step + 8, nct);
    mbar_init(b_go, 1);
    if (half == 1) mbar_arrive_expect_tx(b_recv, kQX);   // armed for the first step; the partner sends after a barrier
    *cta_abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmWc);
    tma_prefetch_desc(&tmWd);
    tma_prefetch_desc(&tmHc);
    tma_prefetch_desc(&tmHd);
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  cluster_arrive_release();                              // every CTA's barriers exist before any remote arrival
  cluster_wait_acquire();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (rank == 0 && t == 0) {
    *reinterpret_cast<volatile uint32_t*>(a.resp + 8) = kStReady;
    __threadfence_system();
  }
  auto active = [&](int step) { return (step & 1) == 0 ? has_c2d : has_d2c; };
  // thread 0: the four relation matrices of `step` into weight buffer step % 2
  auto load_w = [&](int step) {
    const int l = step >> 1, b = step & 1;
    const uint32_t dst = smem_u32(sW + b * kQWBuf), bar = b_wfull + 8 * b;
    mbar_arrive_expect_tx(bar, kQWBuf);
    for (int j = 0; j < kQRel; ++j) {
      if ((step & 1) == 0)
        tma_load_3d(dst + j * kSWBytes, &tmWc, 0, kQRel * half + j, l * kSC, bar);
      else
        tma_load_3d(dst + j * kSWBytes, &tmWd, 0, kQRel * half + j, (2 * l + (zt ? 1 : 0)) * kSC, bar);
    }
  };
  uint32_t wph = 0, ph_full = 0, ph_acc = 0, ph_recv = 0, sph = 0, ph_go = 0;
  int nsync = 0;
  bool w_pending[2] = {false, false};                    // thread 0: weight loads not yet waited for
  uint32_t drain_full = 0;                               // thread 0: 1 + the phase of gathers given up on
  uint64_t tag = 0;
  int head = 0;
  const uint32_t idesc = idesc_bf16_f32(kSRows, kSC);
  const int nchunk = (2 * a.nh + 15) / 16;

  while (!*cta_abort) {
    trace_stamp(a, rank, kTraceSlots - 1, 0);
    // the first step's relation matrices do not depend on the round: load them while waiting for it
    if (t == 0 && active(0)) {
      load_w(0);
      w_pending[0] = true;
    }
    // ------------------------------------------------------------------ the next request (idle watchdog)
    if (rank == 0) {
      const uint32_t cmd = take_request(a, tag, reinterpret_cast<uint32_t*>(sNew));
      if (t == 0) *s_cmd = cmd;
      __syncthreads();
      // one thread per CTA: the command and the detectors into that CTA's shared memory, then its go arrival (the
      // arrival releases this thread's stores)
      if (t < nct) {
        const uint32_t cmd = *s_cmd;
        if (t != 0) {
          if (cmd == kCmdRound)
            for (int e = 0; e < nchunk; ++e)
              st_cluster_v4(map_to_cta(smem_u32(sNew) + 16 * e, t), reinterpret_cast<const uint4*>(sNew)[e]);
          st_cluster_u32(map_to_cta(smem_u32(const_cast<uint32_t*>(s_cmd)), t), cmd);
        }
        fence_acq_rel_cluster();
        mbar_arrive_remote(map_to_cta(b_go, t));
      }
    }
    if (t == 0 && !cl_wait(b_go, ph_go, a.abort_flag, a.idle_ns + 1000000000ull)) *s_cmd = kCmdStop;
    ph_go ^= 1u;
    __syncthreads();
    if (*s_cmd != kCmdRound) break;
    trace_stamp(a, rank, kTraceSlots - 1, 1);
    ++tag;
    // ------------------------------------------------------------------ embed the window and reset the residual
    for (int g = rank * kQThreads + t; g < a.N_c * 8; g += nct * kQThreads) {
      const int n = g >> 3, j = g & 7;
      const int ty = n / nx, tt = (n / a.nh) % a.W, s = n % a.nh;
      const uint8_t det = tt == a.W - 1 ? (sNew[ty * a.nh + s] & 1)
                                        : (__ldcg(a.ring + (ty * a.W + (head + tt) % a.W) * a.nh + s) & 1);
      reinterpret_cast<uint4*>(a.hc + static_cast<int64_t>(n) * kSC)[j] =
          __ldg(reinterpret_cast<const uint4*>(a.embed + (2 * ty + det) * kSC) + j);
      if (j == 0 && (n & 3) == 0) {
        uint32_t w = 0;
        for (int k = 0; k < 4 && n + k < a.N_c; ++k) {
          const int m = n + k;
          const int tym = m / nx, ttm = (m / a.nh) % a.W, sm = m % a.nh;
          const uint8_t dm = ttm == a.W - 1 ? (sNew[tym * a.nh + sm] & 1)
                                            : (__ldcg(a.ring + (tym * a.W + (head + ttm) % a.W) * a.nh + sm) & 1);
          w |= static_cast<uint32_t>(dm) << (8 * k);
        }
        a.res[n >> 2] = w;
      }
    }
    // the new round enters the ring (the newest slot of this window; no CTA reads it this round)
    if (rank == 0)
      for (int e = t; e < 2 * a.nh; e += kQThreads) {
        const int ty = e / a.nh, s = e % a.nh;
        a.ring[(ty * a.W + (head + a.W - 1) % a.W) * a.nh + s] = sNew[e] & 1;
      }
    trace_stamp(a, rank, kTraceSlots - 1, 2);
    if (!cl_sync(b_step, sph, nsync, nct, a, cta_abort)) break;
    trace_stamp(a, rank, kTraceSlots - 1, 3);
    // ------------------------------------------------------------------ L check -> data and L - 1 data -> check steps
    bool failed = false;
    for (int step = 0; step < S && !failed; ++step) {
      const int l = step >> 1;
      const bool c2d = (step & 1) == 0;
      const bool last = step == S - 1;
      const bool next_w = step + 1 < S && active(step + 1);
      trace_stamp(a, rank, step, 0);
      if (active(step)) {
        const CUtensorMap* tm = c2d ? &tmHc : &tmHd;
        const int ob = c2d ? c2d_begin : d2c_begin, oe = c2d ? c2d_end : d2c_end;
        __nv_bfloat16* y = c2d ? a.hd : a.hc;
        const bool resid = !(c2d && l == 0);
        const int on = ob + row;
        const bool o_ok = on < oe;
        // warp j < 4 gathers relation j's 128 source rows, four per lane
        if (warp < kQRel) {
          fence_proxy_async_global();                  // the gathers read what earlier steps stored
          const int32_t* ix = sIdx + ((c2d ? 0 : 1) * kQRel + warp) * kSRows + 4 * lane;
          if (lane == 0) mbar_arrive_expect_tx(b_full + 8 * warp, kSABytes);
          __syncwarp();
          tma_gather4(smem_u32(sA + warp * kSABytes + lane * 512), tm, 0, ix[0], ix[1], ix[2], ix[3],
                      b_full + 8 * warp);
        }
        // the high CTA's residual rows (outputs of earlier steps, through L2)
        uint4 res[4] = {};
        if (half == 1 && resid && o_ok)
#pragma unroll
          for (int q = 0; q < 4; ++q)
            res[q] = __ldcg(reinterpret_cast<const uint4*>(y + static_cast<int64_t>(on) * kSC + 32 * hh) + q);
        bool good = true;
        if (t == 0) {
          const int b = step & 1;
          good = mbar_wait(b_wfull + 8 * b, (wph >> b) & 1, cta_abort, nullptr, a.step_ns);
          trace_stamp(a, rank, step, 1);
          wph ^= 1u << b;
          if (good) w_pending[b] = false;
          for (int j = 0; j < kQRel && good; ++j) {
            good = mbar_wait(b_full + 8 * j, ph_full, cta_abort, nullptr, a.step_ns);
            if (good) {
              tc_fence_after();
              const uint64_t ad = sdesc_k_sw128(smem_u32(sA + j * kSABytes));
              const uint64_t bd = sdesc_k_sw128(smem_u32(sW + b * kQWBuf + j * kSWBytes));
#pragma unroll
              for (int k = 0; k < 4; ++k)
                tc_mma_ss(tmem_base + 64 * j, ad + ((k * 32) >> 4), bd + ((k * 32) >> 4), idesc, k ? 1u : 0u);
            }
          }
          trace_stamp(a, rank, step, 2);
          tc_commit(b_acc);
          if (!good) drain_full = ph_full + 1;         // gathers of this step may still be landing
          // the next step's matrices go to the other buffer, whose last reader (the step before) has completed
          if (next_w && good) {
            load_w(step + 1);
            w_pending[(step + 1) & 1] = true;
          }
        }
        ph_full ^= 1u;
        good = mbar_wait(b_acc, ph_acc, cta_abort, nullptr, a.step_ns) && good && !*cta_abort;
        ph_acc ^= 1u;
        trace_stamp(a, rank, step, 3);
        tc_fence_after();
        const uint32_t tl = tmem_base + (static_cast<uint32_t>(32 * (warp & 3)) << 16) + 32 * hh;
        float s[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) s[e] = 0.f;
        if (half == 0) {
          // relations 0-3 added in order, as float4 chunks (channels 4c .. 4c + 3) of every row, to the partner
#pragma unroll
          for (int j = 0; j < kQRel; ++j) {
            float v[32];
            tmem_ld32(tl + 64 * j, v);
#pragma unroll
            for (int e = 0; e < 32; ++e) s[e] += v[e];
          }
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(sX + ((8 * hh + q) * kSRows + row) * 16) =
                make_float4(s[4 * q], s[4 * q + 1], s[4 * q + 2], s[4 * q + 3]);
          tc_fence_before();
          fence_proxy_async_smem();
          __syncthreads();
          if (t == 0 && good)
            bulk_s2cluster(map_to_cta(smem_u32(sX), rank + 1), smem_u32(sX), kQX, map_to_cta(b_recv, rank + 1));
          trace_stamp(a, rank, step, 4);
        } else {
          const bool rec = cl_wait(b_recv, ph_recv, a.abort_flag, a.step_ns);
          trace_stamp(a, rank, step, 4);
          ph_recv ^= 1u;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 v = *reinterpret_cast<const float4*>(sX + ((8 * hh + q) * kSRows + row) * 16);
            s[4 * q] = v.x;
            s[4 * q + 1] = v.y;
            s[4 * q + 2] = v.z;
            s[4 * q + 3] = v.w;
          }
#pragma unroll
          for (int j = 0; j < kQRel; ++j) {
            float v[32];
            tmem_ld32(tl + 64 * j, v);
#pragma unroll
            for (int e = 0; e < 32; ++e) s[e] += v[e];
          }
          uint32_t o[16];
          const uint32_t* hres = reinterpret_cast<const uint32_t*>(res);
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            uint64_t xv = gelu_tanh_fast2(f2_pack(s[2 * e], s[2 * e + 1]));
            if (resid) xv = f2_add(xv, bf2_to_f2(hres[e]));
            o[e] = f2_to_bf2(xv);
          }
          if (o_ok && rec)
#pragma unroll
            for (int q = 0; q < 4; ++q)
              reinterpret_cast<uint4*>(y + static_cast<int64_t>(on) * kSC + 32 * hh)[q] =
                  make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
          if (last) {
            // the head over 8-channel groups (pairs in order, then the two halves of each pair), the groups added
            // as a tree: ((g0 + g1) + (g2 + g3)) + ((g4 + g5) + (g6 + g7)); this thread holds groups 4 hh .. 4 hh + 3
            float p0[4], p1[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint64_t lg0 = 0, lg1 = 0;
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const uint64_t f = bf2_to_f2(o[4 * q + e]);
                const int col = 32 * hh + 8 * q + 2 * e;
                lg0 = f2_fma(f, *reinterpret_cast<const uint64_t*>(a.head_w + col), lg0);
                lg1 = f2_fma(f, *reinterpret_cast<const uint64_t*>(a.head_w + kSC + col), lg1);
              }
              p0[q] = f2_lo(lg0) + f2_hi(lg0);
              p1[q] = f2_lo(lg1) + f2_hi(lg1);
            }
            const float q0 = (p0[0] + p0[1]) + (p0[2] + p0[3]), q1 = (p1[0] + p1[1]) + (p1[2] + p1[3]);
            if (hh == 1) sLg[row] = make_float2(q0, q1);
            __syncthreads();
            if (hh == 0 && o_ok && rec) {
              const float2 u = sLg[row];
              float l0 = q0 + u.x, l1 = q1 + u.y;
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
          __syncthreads();                             // every thread is past its wait before the barrier is re-armed
          if (t == 0) mbar_arrive_expect_tx(b_recv, kQX);
          if (!rec) good = false;
        }
        if (!good) {
          if (t == 0) atomicExch(a.abort_flag, 1);
          *cta_abort = 1;
        }
      } else if (t == 0 && next_w) {
        load_w(step + 1);
        w_pending[(step + 1) & 1] = true;
      }
      trace_stamp(a, rank, step, 5);
      if (!cl_sync(b_step, sph, nsync, nct, a, cta_abort)) failed = true;
      trace_stamp(a, rank, step, 6);
    }
    if (failed || *cta_abort) break;
    // ------------------------------------------------------------------ publish: results in 16-byte stores, then the tag
    if (rank == 0) {
      const int nres = (a.N_c + 15) / 16, nlg = (a.nq * 8 + 15) / 16;
      volatile uint8_t* rp = a.resp + kRespData;
      for (int e = t; e < nres + nlg; e += kQThreads) {
        const uint4 v = e < nres ? __ldcg(reinterpret_cast<const uint4*>(a.res) + e)
                                 : __ldcg(reinterpret_cast<const uint4*>(a.dev_out + ((a.N_c + 15) & ~15)) + (e - nres));
        st_volatile_u4(rp + 16 * e, v);
      }
      __threadfence_system();
      __syncthreads();
      if (t == 0) *reinterpret_cast<volatile unsigned long long*>(a.resp) = tag;
    }
    trace_stamp(a, rank, kTraceSlots - 1, 4);
    head = (head + 1) % a.W;
  }
  if (rank == 0 && t == 0) {
    const int ab = *reinterpret_cast<volatile int*>(a.abort_flag);
    volatile uint32_t* st = reinterpret_cast<volatile uint32_t*>(a.resp + 8);
    if (ab) *st = kStWatchdog;
    else if (*st != kStIdle) *st = kStStopped;
    __threadfence_system();
  }
  // copies into this CTA's shared memory still in flight land before it is given up (bounded): a weight load issued
  // for a round that never came; after a watchdog, gathers given up on and the partner's sum
  if (t == 0) {
    const uint64_t t0 = globaltimer_ns();
    for (int b = 0; b < 2; ++b)
      if (w_pending[b])
        while (!mbar_try_wait(b_wfull + 8 * b, (wph >> b) & 1) && globaltimer_ns() - t0 < 100000000ull) {
        }
    if (drain_full)
      for (int j = 0; j < kQRel; ++j)
        while (!mbar_try_wait(b_full + 8 * j, (drain_full - 1) & 1) && globaltimer_ns() - t0 < 100000000ull) {
        }
    if (half == 1 && *reinterpret_cast<volatile int*>(a.abort_flag))
      while (!mbar_try_wait_cluster(b_recv, ph_recv) && globaltimer_ns() - t0 < 2000000ull) {
      }
  }
  // every CTA is done with its peers' shared memory before any leaves
  cluster_arrive_release();
  cluster_wait_acquire();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 256);
  }
}

}  // namespace
}  // namespace bpc

using namespace bpc;

struct bpc_stream {
  const bpc_predecoder* pd = nullptr;
  StreamArgs args{};
  CUtensorMap maps[5];          // W_c2d, W_d2c, h_c rows, h_d rows, embedding rows
  uint8_t* host = nullptr;      // mapped: request at 0, response at kRespOff
  uint8_t* host_dev = nullptr;
  void* dev = nullptr;          // hc, hd, ring, res, barrier, abort
  cudaStream_t stream = nullptr;
  bool running = false;
  bool desynced = false;        // a round was given up before its response: later rounds fail until stop / start
  uint64_t tag = 0;
  int smem = 0;
  int layout = BPC_STREAM_AUTO; // requested
  unsigned long long* trace = nullptr;  // device trace buffer (part of dev)
  bool tracing = false;
  int running_layout = 0;       // the layout of the kernel that runs (or ran last)
  int nct = 0;                  // CTAs of the one-cluster layout
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

// The request for sequence number s->tag: every word of the line written whole (aligned 8-byte stores), in any
// order -- each word carries the sequence number, so the kernel takes a word only once it is the new round's.
void write_request(bpc_stream* s, const uint8_t* dets, bool stop) {
  const uint32_t seq = (static_cast<uint32_t>(s->tag) & kSeqMask) | (stop ? kSeqStop : 0u);
  const int n = 2 * s->args.nh, nw = (n + 3) / 4;
  volatile uint64_t* line = reinterpret_cast<volatile uint64_t*>(s->host);
  for (int w = 0; w < nw; ++w) {
    uint32_t d = 0;
    if (dets)
      for (int k = 0; k < 4 && 4 * w + k < n; ++k) d |= static_cast<uint32_t>(dets[4 * w + k]) << (8 * k);
    line[w] = (static_cast<uint64_t>(seq) << 32) | d;
  }
}
volatile uint64_t* resp_tag(bpc_stream* s) { return reinterpret_cast<volatile uint64_t*>(s->host + kRespOff); }
volatile uint32_t* resp_status(bpc_stream* s) { return reinterpret_cast<volatile uint32_t*>(s->host + kRespOff + 8); }

}  // namespace

extern "C" int bpc_stream_create(const bpc_predecoder* h, int32_t window, int32_t nh, int32_t nq,
                                 int32_t idle_timeout_ms, bpc_stream** out) {
  return bpc_stream_create_ex(h, window, nh, nq, idle_timeout_ms, BPC_STREAM_AUTO, out);
}

extern "C" int bpc_stream_create_ex(const bpc_predecoder* h, int32_t window, int32_t nh, int32_t nq,
                                    int32_t idle_timeout_ms, int32_t layout, bpc_stream** out) {
  if (!h || !out) return fail(BPC_ERR_ARG, "null argument");
  *out = nullptr;
  if (layout != BPC_STREAM_AUTO && layout != BPC_STREAM_CLUSTERS && layout != BPC_STREAM_ONE_CLUSTER)
    return fail(BPC_ERR_ARG, "layout must be BPC_STREAM_AUTO, BPC_STREAM_CLUSTERS or BPC_STREAM_ONE_CLUSTER");
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
  if (reinterpret_cast<uintptr_t>(embed) & 15) return fail(BPC_ERR_ARG, "the embedding table is not 16-byte aligned");
  if (2 * window * nh > 2048 || 2 * nh > 1024 || 8 * ((2 * nh + 3) / 4) > kRespOff || kRespData + ((c.n_checks + 15) & ~15) + nq * 8 > 65536 - kRespOff)
    return fail(BPC_ERR_ARG, "the request or response does not fit its line");
  auto* s = new bpc_stream();
  s->pd = h;
  s->layout = layout;
  s->nct = 2 * std::max(tiles_c2d, 2 * tiles_x);
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
  const size_t o_trace = (o_out + ((a.N_c + 15) & ~15) + static_cast<size_t>(nq) * 8 + 16 + 255) & ~size_t(255);
  const size_t total = o_trace + sizeof(unsigned long long) * kTraceCtas * kTraceSlots * kTraceK;
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
  s->trace = reinterpret_cast<unsigned long long*>(d + o_trace);
  a.trace = nullptr;
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
      (e = rows2(&s->maps[2], a.hc, a.N_c)) || (e = rows2(&s->maps[3], a.hd, a.N_d)) ||
      (e = rows2(&s->maps[4], embed, 4))) {
    bpc_stream_destroy(s);
    return e;
  }
  s->smem = 1024 + 2 * c.layers * kSWBytes + kSABytes + 2 * kSPart + 64 + 2048;
  if (cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking) != cudaSuccess)
    return bail(BPC_ERR_LAUNCH, "cudaStreamCreate failed");
  *out = s;
  return 0;
}

namespace {

int wait_ready(bpc_stream* s);

// The one-cluster kernel, if a cluster of s->nct CTAs with its shared memory can be resident on this device:
// 0 launched, 1 not possible here (nothing launched), otherwise an error code.
int launch_one_cluster(bpc_stream* s, void** args) {
  const void* fn = reinterpret_cast<const void*>(&stream_cluster_kernel);
  if (s->nct > kQMaxCtas) return 1;
  if (int e = allow_smem(fn, kQSmem)) return e;
  if (s->nct > 8 && cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
    cudaGetLastError();
    return 1;
  }
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(s->nct);
  lc.blockDim = dim3(kQThreads);
  lc.dynamicSmemBytes = static_cast<size_t>(kQSmem);
  lc.stream = s->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = s->nct;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  int max_clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&max_clusters, fn, &lc) != cudaSuccess || max_clusters < 1) {
    cudaGetLastError();
    return 1;
  }
  const cudaError_t le = cudaLaunchKernelExC(&lc, fn, args);
  if (le != cudaSuccess)
    return fail(BPC_ERR_LAUNCH, std::string("one-cluster stream kernel launch: ") + cudaGetErrorString(le));
  return 0;
}

}  // namespace

extern "C" int bpc_stream_start(bpc_stream* s) {
  if (!s) return fail(BPC_ERR_ARG, "null stream");
  if (s->running) return fail(BPC_ERR_ARG, "the stream kernel already runs");
  std::memset(s->host, 0, 65536);
  s->tag = 0;
  s->desynced = false;
  if (cudaMemsetAsync(s->args.bar, 0, 256, s->stream) != cudaSuccess ||
      cudaMemsetAsync(s->args.ring, 0, 2 * s->args.W * s->args.nh, s->stream) != cudaSuccess)
    return fail(BPC_ERR_LAUNCH, "cudaMemsetAsync failed");
  s->args.trace = s->tracing ? s->trace : nullptr;
  if (s->tracing &&
      cudaMemsetAsync(s->trace, 0, sizeof(unsigned long long) * kTraceCtas * kTraceSlots * kTraceK, s->stream) !=
          cudaSuccess)
    return fail(BPC_ERR_LAUNCH, "cudaMemsetAsync failed");
  // BPC_STREAM_AUTO runs the 8-cluster layout: measured faster on B200 (the one-cluster layout pulls four relations'
  // gathered rows through each of its 16 SMs)
  if (s->layout == BPC_STREAM_ONE_CLUSTER) {
    void* args[] = {&s->maps[0], &s->maps[1], &s->maps[2], &s->maps[3], &s->args};
    const int e = launch_one_cluster(s, args);
    if (e > 1) return e;
    if (e == 1)
      return fail(BPC_ERR_LAUNCH, "a cluster of " + std::to_string(s->nct) + " CTAs cannot be resident on this device");
    s->running_layout = BPC_STREAM_ONE_CLUSTER;
    return wait_ready(s);
  }
  if (int e = allow_smem(reinterpret_cast<const void*>(&stream_kernel), s->smem)) return e;
  void* args[] = {&s->maps[0], &s->maps[1], &s->maps[2], &s->maps[3], &s->maps[4], &s->args};
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
  s->running_layout = BPC_STREAM_CLUSTERS;
  return wait_ready(s);
}

namespace {

int wait_ready(bpc_stream* s) {
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

}  // namespace

extern "C" int bpc_stream_layout(const bpc_stream* s) { return s ? s->running_layout : -1; }

extern "C" int bpc_stream_trace(bpc_stream* s, int32_t on) {
  if (!s) return fail(BPC_ERR_ARG, "null stream");
  if (s->running) return fail(BPC_ERR_ARG, "tracing is set before start");
  s->tracing = on != 0;
  return 0;
}

extern "C" int bpc_stream_trace_read(const bpc_stream* s, uint64_t* out, int64_t n) {
  if (!s || !out) return fail(BPC_ERR_ARG, "null argument");
  if (s->running) return fail(BPC_ERR_ARG, "the trace is read after stop");
  const int64_t total = static_cast<int64_t>(kTraceCtas) * kTraceSlots * kTraceK;
  if (n < total) return fail(BPC_ERR_SPACE, "the trace holds " + std::to_string(total) + " values");
  if (cudaMemcpy(out, s->trace, sizeof(unsigned long long) * total, cudaMemcpyDeviceToHost) != cudaSuccess)
    return fail(BPC_ERR_LAUNCH, "cudaMemcpy of the trace failed");
  return 0;
}

extern "C" int bpc_stream_round(bpc_stream* s, const uint8_t* round_dets, uint8_t* residual, float* logits,
                                int64_t timeout_us) {
  if (!s || !round_dets) return fail(BPC_ERR_ARG, "null argument");
  if (!s->running) return fail(BPC_ERR_ARG, "the stream kernel is not running");
  if (s->desynced)
    return fail(BPC_ERR_DEVICE, "an earlier round timed out before its response; stop and start the stream again");
  const StreamArgs& a = s->args;
  const uint64_t tag = ++s->tag;
  write_request(s, round_dets, false);
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
  ++s->tag;
  write_request(s, nullptr, true);
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
