// Device helpers shared by the bipartite-conv kernels: mbarriers with bounded waits, TMA tensor loads,
// tcgen05 (TMEM allocation, MMA, commit, loads) and the shared-memory matrix descriptors, all as inline PTX for sm_100a.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace bpc {

// Device status word values (written with atomicExch into the caller-visible status buffer).
enum : int {
  kStatusOk = 0,
  kStatusTimeout = 1,  // an mbarrier wait gave up after the watchdog limit
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------------------------------------------
// Programmatic dependent launch: a kernel launched with programmatic stream serialization may start while the
// previous kernel of the stream still runs.  pdl_launch_dependents lets the next kernel start; pdl_wait blocks the
// calling thread until the previous kernel has completed and its memory is visible (a no-op without the launch
// attribute).  Everything before pdl_wait may touch only shared memory, tensor memory and inputs no kernel of the
// stream writes.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---------------------------------------------------------------------------------------------------------------
// mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   bar),
               "r"(bytes)
               : "memory");
}
// Add `bytes` to the transaction count of the current phase without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase of `parity` to complete.  Gives up after `timeout_ns` of wall time (or when another role of
// the CTA already gave up, *abort != 0), records kStatusTimeout in *status and returns false.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort, int* status,
                                          uint64_t timeout_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (globaltimer_ns() - t0 > timeout_ns) {
      *abort = 1;
      if (status) atomicExch(status, kStatusTimeout);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// TMA: tiled 3D tensor load into this CTA's shared memory, completion counted in bytes on an mbarrier.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int32_t c0, int32_t c1, int32_t c2,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------------------------------------------
// tcgen05: tensor memory and the 5th-generation MMA
__device__ __forceinline__ void tmem_alloc(uint32_t slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 or f16 inputs, fp32 accumulate), issued by one thread.
__device__ __forceinline__ void tc_mma_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on an mbarrier of this CTA when every tcgen05 operation issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane (base + i), columns col .. col + 31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// TMA gather of 4 rows (row indices r0..r3, channels c0 .. c0 + 63 of a 2D tensor map with a one-row box) into 512
// consecutive bytes of shared memory, in the map's swizzled layout; completion counted in bytes on `bar`.
__device__ __forceinline__ void tma_gather4(uint32_t dst, const CUtensorMap* map, int32_t c0, int32_t r0, int32_t r1,
                                            int32_t r2, int32_t r3, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// ---------------------------------------------------------------------------------------------------------------
// Thread-block clusters: rank, barrier halves, distributed shared memory
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_to_cta(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// bulk copy of `bytes` (a multiple of 16) from this CTA's shared memory to another CTA's of the cluster, the bytes
// counted on an mbarrier of the destination CTA
__device__ __forceinline__ void bulk_s2cluster(uint32_t dst_cluster, uint32_t src, uint32_t bytes,
                                               uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst_cluster),
      "r"(src), "r"(bytes), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until the bulk copies this thread issued have finished reading their source
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Wait until every committed bulk group of this thread has completed (its global writes done).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// TMA: tiled 2D store of a box from this CTA's shared memory (bulk group completion; rows past the map are dropped).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int32_t c0, int32_t c1, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(src)
               : "memory");
}
// acquire side of the remote arrivals (cluster scope): a bounded wait like mbar_wait
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// ---------------------------------------------------------------------------------------------------------------
// CTA pairs (cta_group::2): one MMA spans the tensor cores of two CTAs of a cluster.  A is split by rows (M / 2
// rows in each CTA's shared memory, at the same offset), B by columns (N / 2 rows of the K-major B in each CTA), and
// each CTA's tensor memory holds its M / 2 rows of D.  One thread of the even CTA issues the MMA.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_mma_ss_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the mbarrier at offset `bar` of every CTA in `cta_mask` when the pair MMAs issued so far by this
// thread have completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(cta_mask)
      : "memory");
}
// TMA: tiled 2D load into this CTA's shared memory, bytes counted on an mbarrier of this CTA.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int32_t c0, int32_t c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}
// The same load into this CTA's shared memory with the bytes counted on an mbarrier of the pair's even CTA
// (`bar_cluster`: a shared::cluster address from map_to_cta).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int32_t c0, int32_t c1,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar_cluster)
      : "memory");
}
// The 3D form of tma_load_2d_pair.
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, int32_t c0, int32_t c1,
                                                 int32_t c2, uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
      "%4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar_cluster)
      : "memory");
}
// Arrive on an mbarrier of another CTA of the cluster (release at cluster scope: this thread's earlier writes,
// shared::cluster stores included, are visible to a cluster-scope acquire that sees the phase complete).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
__device__ __forceinline__ void st_cluster_u32(uint32_t addr_cluster, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr_cluster), "r"(v) : "memory");
}
// Bounded wait with cluster-scope acquire (for barriers that receive arrivals from the other CTA of a pair).  On a
// timeout or an abort it records the status and returns false, like mbar_wait.
__device__ __forceinline__ bool mbar_wait_cl(uint32_t bar, uint32_t parity, volatile int* abort, int* status,
                                             uint64_t timeout_ns) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (*abort) return false;
    if (globaltimer_ns() - t0 > timeout_ns) {
      *abort = 1;
      if (status) atomicExch(status, kStatusTimeout);
      return false;
    }
  }
}

// byte offset of float4 chunk c (channels 4c .. 4c + 3) of row m (0..15) in receive slot r: rows of 16 chunks,
// XOR-swizzled by row
__device__ __forceinline__ uint32_t recv_off(int r, int m, int c) {
  return static_cast<uint32_t>(r * (16 * 256) + m * 256 + ((c ^ (m & 15)) << 4));
}

// Shared-memory matrix descriptor of a K-major operand stored in the 128-byte swizzled canonical layout: rows of
// 64 bf16 (128 B), 8-row groups 1024 B apart.  Fields: start address >> 4 (bits 0-13), leading byte offset >> 4
// (16-29, unused for this layout: 1), stride byte offset >> 4 (32-45), descriptor version 1 (46-47), swizzle mode
// 2 = 128 B (61-63).
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}
// Descriptor of a K-major operand in the canonical layout without swizzle: 8-row x 16-byte core matrices stored as
// 128 contiguous bytes, core matrices adjacent in M `sbo` bytes apart and adjacent in K `lbo` bytes apart.
__device__ __forceinline__ uint64_t sdesc_k_none(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  return d;
}
// Descriptor of an MN-major operand (the M or N index contiguous) in the 128-byte swizzled canonical layout, as a
// TMA box of rows of 64 bf16 with SWIZZLE_128B writes it: each 128-byte row holds 64 consecutive M (or N) elements
// at one K index, K rows 128 bytes apart, 8-row groups (K) `sbo` bytes apart, 64-element M/N groups `lbo` bytes apart.
__device__ __forceinline__ uint64_t sdesc_mn_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}
// 1D bulk copy global -> this CTA's shared memory (both 16-byte aligned, size a multiple of 16), counted on an
// mbarrier in bytes.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
               : "memory");
}

// Instruction descriptor for kind::f16: fp32 accumulator (bits 4-5 = 1), A and B bf16 (bits 7-9, 10-12 = 1),
// both K-major (bits 15, 16 = 0), N >> 3 in bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}
// The same with A and B MN-major (bits 15 and 16 set): A (M x K) stored M-contiguous, B (N x K) N-contiguous.
__host__ __device__ constexpr uint32_t idesc_bf16_f32_mn(int M, int N) {
  return idesc_bf16_f32(M, N) | (1u << 15) | (1u << 16);
}

// GELU in its tanh form (Hendrycks & Gimpel 2016): 0.5 x (1 + tanh(sqrt(2 / pi) (x + 0.044715 x^3))).
// gelu_tanh: CUDA's tanhf (fp32 networks).  gelu_tanh_fast: the hardware tanh.approx.f32 (one MUFU op, relative
// error about 2^-11), used where the result is rounded to bf16 (relative step 2^-8) right after.
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Packed fp32 pairs (two lanes of one 64-bit register) for the sm_100 f32x2 FMA-pipe instructions.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  return static_cast<uint64_t>(__float_as_uint(lo)) | (static_cast<uint64_t>(__float_as_uint(hi)) << 32);
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// bf16 pair (low half = first element) <-> packed fp32 pair
__device__ __forceinline__ uint64_t bf2_to_f2(uint32_t h) { return f2_pack(__uint_as_float(h << 16), __uint_as_float(h & 0xFFFF0000u)); }
__device__ __forceinline__ uint32_t f2_to_bf2(uint64_t v) {
  const __nv_bfloat162 b = __floats2bfloat162_rn(f2_lo(v), f2_hi(v));
  return *reinterpret_cast<const uint32_t*>(&b);
}
// GELU (tanh form) of a packed pair: u = x (c1 + c2 x^2), 0.5 x (1 + tanh(u)), tanh on the MUFU unit.
__device__ __forceinline__ uint64_t gelu_tanh_fast2(uint64_t x) {
  const uint64_t kC1 = f2_pack(0.7978845608028654f, 0.7978845608028654f);
  const uint64_t kC2 = f2_pack(0.7978845608028654f * 0.044715f, 0.7978845608028654f * 0.044715f);
  const uint64_t kHalf = f2_pack(0.5f, 0.5f);
  const uint64_t u = f2_mul(f2_fma(f2_mul(x, x), kC2, kC1), x);
  const uint64_t t = f2_pack(tanh_approx(f2_lo(u)), tanh_approx(f2_hi(u)));
  const uint64_t hx = f2_mul(x, kHalf);
  return f2_fma(hx, t, hx);
}

// SiLU of a packed pair: x sigmoid(x) = h + h tanh(h) with h = x / 2, tanh on the MUFU unit (used where the result
// is rounded to bf16 right after).
__device__ __forceinline__ uint64_t silu_tanh_fast2(uint64_t x) {
  const uint64_t kHalf = f2_pack(0.5f, 0.5f);
  const uint64_t h = f2_mul(x, kHalf);
  const uint64_t t = f2_pack(tanh_approx(f2_lo(h)), tanh_approx(f2_hi(h)));
  return f2_fma(h, t, h);
}
// SiLU with CUDA's expf (fp32 networks)
__device__ __forceinline__ float silu_exact(float x) { return x / (1.0f + expf(-x)); }

// GELU (tanh form) as the training network's residual steps compute it before rounding to bf16:
// t = tanh.approx(k (x + c x^3)), x (1 + t) / 2, k = sqrt(2 / pi), c = 0.044715 (one definition for the memory-bound
// passes and the step kernel's fused epilogue, so both give the same bits).
__device__ __forceinline__ float gelu_tanh_pass(float x) {
  const float t = tanh_approx(0.7978845608028654f * fmaf(0.044715f * x, x * x, x));
  return 0.5f * x * (1.0f + t);
}

__device__ __forceinline__ float gelu_tanh(float x) {
  const float u = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
  return 0.5f * x * (1.0f + tanhf(u));
}
__device__ __forceinline__ float gelu_tanh_fast(float x) {
  const float u = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
  const float hx = 0.5f * x;
  return fmaf(hx, tanh_approx(u), hx);
}

}  // namespace bpc
