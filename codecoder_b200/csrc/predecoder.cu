// Pre-decoder forward: detector bits -> L x [check -> data, data -> check] bipartite convolutions -> X/Z head ->
// threshold -> XOR syndrome cancellation, on device buffers, with the caller's workspace.
//
// HBM layout of one chunk of S shots (S a multiple of 256; the workspace fixes S):
//   h_c   (N_c, S, C)  check features, node-major; on the tensor-core paths blocked by TM shots (TM = 128 for the
//                      CTA-pair steps at C = 128, 256 for the wide-tile steps): the TM shots of one node are TM x C
//                      contiguous, channel groups of 8 outermost within the block
//   h_d   (N_d, S, C)  data features, same layout
//   bits  (N_c, S/32)  uint32 residual syndrome, bit s % 32 of word s / 32 = shot s
// Per chunk: embed (det -> h_c, det -> bits), 2 L bipartite steps (the last check -> data step also writes the logits
// and XORs the predicted flips into bits), unpack (bits -> residual bytes).  Logits go straight to the caller's
// (B, N_d, 2) buffer from the head epilogue.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "bpc.h"
#include "bpc_common.cuh"
#include "bpc_internal.h"

struct bpc_predecoder {
  bpc_predecoder_config cfg;
  int device = 0;                // device current at create: tables, weights and status word live there
  int32_t* c2d = nullptr;        // (N_d, K)
  int32_t* d2c = nullptr;        // (N_c, K)
  int32_t* xor_nbr = nullptr;    // (N_d, 2, 2)
  uint8_t* check_type = nullptr; // (N_c)
  int32_t* check_order = nullptr; // (N_c) processing order of the data -> check steps, or null
  int32_t* check_order_typed = nullptr;  // (N_c) the same order grouped by check type (X checks first)
  void* embed = nullptr;         // (4, C)
  void* w_c2d = nullptr;         // (L, C, K C)
  void* w_d2c = nullptr;         // (L, 2, C, K C)
  float* head_w = nullptr;       // (2, C)
  float* head_b = nullptr;       // (2)
  int* status = nullptr;         // device watchdog status word
  unsigned long long* tile_counter = nullptr;   // dynamic tile scheduling of the tensor-core steps (2 words)
  bool weights_set = false;
  uint64_t timeout_ns = 2000000000ull;
  std::vector<cudaEvent_t> step_events;   // optional (before, after) pairs around each bipartite-step launch
};

namespace bpc {
namespace {

constexpr int kEmbShots = 128;
// Passes of at most this many shots run the node-tiled kernels (rows of the MMA = nodes), larger ones the
// shot-tiled kernels (rows = shots): below it a shot tile would be mostly empty.
constexpr int64_t kNodePathMaxShots = 64;
constexpr int kEmbNodes = 32;

size_t esize(int dtype) { return dtype == BPC_DTYPE_F32 ? 4 : 2; }
size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// det (rows of N_c bytes, shot-major) -> h_c features = embed[2 type(n) + det] and bits[n][s / 32].
// Feature element (shot s, node n, channel c) goes to n node_stride + (c / 8) cg_stride + s shot_stride + c % 8 (rows
// layouts, tm = 0) or, blocked with tile tm, to n node_stride + (s / tm) C tm + (c / 8) tm 8 + (s % tm) 8 + c % 8.
template <typename T>
__global__ void __launch_bounds__(256) embed_kernel(const uint8_t* __restrict__ det, int64_t shots, int N_c, int C,
                                                   const uint8_t* __restrict__ ctype, const T* __restrict__ embed,
                                                   T* __restrict__ hc, int64_t node_stride, int64_t cg_stride,
                                                   int64_t shot_stride, int tm, uint32_t* __restrict__ bits,
                                                   int64_t words) {
  __shared__ uint8_t tile[kEmbNodes][kEmbShots + 4];
  __shared__ __align__(16) T emb[4 * 256];
  __shared__ uint8_t types[kEmbNodes];
  const int64_t s0 = static_cast<int64_t>(blockIdx.x) * kEmbShots;
  const int n0 = blockIdx.y * kEmbNodes;
  pdl_launch_dependents();
  for (int e = threadIdx.x; e < 4 * C; e += blockDim.x) emb[e] = embed[e];
  if (threadIdx.x < kEmbNodes) types[threadIdx.x] = n0 + threadIdx.x < N_c ? ctype[n0 + threadIdx.x] : 0;
  pdl_wait();                               // det, and the buffers earlier kernels still read, are shared
  for (int e = threadIdx.x; e < kEmbNodes * kEmbShots; e += blockDim.x) {
    const int s = e / kEmbNodes, j = e - s * kEmbNodes;
    const int64_t shot = s0 + s;
    const int n = n0 + j;
    tile[j][s] = (shot < shots && n < N_c) ? (det[shot * N_c + n] & 1) : 0;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // bit-packed residual initialised with the detectors
  for (int j = warp; j < kEmbNodes; j += blockDim.x / 32) {
    const int n = n0 + j;
    if (n >= N_c) break;
    for (int w = 0; w < kEmbShots / 32; ++w) {
      const uint32_t m = __ballot_sync(0xffffffffu, tile[j][w * 32 + lane] != 0);
      const int64_t word = (s0 >> 5) + w;
      if (lane == 0 && word < words) bits[static_cast<int64_t>(n) * words + word] = m;
    }
  }
  // features in 8-element groups (16 bytes of bf16, 32 of fp32: two 16-byte vectors): one warp per (node, group),
  // lanes over the shots (contiguous in the chunked layout); a block's shots lie in one tile of the chunked layout
  // (kEmbShots divides tm), so the tile offset is computed once
  constexpr int kVec = 16 / sizeof(T);
  const int groups = C / 8;
  const int smax = static_cast<int>((shots - s0) < kEmbShots ? (shots - s0) : kEmbShots);
  const int64_t tile_off = tm ? (s0 / tm) * C * static_cast<int64_t>(tm) : 0;
  const int s_in_tile = tm ? static_cast<int>(s0 % tm) : 0;
  for (int jg = warp; jg < kEmbNodes * groups; jg += blockDim.x / 32) {
    const int j = jg / groups, g = jg - j * groups;
    const int n = n0 + j;
    if (n >= N_c) break;
    T* base = hc + static_cast<int64_t>(n) * node_stride;
    T* gbase = tm ? base + tile_off + static_cast<int64_t>(g) * tm * 8 + static_cast<int64_t>(s_in_tile) * 8
                  : base + g * cg_stride + s0 * shot_stride;
    const int64_t sstep = tm ? 8 : shot_stride;
    for (int s = lane; s < smax; s += 32) {
      const int tok = 2 * types[j] + tile[j][s];
      const uint4* src = reinterpret_cast<const uint4*>(emb + tok * C + g * 8);
      T* dst = gbase + s * sstep;
#pragma unroll
      for (int v = 0; v < 8 / kVec; ++v) reinterpret_cast<uint4*>(dst)[v] = src[v];
    }
  }
}

// bits[n][s / 32] -> residual[shot][n] bytes
__global__ void __launch_bounds__(256) unpack_kernel(const uint32_t* __restrict__ bits, int64_t words, int64_t shots,
                                                    int N_c, uint8_t* __restrict__ out) {
  __shared__ uint32_t w[kEmbNodes][kEmbShots / 32];
  const int64_t s0 = static_cast<int64_t>(blockIdx.x) * kEmbShots;
  const int n0 = blockIdx.y * kEmbNodes;
  pdl_launch_dependents();
  pdl_wait();
  for (int e = threadIdx.x; e < kEmbNodes * (kEmbShots / 32); e += blockDim.x) {
    const int j = e / (kEmbShots / 32), k = e - j * (kEmbShots / 32);
    const int64_t word = (s0 >> 5) + k;
    w[j][k] = (n0 + j < N_c && word < words) ? bits[static_cast<int64_t>(n0 + j) * words + word] : 0u;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < kEmbShots * kEmbNodes; e += blockDim.x) {
    const int s = e / kEmbNodes, j = e - s * kEmbNodes;
    const int64_t shot = s0 + s;
    if (shot < shots && n0 + j < N_c) out[shot * N_c + n0 + j] = static_cast<uint8_t>((w[j][s >> 5] >> (s & 31)) & 1u);
  }
}

struct Layout {
  int64_t S;
  size_t off_hc, off_hd, off_bits, total;
};

// Shot capacity S of a pass: a multiple of 256, the tensor-core kernel's tile in the chunked layout.
Layout layout_for(const bpc_predecoder_config& c, int64_t chunk) {
  Layout L;
  L.S = ((chunk + 255) / 256) * 256;
  const size_t es = esize(c.dtype);
  L.off_hc = 0;
  L.off_hd = align256(L.off_hc + static_cast<size_t>(c.n_checks) * L.S * c.channels * es);
  L.off_bits = align256(L.off_hd + static_cast<size_t>(c.n_data) * L.S * c.channels * es);
  L.total = align256(L.off_bits + static_cast<size_t>(c.n_checks) * (L.S / 32) * 4);
  return L;
}

template <typename T>
int copy_in(T** dst, const void* src, size_t bytes) {
  if (*dst == nullptr) {
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(dst), bytes);
    if (e != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("cudaMalloc: ") + cudaGetErrorString(e));
  }
  cudaError_t e = cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("cudaMemcpy: ") + cudaGetErrorString(e));
  return 0;
}

}  // namespace
}  // namespace bpc

using namespace bpc;

extern "C" int bpc_predecoder_create(const bpc_predecoder_config* cfg, const int32_t* c2d, const int32_t* d2c,
                                     const int32_t* xor_nbr, const uint8_t* check_type, const int32_t* check_order,
                                     bpc_predecoder** out) {
  if (!cfg || !c2d || !d2c || !xor_nbr || !check_type || !out) return fail(BPC_ERR_ARG, "null argument");
  *out = nullptr;
  const auto& c = *cfg;
  if (c.layers < 1 || c.channels < 8 || c.channels > 256 || c.channels % 8 || c.K < 1 || c.K > 32 ||
      c.n_checks < 1 || c.n_data < 1 || c.z_check_begin < 0 || c.z_check_begin > c.n_checks ||
      (c.dtype != BPC_DTYPE_BF16 && c.dtype != BPC_DTYPE_F32))
    return fail(BPC_ERR_ARG, "invalid pre-decoder configuration");
  auto* h = new bpc_predecoder();
  h->cfg = c;
  if (cudaGetDevice(&h->device) != cudaSuccess) {
    delete h;
    return fail(BPC_ERR_LAUNCH, "cudaGetDevice failed");
  }
  int e = 0;
  if ((e = copy_in(&h->c2d, c2d, sizeof(int32_t) * c.n_data * c.K)) ||
      (e = copy_in(&h->d2c, d2c, sizeof(int32_t) * c.n_checks * c.K)) ||
      (e = copy_in(&h->xor_nbr, xor_nbr, sizeof(int32_t) * c.n_data * 4)) ||
      (e = copy_in(&h->check_type, check_type, c.n_checks))) {
    bpc_predecoder_destroy(h);
    return e;
  }
  if (check_order) {
    std::vector<char> seen(c.n_checks, 0);
    for (int i = 0; i < c.n_checks; ++i) {
      if (check_order[i] < 0 || check_order[i] >= c.n_checks || seen[check_order[i]]) {
        bpc_predecoder_destroy(h);
        return fail(BPC_ERR_ARG, "check_order is not a permutation of the check nodes");
      }
      seen[check_order[i]] = 1;
    }
    if ((e = copy_in(&h->check_order, check_order, sizeof(int32_t) * c.n_checks))) {
      bpc_predecoder_destroy(h);
      return e;
    }
  }
  {
    // the data -> check order grouped by type (the CTA-pair steps give each check type its own pairs)
    std::vector<int32_t> typed;
    typed.reserve(c.n_checks);
    for (int ty = 0; ty < 2; ++ty)
      for (int i = 0; i < c.n_checks; ++i) {
        const int n = check_order ? check_order[i] : i;
        if ((n >= c.z_check_begin) == (ty == 1)) typed.push_back(n);
      }
    if ((e = copy_in(&h->check_order_typed, typed.data(), sizeof(int32_t) * c.n_checks))) {
      bpc_predecoder_destroy(h);
      return e;
    }
  }
  const unsigned long long zero64[2] = {0, 0};
  if ((e = copy_in(&h->tile_counter, zero64, sizeof(zero64)))) {
    bpc_predecoder_destroy(h);
    return e;
  }
  int zero = 0;
  if ((e = copy_in(&h->status, &zero, sizeof(int)))) {
    bpc_predecoder_destroy(h);
    return e;
  }
  *out = h;
  return 0;
}

extern "C" int bpc_predecoder_set_weights(bpc_predecoder* h, const void* embed, const void* w_c2d, const void* w_d2c,
                                          const float* head_w, const float* head_b) {
  if (!h || !embed || !w_c2d || !w_d2c || !head_w || !head_b) return fail(BPC_ERR_ARG, "null argument");
  const auto& c = h->cfg;
  const size_t es = esize(c.dtype);
  const size_t wl = static_cast<size_t>(c.channels) * c.K * c.channels;
  int e = 0;
  if ((e = copy_in(&h->embed, embed, 4 * c.channels * es)) ||
      (e = copy_in(&h->w_c2d, w_c2d, c.layers * wl * es)) ||
      (e = copy_in(&h->w_d2c, w_d2c, 2 * c.layers * wl * es)) ||
      (e = copy_in(&h->head_w, head_w, 2 * c.channels * sizeof(float))) ||
      (e = copy_in(&h->head_b, head_b, 2 * sizeof(float))))
    return e;
  h->weights_set = true;
  return 0;
}

extern "C" size_t bpc_predecoder_workspace_size(const bpc_predecoder* h, int64_t chunk_shots) {
  if (!h || chunk_shots < 1) return 0;
  return layout_for(h->cfg, chunk_shots).total;
}

extern "C" int bpc_predecoder_forward(bpc_predecoder* h, const uint8_t* det, float* logits, uint8_t* residual,
                                      int64_t B, void* workspace, size_t workspace_bytes, bpc_stream_t stream_) {
  if (!h || !h->weights_set) return fail(BPC_ERR_ARG, "pre-decoder without weights");
  if (B < 0) return fail(BPC_ERR_ARG, "negative batch");
  if (B == 0) return 0;
  if (!det || !logits || !residual || !workspace) return fail(BPC_ERR_ARG, "null buffer");
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return fail(BPC_ERR_ARG, "workspace must be 256-byte aligned");
  if (reinterpret_cast<uintptr_t>(logits) & 7) return fail(BPC_ERR_ARG, "logits must be 8-byte aligned");
  const auto& c = h->cfg;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  // largest chunk (multiple of 128 shots, at most B rounded up) whose layout fits the workspace
  int64_t chunk = ((B + 255) / 256) * 256;
  const size_t per256 = layout_for(c, 256).total;
  if (workspace_bytes < per256) return fail(BPC_ERR_SPACE, "workspace smaller than one 256-shot pass");
  while (chunk > 256 && layout_for(c, chunk).total > workspace_bytes) {
    const int64_t fit = static_cast<int64_t>(workspace_bytes / per256) * 256;
    chunk = std::max<int64_t>(256, std::min(chunk - 256, fit));
  }
  const Layout L = layout_for(c, chunk);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* hc = ws + L.off_hc;
  void* hd = ws + L.off_hd;
  uint32_t* bits = reinterpret_cast<uint32_t*>(ws + L.off_bits);
  const int64_t words = L.S / 32;
  const bool f32 = c.dtype == BPC_DTYPE_F32;
  const bool tc = !f32 && c.channels >= 64 && c.channels % 32 == 0;
  const bool nodes = tc && B <= kNodePathMaxShots && (c.channels == 64 || c.channels == 128);
  const bool shot_tiles = tc && !nodes;
  // hidden-128 steps: the single-CTA wide-tile kernel; BPC_STEP_KERNEL=pair selects the CTA-pair kernel with resident
  // relation matrices (same bits; measured slower on B200: half of its shared memory holds W, so half as many
  // activation bytes are in flight and the loads' latency is not covered)
  // activation bytes are in flight and the loads' latency is not covered); BPC_STEP_KERNEL=pair_stream selects the
  // CTA-pair kernel with the W halves streamed alongside two 128-shot blocks per CTA
  const char* sk = std::getenv("BPC_STEP_KERNEL");
  const bool pair_stream = sk && std::strcmp(sk, "pair_stream") == 0;
  const bool pair = shot_tiles && c.channels == 128 && c.K <= 8 && sk && (std::strcmp(sk, "pair") == 0 || pair_stream);
  const size_t es = esize(c.dtype);
  const size_t wl = static_cast<size_t>(c.channels) * c.K * c.channels;

  // the two steps of layer l as bipartite-conv problems on the chunk's buffers
  // shot-tiled tensor-core path: blocked (node, S / TM, C / 8, TM, 8) activations; node-tiled tensor-core and
  // CUDA-core paths: node-major rows (node, S, C)
  const int tm = pair ? gmm_pair_tile_shots() : shot_tiles ? gmm_tc_tile_shots(c.channels) : 0;
  const int64_t shot_stride = c.channels;
  const int64_t cg_stride = 8;
  const int64_t node_stride = L.S * c.channels;
  if (shot_tiles && L.S % tm != 0) return fail(BPC_ERR_ARG, "pass size is not a multiple of the tensor-core tile");
  if (tm % kEmbShots != 0) return fail(BPC_ERR_ARG, "the embedding's shot block must divide the tensor-core tile");
  GmmProblem c2d, d2c;
  c2d.x = hc;
  c2d.blocked = shot_tiles;
  c2d.x_shot_stride = shot_stride;
  c2d.x_node_stride = node_stride;
  c2d.x_cg_stride = cg_stride;
  c2d.NS = c.n_checks;
  c2d.idx = h->c2d;
  c2d.NT = c.n_data;
  c2d.K = c.K;
  c2d.Ci = c2d.Co = c.channels;
  c2d.y = hd;
  c2d.y_shot_stride = shot_stride;
  c2d.y_node_stride = node_stride;
  c2d.y_cg_stride = cg_stride;
  c2d.n_wtypes = 1;
  c2d.type_split = c.n_data;
  d2c = c2d;
  d2c.x = hd;
  d2c.NS = c.n_data;
  d2c.idx = h->d2c;
  d2c.NT = c.n_checks;
  d2c.y = hc;
  d2c.n_wtypes = 2;
  d2c.type_split = c.z_check_begin;
  d2c.order = h->check_order;
  d2c.epi = kEpiGeluResid;

  GmmMaps mc2d, md2c;
  std::vector<CUtensorMap> wm_c2d, wm_d2c;
  if (shot_tiles) {
    c2d.shots = d2c.shots = L.S;
    c2d.w = h->w_c2d;
    d2c.w = h->w_d2c;
    auto make = [&](const GmmProblem& q, GmmMaps* m) { return pair ? gmm_pair_make_maps(q, m) : gmm_tc_make_maps(q, m); };
    if (int e = make(c2d, &mc2d)) return e;
    if (int e = make(d2c, &md2c)) return e;
    for (int l = 0; l < c.layers; ++l) {
      GmmMaps tmp;
      c2d.w = static_cast<const uint8_t*>(h->w_c2d) + l * wl * es;
      d2c.w = static_cast<const uint8_t*>(h->w_d2c) + 2 * l * wl * es;
      if (int e = make(c2d, &tmp)) return e;
      wm_c2d.push_back(tmp.w);
      if (int e = make(d2c, &tmp)) return e;
      wm_d2c.push_back(tmp.w);
    }
  }

  size_t n_rec = 0;
  for (int64_t b0 = 0; b0 < B; b0 += L.S) {
    const int64_t Sb = std::min<int64_t>(L.S, B - b0);
    {
      dim3 grid(static_cast<unsigned>((Sb + kEmbShots - 1) / kEmbShots),
                static_cast<unsigned>((c.n_checks + kEmbNodes - 1) / kEmbNodes));
      const uint8_t* det_b = det + b0 * c.n_checks;
      int Nc = c.n_checks, Cc = c.channels;
      int tm_i = tm;
      int64_t Sb_i = Sb, ns = node_stride, cgs = cg_stride, ss = shot_stride, wd = words;
      const uint8_t* ct = h->check_type;
      const void* emb = h->embed;
      void* hcp = hc;
      uint32_t* bp = bits;
      void* eargs[] = {&det_b, &Sb_i, &Nc, &Cc, &ct, &emb, &hcp, &ns, &cgs, &ss, &tm_i, &bp, &wd};
      const void* efn = f32 ? reinterpret_cast<const void*>(&embed_kernel<float>)
                            : reinterpret_cast<const void*>(&embed_kernel<__nv_bfloat16>);
      if (nodes) {
        if (int e = launch_pdl(efn, grid, dim3(256), 0, stream, eargs, 1, "embed_kernel")) return e;
      } else if (cudaLaunchKernel(efn, grid, dim3(256), eargs, 0, stream) != cudaSuccess) {
        return fail(BPC_ERR_LAUNCH, std::string("embed_kernel: ") + cudaGetErrorString(cudaGetLastError()));
      }
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("embed_kernel: ") + cudaGetErrorString(e));
    }
    c2d.shots = d2c.shots = Sb;
    for (int l = 0; l < c.layers; ++l) {
      c2d.w = static_cast<const uint8_t*>(h->w_c2d) + l * wl * es;
      d2c.w = static_cast<const uint8_t*>(h->w_d2c) + 2 * l * wl * es;
      c2d.epi = l == 0 ? kEpiGeluInit : kEpiGeluResid;
      c2d.head = HeadEpilogue();
      if (l == c.layers - 1) {
        c2d.head.head_w = h->head_w;
        c2d.head.head_b = h->head_b;
        c2d.head.logits = logits + b0 * c.n_data * 2;
        c2d.head.lg_shot_stride = static_cast<int64_t>(c.n_data) * 2;
        c2d.head.lg_node_stride = 2;
        c2d.head.res_bits = bits;
        c2d.head.res_words = words;
        c2d.head.xor_nbr = h->xor_nbr;
      }
      for (int step = 0; step < 2; ++step) {
        const GmmProblem& p = step == 0 ? c2d : d2c;
        const bool rec = 2 * n_rec + 1 < h->step_events.size();
        if (shot_tiles && !pair) {   // the tile counter of the dynamic scheduler starts at zero
          cudaError_t me = cudaMemsetAsync(h->tile_counter, 0, sizeof(unsigned long long), stream);
          if (me != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("cudaMemsetAsync: ") + cudaGetErrorString(me));
        }
        if (rec) cudaEventRecord(h->step_events[2 * n_rec], stream);
        int e;
        if (nodes) {
          e = gmm_nodes_launch(p, h->status, h->timeout_ns, stream);
        } else if (pair) {
          GmmMaps m = step == 0 ? mc2d : md2c;
          m.w = step == 0 ? wm_c2d[l] : wm_d2c[l];
          e = gmm_pair_launch(p, m, step == 0 ? nullptr : h->check_order_typed, c.z_check_begin, h->tile_counter,
                              h->status, h->timeout_ns, stream, pair_stream);
        } else if (tc) {
          GmmMaps m = step == 0 ? mc2d : md2c;
          m.w = step == 0 ? wm_c2d[l] : wm_d2c[l];
          GmmProblem pc = p;
          pc.tile_counter = h->tile_counter;
          e = gmm_tc_launch(pc, m, h->status, h->timeout_ns, stream);
        } else {
          e = gmm_fma_launch(p, f32, stream);
        }
        if (e) return e;
        if (rec) cudaEventRecord(h->step_events[2 * n_rec + 1], stream);
        n_rec += rec;
      }
    }
    {
      dim3 grid(static_cast<unsigned>((Sb + kEmbShots - 1) / kEmbShots),
                static_cast<unsigned>((c.n_checks + kEmbNodes - 1) / kEmbNodes));
      const uint32_t* bp = bits;
      int64_t wd = words, Sb_i = Sb;
      int Nc = c.n_checks;
      uint8_t* outp = residual + b0 * c.n_checks;
      void* uargs[] = {&bp, &wd, &Sb_i, &Nc, &outp};
      if (nodes) {
        if (int e = launch_pdl(reinterpret_cast<const void*>(&unpack_kernel), grid, dim3(256), 0, stream, uargs, 1,
                               "unpack_kernel"))
          return e;
      } else {
        unpack_kernel<<<grid, 256, 0, stream>>>(bits, words, Sb, c.n_checks, residual + b0 * c.n_checks);
      }
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("unpack_kernel: ") + cudaGetErrorString(e));
    }
  }
  return 0;
}

namespace bpc {
int predecoder_internals(const bpc_predecoder* h, bpc_predecoder_config* cfg, const void** embed, const void** w_c2d,
                         const void** w_d2c, const float** head_w, const float** head_b, const int32_t** c2d,
                         const int32_t** d2c, const int32_t** xor_nbr) {
  if (!h) return fail(BPC_ERR_ARG, "null pre-decoder");
  if (!h->weights_set) return fail(BPC_ERR_ARG, "pre-decoder without weights");
  *cfg = h->cfg;
  *embed = h->embed;
  *w_c2d = h->w_c2d;
  *w_d2c = h->w_d2c;
  *head_w = h->head_w;
  *head_b = h->head_b;
  *c2d = h->c2d;
  *d2c = h->d2c;
  *xor_nbr = h->xor_nbr;
  return 0;
}
}  // namespace bpc

namespace bpc {
int predecoder_device(const bpc_predecoder* h) { return h ? h->device : -1; }
}  // namespace bpc

extern "C" int bpc_predecoder_record_step_events(bpc_predecoder* h, void* const* events, int n_pairs) {
  if (!h || n_pairs < 0 || (n_pairs > 0 && !events)) return fail(BPC_ERR_ARG, "invalid event list");
  h->step_events.assign(reinterpret_cast<cudaEvent_t const*>(events),
                        reinterpret_cast<cudaEvent_t const*>(events) + 2 * static_cast<size_t>(n_pairs));
  return 0;
}

extern "C" int bpc_predecoder_status(bpc_predecoder* h, bpc_stream_t stream, int* status) {
  if (!h || !status) return fail(BPC_ERR_ARG, "null argument");
  int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, h->status, sizeof(int), cudaMemcpyDeviceToHost,
                                  reinterpret_cast<cudaStream_t>(stream));
  if (e == cudaSuccess) e = cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(BPC_ERR_LAUNCH, std::string("status read: ") + cudaGetErrorString(e));
  *status = v;
  if (v != 0) {
    const int zero = 0;
    cudaMemcpy(h->status, &zero, sizeof(int), cudaMemcpyHostToDevice);
    return fail(BPC_ERR_DEVICE, "a kernel watchdog fired (status " + std::to_string(v) + ")");
  }
  return 0;
}

extern "C" void bpc_predecoder_destroy(bpc_predecoder* h) {
  if (!h) return;
  for (void* p : {static_cast<void*>(h->c2d), static_cast<void*>(h->d2c), static_cast<void*>(h->xor_nbr),
                  static_cast<void*>(h->check_order), static_cast<void*>(h->check_order_typed),
                  static_cast<void*>(h->check_type), h->embed, h->w_c2d, h->w_d2c, static_cast<void*>(h->head_w),
                  static_cast<void*>(h->head_b), static_cast<void*>(h->status), static_cast<void*>(h->tile_counter)})
    if (p) cudaFree(p);
  delete h;
}
