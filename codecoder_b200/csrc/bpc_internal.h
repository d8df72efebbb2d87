// Internal launch interface of the bipartite-conv kernels (host side, shared by the C ABI and the pre-decoder).
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include "bpc.h"

namespace bpc {

enum EpiMode : int {
  kEpiStore = 0,      // y = acc
  kEpiGeluInit = 1,   // y = GELU(acc)
  kEpiGeluResid = 2,  // y = y + GELU(acc)
  kEpiAffineSilu = 3, // y = SiLU(scale[c] acc + shift[c])  (an inference BatchNorm folded into scale / shift)
  kEpiAdd = 4,        // y = y + acc  (row layouts: accumulate a second input gradient onto the first)
  kEpiGeluStream = 5, // y = acc (bf16, kept), and the residual stream: out = h + bf16(GELU(y)) (h fp32 -> out fp32 and
                      // its bf16 copy out16; h bf16 -> out bf16; no h -> out = bf16(GELU(y)))  (row layouts)
};

// Optional work fused into the epilogue of the last check -> data step of the pre-decoder.
struct HeadEpilogue {
  const float* head_w = nullptr;   // (2, Co) fp32, null = no head
  const float* head_b = nullptr;   // (2,)
  float* logits = nullptr;         // logits[shot * lg_shot_stride + node * lg_node_stride + j], j = 0 X, 1 Z
  int64_t lg_shot_stride = 0, lg_node_stride = 0;
  uint32_t* res_bits = nullptr;    // residual bits (checks, res_words), bit s % 32 of word s / 32 = shot s
  int64_t res_words = 0;
  const int32_t* xor_nbr = nullptr;  // (NT, 2, 2) checks flipped by a predicted X / Z flip, -1 = none
};

// y[s, n, :] (op)= sum_r x[s, idx[n, r], :] W_{type(n), r}^T over relations r whose source is in [0, NS).
// Two layouts for x and y (strides in elements, channels in groups of 8 = 16 bytes of bf16):
//   rows     channel c of shot s at node n is at n node_stride + (c / 8) cg_stride + s shot_stride + c % 8
//            (cg_stride = 8: a shot's channels contiguous; shot-major (B, N, C) or node-major (N, B, C))
//   blocked  the tensor-core pre-decoder layout (node, shots / TM, C / 8, TM, 8), TM = gmm_tc_tile_shots(Co):
//            element (s, n, c) at n node_stride + (s / TM) C TM + (c / 8) TM 8 + (s % TM) 8 + c % 8, so one tile
//            (TM shots of one node) is one contiguous block of C TM elements; node_stride = C x shot capacity.
// W holds n_wtypes stacked (Co, K Ci) matrices; target n uses set (n >= type_split).  `order`, if set, is the
// processing order of the targets (a permutation of 0 .. NT - 1).
struct GmmProblem {
  const void* x = nullptr;
  int64_t x_shot_stride = 0, x_node_stride = 0, x_cg_stride = 8;
  bool blocked = false;
  const int32_t* order = nullptr;
  int64_t shots = 0;
  int NS = 0;
  const void* w = nullptr;
  int n_wtypes = 1, type_split = 0;
  const int32_t* idx = nullptr;
  int NT = 0, K = 0, Ci = 0, Co = 0;
  void* y = nullptr;
  int64_t y_shot_stride = 0, y_node_stride = 0, y_cg_stride = 8;
  int epi = kEpiStore;
  const float* epi_scale = nullptr;   // kEpiAffineSilu: per output channel (Co,) fp32
  const float* epi_shift = nullptr;
  HeadEpilogue head;
  // kEpiGeluStream: the residual stream rows of the targets (channel c of shot s at node n: s res_shot_stride +
  // n res_node_stride + c), 16-byte aligned
  const void* res_h = nullptr;
  bool res_f32 = false;
  void* res_out = nullptr;
  void* res_out16 = nullptr;
  int64_t res_shot_stride = 0, res_node_stride = 0;
  // tensor-core path: a device counter that is zero when the kernel starts hands out tiles dynamically (null:
  // static striding)
  unsigned long long* tile_counter = nullptr;
};

// Tensor maps a caller may prepare once and reuse across launches (the pre-decoder does).
struct GmmMaps {
  CUtensorMap x;
  CUtensorMap w;
};

void set_error(const std::string& msg);
int fail(int code, const std::string& msg);

// tcgen05 path: bf16 x / W / y, fp32 accumulation in tensor memory.  Ci >= 64 and Ci % 8 == 0, Co % 32 == 0,
// Co <= 256.  Returns 0 or an error code (message in the thread's last error).
int gmm_tc_check(const GmmProblem& p);
int gmm_tc_make_maps(const GmmProblem& p, GmmMaps* maps);
int gmm_tc_launch(const GmmProblem& p, const GmmMaps& maps, int* status, uint64_t timeout_ns, cudaStream_t stream);
// Shots per tensor-core tile (TM of the blocked layout) for C_out.
int gmm_tc_tile_shots(int Co);

// Node-tiled tcgen05 path for small batches (rows of the MMA = 128 target nodes of one shot): bf16, rows layouts
// with contiguous channels, Ci and Co in {64, 128}.  Same bits as gmm_tc_launch for the same shot.
bool gmm_nodes_supported(const GmmProblem& p);
int gmm_nodes_launch(const GmmProblem& p, int* status, uint64_t timeout_ns, cudaStream_t stream);

// CTA-pair tcgen05 path (cta_group::2) for blocked hidden-128 steps with GELU epilogues (optionally the head) and
// at most 8 relations: W halves resident in shared memory, activations in the blocked layout with 128-shot blocks
// (gmm_pair_tile_shots()).  type_order: for two weight types, the targets in processing order grouped by type
// (n_type0 of type 0 first); counters: two device words the launch clears.  stream_w: the W halves are not resident
// but stream with the activations (two 128-shot blocks per CTA, 512-shot pair tiles).
bool gmm_pair_supported(const GmmProblem& p);
int gmm_pair_make_maps(const GmmProblem& p, GmmMaps* maps);
int gmm_pair_launch(const GmmProblem& p, const GmmMaps& maps, const int32_t* type_order, int n_type0,
                    unsigned long long* counters, int* status, uint64_t timeout_ns, cudaStream_t stream,
                    bool stream_w = false);
int gmm_pair_tile_shots();

// CUDA-core path: fp32 (f32 = true) or bf16 storage, fp32 accumulation.  Any Ci, Co % 4 == 0, Co <= 256.
int gmm_fma_launch(const GmmProblem& p, bool f32, cudaStream_t stream);

int num_sms();
// Opt a kernel in to `bytes` of dynamic shared memory on the current device (once per device and kernel).
int allow_smem(const void* fn, int bytes);
// Launch with programmatic stream serialization (the kernel's prologue may overlap the previous kernel; the kernel
// calls pdl_wait before it reads what earlier kernels wrote), optionally as clusters of cluster_x CTAs.
int launch_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, void** args, int cluster_x,
               const char* what);

// cuTensorMapEncodeTiled through the runtime's driver entry point (null when the driver lacks it).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// Backward (gmm_bwd.cu).  W (Co, K, Ci) -> W' (Ci, K, Co).
int transpose_w_launch(const void* w, void* wt, int K, int Ci, int Co, int32_t dtype, cudaStream_t stream);
// dw (Co, K Ci) fp32 = sum over rows of gy^T gather(x); ws holds the per-split partial sums.
int gmm_wgrad_launch(const void* x, const void* gy, const int32_t* idx, float* dw, void* ws, size_t ws_bytes,
                     int64_t B, int32_t NS, int32_t NT, int32_t K, int32_t Ci, int32_t Co, int32_t dtype,
                     int* status, cudaStream_t stream);
size_t gmm_wgrad_workspace(int64_t B, int32_t NT, int32_t K, int32_t Ci, int32_t Co, int32_t dtype);

// The device tables and weights of a pre-decoder handle (predecoder.cu), for kernels built on the same model.
int predecoder_internals(const struct bpc_predecoder* h, bpc_predecoder_config* cfg, const void** embed,
                         const void** w_c2d, const void** w_d2c, const float** head_w, const float** head_b,
                         const int32_t** c2d, const int32_t** d2c, const int32_t** xor_nbr);

// CUDA device ordinal that was current when the pre-decoder handle was created (its tables and weights live there).
int predecoder_device(const struct bpc_predecoder* h);

// Device status word of the stand-alone op entry points (bpc_gather_mm_*), one per device.
int* op_status_ptr();

}  // namespace bpc
