/* bpc.h -- C ABI of the B200 bipartite-conv pre-decoder library (libbpc.so).
 *
 * Plain pointers and sizes only.  Every device pointer is caller-owned device memory, every launch goes on the
 * caller's stream (a cudaStream_t passed as bpc_stream_t; 0 = the legacy default stream), and no entry point
 * allocates device memory after bpc_predecoder_create / bpc_predecoder_set_weights.  Every function returns
 * BPC_OK (0) or an error code; bpc_last_error() gives the calling thread's last message.  The reference's host side
 * returns 0 / non-0 with an error buffer in the same way (evaluation/timing/d7/router.cc:229,380).
 */
#ifndef BPC_H_
#define BPC_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define BPC_API __attribute__((visibility("default")))
#else
#define BPC_API
#endif

typedef struct CUstream_st* bpc_stream_t;

enum {
  BPC_OK = 0,
  BPC_ERR_ARG = 2,      /* invalid shape, stride, alignment or dtype */
  BPC_ERR_DRIVER = 3,   /* the CUDA driver lacks an entry point or rejected a tensor map */
  BPC_ERR_LAUNCH = 4,   /* a kernel launch or CUDA runtime call failed */
  BPC_ERR_DEVICE = 5,   /* a kernel reported a watchdog timeout through the status word */
  BPC_ERR_SPACE = 6     /* the workspace is smaller than bpc_predecoder_workspace_size() */
};

enum { BPC_DTYPE_F32 = 0, BPC_DTYPE_BF16 = 1 };

/* Library version, (major << 16) | minor. */
BPC_API int bpc_version(void);

/* Copies the calling thread's last error message (NUL-terminated, truncated to len) and returns its length. */
BPC_API int bpc_last_error(char* buf, int len);

/* One bipartite-convolution step, the reference's gather_mm forward:
 *   y[b, n, :] = sum_r x[b, idx[n, r], :] W_r^T,   W (Co, K*Ci) row-major, W_r = W[:, r*Ci:(r+1)*Ci]
 * x (B, NS, Ci), y (B, NT, Co), idx (NT, K) int32 with NS (or any value outside [0, NS)) reading a zero row.
 * dtype BPC_DTYPE_BF16: bf16 x / w / y, fp32 accumulation (tcgen05 tensor cores when Ci >= 64, Co % 32 == 0,
 * Co <= 256, K <= 16; CUDA cores otherwise); BPC_DTYPE_F32: fp32 throughout on the CUDA cores.
 * Replaces: training/bb/ising_compare/bb/cascade_net.py:140-153,174-175 (_GatherMM.forward / gather_mm) and
 * cascade_triton.py:100-117,139-148 (gmm with transposed=False, the op cascade::gmm). */
BPC_API int bpc_gather_mm_fwd(const void* x, const void* w, const int32_t* idx, void* y, int64_t B, int32_t NS, int32_t NT,
                      int32_t K, int32_t Ci, int32_t Co, int32_t dtype, bpc_stream_t stream);

/* Epilogues of bpc_gather_mm_fwd_ex. */
enum { BPC_EPILOGUE_STORE = 0, BPC_EPILOGUE_AFFINE_SILU = 1, BPC_EPILOGUE_ADD = 2 };

/* bpc_gather_mm_fwd with two weight sets and an epilogue, for the layers around the op (no reference counterpart as
 * one call; it computes what the reference's BipartiteConv / Block compose from several calls):
 *   y[b, n, :] = epi( sum_r x[b, idx[n, r], :] W_{t(n), r}^T ),  t(n) = (n >= type_split), W = n_wtypes stacked
 *   (Co, K*Ci) matrices; epi = identity (BPC_EPILOGUE_STORE), c -> SiLU(scale[c] v + shift[c])
 *   (BPC_EPILOGUE_AFFINE_SILU: an inference BatchNorm + SiLU; scale / shift fp32 (Co,) device vectors), or
 *   y[b, n, :] += v (BPC_EPILOGUE_ADD: y is read and written, same dtype).
 * The concatenation of the reference's per-type calls (cascade_net.py:228-233) is one call with n_wtypes = 2 when
 * the targets are ordered by type. */
BPC_API int bpc_gather_mm_fwd_ex(const void* x, const void* w, const int32_t* idx, void* y, int64_t B, int32_t NS,
                                 int32_t NT, int32_t K, int32_t Ci, int32_t Co, int32_t n_wtypes, int32_t type_split,
                                 int32_t epilogue, const float* scale, const float* shift, int32_t dtype,
                                 bpc_stream_t stream);

/* The boundary between two Cascade bottleneck blocks in one launch (eval; H = 512 with a 128-channel bottleneck, the
 * reference's C14 blocks, cascade_net.py:236-259): from the output x3 of one block's bipartite convolution to the
 * input of the next block's convolution,
 *   u = bf16(x3 W_up^T);  h' = scale_h h + scale_u u (fp32, written to h_out unless it is NULL; h_out may be h);
 *   x1 = bf16(SiLU(a1 h' + b1));
 *   w_down != NULL: y = bf16(SiLU(a2 (x1 W_down^T) + b2)) (rows, Hb): the next block's down projection + BN2 + SiLU;
 *   w_down == NULL: y = x1 (rows, H), or nothing when y is NULL (after the last block: a1, b1 = bn_out).
 * x3 (rows, Hb) bf16, w_up (H, Hb) bf16, h (rows, H) fp32, w_down (Hb, H) bf16; a1, b1 (H) and a2, b2 (Hb) fp32 (the
 * folded inference BatchNorms).  The same bits as bpc_residual_affine_silu around a bf16 up GEMM and the op's
 * affine + SiLU down projection.  Buffers 16-byte aligned (a2, b2: 8-byte). */
BPC_API int bpc_cascade_boundary(const void* x3, const void* w_up, const float* h, float* h_out, float scale_h,
                                 float scale_u, const float* a1, const float* b1, const void* w_down, const float* a2,
                                 const float* b2, void* y, int64_t rows, int32_t H, int32_t Hb, bpc_stream_t stream);

/* bpc_cascade_boundary for the first block of a Cascade network, whose stream is the embedding of the detector tokens
 * (CascadeBB.tokens / backbone, cascade_net.py:310-318): h[shot, node] = E[tbase[node] + det[shot, gidx[node]]]
 * (gidx[node] == D: no detector, token tbase[node]) is read from the 5 x H table instead of memory.  det (B, D) uint8,
 * gidx, tbase (N) int32, E (5, H) fp32 16-byte aligned; rows = B N; the rest as bpc_cascade_boundary. */
BPC_API int bpc_cascade_boundary_tokens(const void* x3, const void* w_up, const uint8_t* det, const int32_t* gidx,
                                        const int32_t* tbase, const float* E, int32_t D, int32_t N, float* h_out,
                                        float scale_h, float scale_u, const float* a1, const float* b1,
                                        const void* w_down, const float* a2, const float* b2, void* y, int64_t B,
                                        int32_t H, int32_t Hb, bpc_stream_t stream);

/* The Cascade network's stem and its first block's BN1 + SiLU in one pass (cascade_net.py:279-285,310-318 and the
 * Block's first BatchNorm): x1[shot, node, :] = bf16(SiLU(a1 E[token] + b1)) with the token as in
 * bpc_cascade_boundary_tokens, without writing the embedded stream.  x1 (B, N, H) bf16 16-byte aligned, H % 8 == 0. */
BPC_API int bpc_cascade_stem(const uint8_t* det, const int32_t* gidx, const int32_t* tbase, const float* E, int32_t D,
                             int32_t N, const float* a1, const float* b1, void* x1, int64_t B, int32_t H,
                             bpc_stream_t stream);

/* One memory-bound pass over a (rows, H) fp32 residual stream of the Cascade bottleneck block (no reference
 * counterpart as one call; it replaces the casts, scale, add and activation torch runs between the reference Block's
 * up projection and the next block's first BatchNorm, cascade_net.py:236-259):
 *   v = scale_h h + scale_u u (u bf16 (rows, H), may be NULL);  out = v (fp32, may be NULL);
 *   x = SiLU(a[c] v + b[c]) (bf16, may be NULL; a, b fp32 (H,): an inference BatchNorm folded to scale and shift;
 *   SiLU as x/2 + x/2 tanh(x/2) on the hardware tanh, its result rounded to bf16).
 * H % 8 == 0; every pointer 16-byte aligned. */
BPC_API int bpc_residual_affine_silu(const float* h, const void* u, float* out, void* x, int64_t rows, int32_t H,
                                     float scale_h, float scale_u, const float* a, const float* b, bpc_stream_t stream);

/* The residual steps of the training network around the op, one memory-bound pass each (no reference counterpart as
 * one call; torch runs GELU, the residual add and the casts as separate kernels):
 *   forward   y = h + bf16(GELU(a))   h bf16 -> y bf16 (rounded once); h f32 -> y f32 and y_bf16 = bf16(y);
 *             h NULL -> y = bf16(GELU(a)) (h_dtype ignored)
 *   backward  g = gy (+ gy_bf16, f32 stream only; on the f32 stream either may be NULL = zero);  gh = g (f32
 *             stream; may be NULL);
 *             ga = bf16(GELU'(a) * g), g rounded to bf16 first on the f32 stream
 * a and ga are bf16 (n_types, B, NT / n_types, C): the pre-activations of target type t are one contiguous block;
 * h, y, gy, gh are (B, NT, C).  GELU is the tanh form.  C % 8 == 0, every pointer 16-byte aligned. */
BPC_API int bpc_gelu_residual_fwd(const void* a, const void* h, void* y, void* y_bf16, int64_t B, int32_t NT, int32_t C,
                                  int32_t n_types, int32_t h_dtype, bpc_stream_t stream);
BPC_API int bpc_gelu_residual_bwd(const void* gy, const void* gy_bf16, const void* a, void* gh, void* ga, int64_t B,
                                  int32_t NT, int32_t C, int32_t n_types, int32_t gy_dtype, bpc_stream_t stream);

/* The detector-token embedding of the training network (cascade_net.py:279-285,310-312: tok = 2 type + bit, here
 * with the 4 tokens of a rotated-surface check), forward and weight gradient:
 *   forward   h[b, n, :] = E[2 check_type[n] + det[b, n], :]  (fp32 (B, N, C)) and h_bf16 = bf16(h), one pass
 *   backward  dE[k, :] = sum over (b, n) with token k of g[b, n, :] + g_bf16[b, n, :] (either may be NULL), fp32 (4, C),
 *             deterministic (fixed per-block partial sums in `workspace`, then a fixed-order sum)
 * det (B, N) uint8 0/1, check_type (N) uint8 0/1, E (4, C) fp32; C % 8 == 0 (forward), C % 4 == 0 and C <= 256
 * with g 16-byte and g_bf16 8-byte aligned (backward). */
BPC_API int bpc_embed_tokens_fwd(const uint8_t* det, const uint8_t* check_type, const float* E, float* h, void* h_bf16,
                                 int64_t B, int32_t N, int32_t C, bpc_stream_t stream);
BPC_API size_t bpc_embed_tokens_bwd_workspace_size(int32_t C);
BPC_API int bpc_embed_tokens_bwd(const uint8_t* det, const uint8_t* check_type, const float* g, const void* g_bf16,
                                 float* dE, void* workspace, size_t workspace_bytes, int64_t B, int32_t N, int32_t C,
                                 bpc_stream_t stream);

/* The training network's X/Z head and its loss, one pass each way (the head linear(h_d, W, b) under bf16 autocast and
 * the mean BCE-with-logits of the reference's training step, cascade_train.py:292-320):
 *   forward:  z_j = bf16(sum_c hd[r, c] W[j, c] + b[j]) (W, b rounded to bf16);  *loss = mean over r, j of
 *             BCE-with-logits(z_j, labels[r, j])
 *   backward: g_j = bf16((sigmoid(z_j) - labels[r, j]) *grad_loss / n);  dh[r, c] = bf16(g_0 W[0, c] + g_1 W[1, c]);
 *             dW[j, c] = bf16(sum_r g_j hd[r, c]);  db[j] = bf16(sum_r g_j)   (n = 2 rows; fixed-order fp32 sums)
 * hd, dh (rows, C) bf16 8-byte aligned, C % 4 == 0 and C <= 128; W (2, C), b (2), loss, grad_loss, dW, db fp32 device
 * memory; labels (rows, 2) uint8 0/1; workspace of bpc_head_bce_workspace_size(C) bytes; rows > 0. */
BPC_API size_t bpc_head_bce_workspace_size(int32_t C);
BPC_API int bpc_head_bce_fwd(const void* hd, const float* W, const float* b, const uint8_t* labels, float* loss,
                             void* workspace, size_t workspace_bytes, int64_t rows, int32_t C, bpc_stream_t stream);
BPC_API int bpc_head_bce_bwd(const void* hd, const float* W, const float* b, const uint8_t* labels,
                             const float* grad_loss, void* dh, float* dW, float* db, void* workspace,
                             size_t workspace_bytes, int64_t rows, int32_t C, bpc_stream_t stream);

/* One residual step of the training network in one launch (one weight set; row layouts; bf16; the wide-tile
 * tensor-core kernel: C_in, C_out in {64, 96, 128}): a = gather_mm(x, w, idx), (B, NT, Co) bf16, kept for the
 * backward, and in the same epilogue the residual stream of these NT targets, as bpc_gelu_residual_fwd computes it:
 *   g = bf16(GELU(a));  h fp32: out = h + g (fp32) and out_bf16 = bf16(out);  h bf16: out = bf16(h + g);  h NULL:
 *   out = g (bf16).
 * h, out, out_bf16: the targets' first row of (B, *, Co) streams whose shots are stream_shot_stride elements apart
 * (a target type's block of a type-major stream), 16-byte aligned.  No reference counterpart: the reference composes
 * gather_mm, GELU and the add under autocast (cascade_net.py:140-175,228-233). */
BPC_API int bpc_gather_mm_fwd_gelu(const void* x, const void* w, const int32_t* idx, void* a, int64_t B, int32_t NS,
                                   int32_t NT, int32_t K, int32_t Ci, int32_t Co, const void* h, int32_t h_dtype,
                                   void* out, void* out_bf16, int64_t stream_shot_stride, bpc_stream_t stream);
/* Input gradient of bpc_gather_mm_fwd through the target table:
 *   gx[b, s, :] = sum_r gy[b, tgt[s, r], :] W_r,   tgt (NS, K) int32, NT (or any value outside [0, NT)) = none
 * gy (B, NT, Co), gx (B, NS, Ci), W (Co, K*Ci) as in the forward.  tgt[s, r] is the target that reads source s
 * through relation r, the reference's where(inv < NT*K, inv // K, NT).  w_t is caller scratch of K*Ci*Co elements
 * of dtype that receives W rearranged as (Ci, K*Co), so the forward kernels compute the sum (tensor cores when
 * Co >= 64, Ci % 32 == 0, Ci <= 256, K <= 16 and bf16).
 * Replaces: cascade_triton.py:100-117 (gmm with transposed=True), cascade_net.py:155-171 (_GatherMM.backward, gx). */
BPC_API int bpc_gather_mm_dgrad(const void* gy, const void* w, const int32_t* tgt, void* gx, void* w_t, int64_t B,
                                int32_t NT, int32_t NS, int32_t K, int32_t Ci, int32_t Co, int32_t dtype,
                                bpc_stream_t stream);

/* bpc_gather_mm_dgrad that adds into gx when accumulate != 0 (gx += the sum, rounded once to gx's dtype): the input
 * gradient of a source read by targets of two types (two weight sets, two target tables) in two calls, where
 * autograd over the reference's per-type calls (cascade_net.py:228-233) sums two gradients. */
BPC_API int bpc_gather_mm_dgrad_ex(const void* gy, const void* w, const int32_t* tgt, void* gx, void* w_t, int64_t B,
                                   int32_t NT, int32_t NS, int32_t K, int32_t Ci, int32_t Co, int32_t accumulate,
                                   int32_t dtype, bpc_stream_t stream);

/* Weight gradient of bpc_gather_mm_fwd, fp32 and deterministic (fixed split of the rows, fixed-order sum):
 *   dw[o, r*Ci + i] = sum_{b, n} gy[b, n, o] x[b, idx[n, r], i]      (pads contribute nothing)
 * x (B, NS, Ci), gy (B, NT, Co), idx (NT, K) int32, dw (Co, K*Ci) fp32.  workspace: caller scratch of at least
 * bpc_gather_mm_wgrad_workspace_size() bytes (per-split fp32 partial sums), 16-byte aligned.
 * Replaces: cascade_triton.py:64-93,120-136,151-158 (_gmm_wgrad, gmm_wgrad, the op cascade::gmm_wgrad). */
BPC_API int bpc_gather_mm_wgrad(const void* x, const void* gy, const int32_t* idx, float* dw, void* workspace,
                                size_t workspace_bytes, int64_t B, int32_t NS, int32_t NT, int32_t K, int32_t Ci,
                                int32_t Co, int32_t dtype, bpc_stream_t stream);

/* Workspace bytes bpc_gather_mm_wgrad needs for these shapes on the current device. */
BPC_API size_t bpc_gather_mm_wgrad_workspace_size(int64_t B, int32_t NS, int32_t NT, int32_t K, int32_t Ci, int32_t Co,
                                                  int32_t dtype);

/* Synchronises `stream`, reads and clears the current device's watchdog status word of the three gather_mm entry
 * points (0 = every bounded wait completed).  Returns BPC_ERR_DEVICE when a tensor-core kernel gave up a wait, in
 * which case that launch's output is not valid. */
BPC_API int bpc_gather_mm_status(bpc_stream_t stream, int* status);

/* ------------------------------------------------------------------------------------------------------------
 * Pre-decoder: detectors (B, N_c) uint8 -> per-data-node X/Z logits (B, N_d, 2) fp32 and the residual syndrome
 * (B, N_c) uint8, through `layers` x [check -> data, data -> check] bipartite convolutions of width `channels`.
 * Replaces the module stack BipartiteConv.forward / CascadeBB.forward (cascade_net.py:228-233,342-343) for the
 * rotated surface code; the X/Z head and the syndrome cancellation have no reference counterpart in-tree (the
 * reference calls NVIDIA Ising-Decoding's pre-decoder for the residual, evaluation/convlines/opponents.py:43-86). */
typedef struct bpc_predecoder bpc_predecoder;

typedef struct {
  int32_t layers;          /* L */
  int32_t channels;        /* C */
  int32_t K;               /* relations per target (8 for the rotated surface code) */
  int32_t dtype;           /* BPC_DTYPE_BF16 or BPC_DTYPE_F32 */
  int32_t n_checks;        /* N_c */
  int32_t n_data;          /* N_d */
  int32_t z_check_begin;   /* first Z-check node: checks [0, z) use the X weights of a data -> check step */
} bpc_predecoder_config;

/* Tables (host memory, copied): c2d (N_d, K) int32 source check per data node (N_c = pad), d2c (N_c, K) int32 source
 * data node per check (N_d = pad), xor_nbr (N_d, 2, 2) int32 checks flipped by a predicted X / Z flip (-1 = none),
 * check_type (N_c) uint8 0 X / 1 Z, check_order (N_c) int32 the order in which a data -> check step visits the checks
 * (a permutation; NULL = node order; visiting X and Z checks of one round together lets each data block be read
 * from HBM once per step).  Allocates the handle's device tables and weights. */
BPC_API int bpc_predecoder_create(const bpc_predecoder_config* cfg, const int32_t* c2d, const int32_t* d2c,
                          const int32_t* xor_nbr, const uint8_t* check_type, const int32_t* check_order,
                          bpc_predecoder** out);

/* Weights (host memory, copied; element type = cfg.dtype except head_w / head_b which are fp32):
 * embed (4, C); w_c2d (L, C, K*C); w_d2c (L, 2, C, K*C) (X then Z checks); head_w (2, C); head_b (2). */
BPC_API int bpc_predecoder_set_weights(bpc_predecoder* h, const void* embed, const void* w_c2d, const void* w_d2c,
                               const float* head_w, const float* head_b);

/* Workspace bytes that let bpc_predecoder_forward process `chunk_shots` shots per pass (rounded up to 128). */
BPC_API size_t bpc_predecoder_workspace_size(const bpc_predecoder* h, int64_t chunk_shots);

/* Forward pass on device buffers: det (B, N_c) uint8, logits (B, N_d, 2) fp32, residual (B, N_c) uint8.  Shots are
 * processed in chunks of the size the workspace allows; nothing is allocated.  Asynchronous on `stream`. */
BPC_API int bpc_predecoder_forward(bpc_predecoder* h, const uint8_t* det, float* logits, uint8_t* residual, int64_t B,
                           void* workspace, size_t workspace_bytes, bpc_stream_t stream);

/* Measurement hook: `events` holds 2 * n_pairs cudaEvent_t created by the caller (timing enabled).  Every later
 * bpc_predecoder_forward records events[2 i] just before and events[2 i + 1] just after its i-th bipartite-step
 * launch (i counts from 0 in each call, in launch order: per chunk, per layer, check -> data then data -> check), for
 * as many launches as there are pairs.  n_pairs = 0 turns it off.  No reference counterpart (the reference times
 * whole CUDA-graph replays, evaluation/timing/gpu_term.py:5-10). */
BPC_API int bpc_predecoder_record_step_events(bpc_predecoder* h, void* const* events, int n_pairs);

/* Reads (and clears) the device status word the kernels' watchdogs write; synchronises `stream`.
 * *status = 0 when every wait completed.  Returns BPC_ERR_DEVICE when a watchdog fired. */
BPC_API int bpc_predecoder_status(bpc_predecoder* h, bpc_stream_t stream, int* status);

BPC_API void bpc_predecoder_destroy(bpc_predecoder* h);

/* Forward pass for callers that cannot allocate device memory (a host whose memory pool owns the device heap, a
 * real-time loop that must not enter the CUDA allocator, a plugin handed only input and output pointers).  Same
 * contract as bpc_predecoder_forward, but the scratch is a fixed array inside the library's device image
 * (bpc_noalloc_scratch_bytes(), 64 MiB, held by every GPU that loads the library until exit), so the caller passes
 * only det, logits and residual.  A network whose 256-shot pass needs more scratch than that is rejected with
 * BPC_ERR_SPACE, and a handle created on another device than the current one with BPC_ERR_ARG.  The first call in
 * each CUDA context looks the array's address up (cudaGetSymbolAddress) and should come before any stream capture;
 * every call shares the array, so calls whose work overlaps on the GPU race.
 * No counterpart in the reference (it allocates through torch). */
BPC_API int bpc_predecoder_forward_noalloc(bpc_predecoder* h, const uint8_t* det, float* logits, uint8_t* residual,
                                           int64_t B, bpc_stream_t stream);

/* ------------------------------------------------------------------------------------------------------------
 * Persistent streaming pre-decoder (sliding window of `window` rounds, batch 1): one resident kernel serves rounds
 * through a request line in mapped host memory -- the reference's persistent-kernel protocol
 * (evaluation/timing/d7/router.cc:170-223,576-650, kernel.cu:310-369,440-527; s9_pers_*): a tagged request with
 * the round's detectors, a response with the same tag, a stop command, and watchdogs (an idle limit while waiting
 * for requests, a step limit on every wait inside a round) that end the kernel with a status instead of a hang.
 * Served networks: bf16, C = 64, K = 8, at most 8 layers, at most 8 tiles of 128 nodes per step (d = 17 with a
 * window of 3 rounds is 7 and 8).  Two layouts of the same arithmetic (the same bits):
 *   BPC_STREAM_CLUSTERS     8 clusters x 8 CTAs (64 SMs), one relation per CTA, a bounded grid barrier per step;
 *   BPC_STREAM_ONE_CLUSTER  one cluster of 2 x (tiles per step) CTAs (16 SMs at d = 17), a CTA pair per tile, bounded
 *                           cluster barriers on mbarriers: no step hand-off through L2 flags;
 *   BPC_STREAM_AUTO         the layout measured faster on B200: the 8 clusters (per step ~4.5 us against ~6 us; the
 *                           one-cluster layout pulls four relations' gathered rows through each of its SMs). */
typedef struct bpc_stream bpc_stream;
#define BPC_STREAM_AUTO 0
#define BPC_STREAM_CLUSTERS 1
#define BPC_STREAM_ONE_CLUSTER 2

/* The pre-decoder's tables and weights (device, not copied: keep h alive), the window and the detectors (nh per
 * check type) and data qubits (nq) per round.  Allocates the device state and the mapped lines. */
BPC_API int bpc_stream_create(const bpc_predecoder* h, int32_t window, int32_t nh, int32_t nq, int32_t idle_timeout_ms,
                              bpc_stream** out);
/* bpc_stream_create with a layout (BPC_STREAM_*); bpc_stream_create is BPC_STREAM_AUTO. */
BPC_API int bpc_stream_create_ex(const bpc_predecoder* h, int32_t window, int32_t nh, int32_t nq,
                                 int32_t idle_timeout_ms, int32_t layout, bpc_stream** out);
/* Launches the resident kernel on the handle's own non-blocking stream and waits for it to report ready. */
BPC_API int bpc_stream_start(bpc_stream* s);
/* One round: round_dets (2 nh) host bytes, this round's X then Z detectors -> residual (N_c bytes) of the window and
 * logits (nq x 2 fp32) of the newest round, host buffers (either may be NULL).  Spins on the response tag for at most
 * timeout_us (<= 0: no limit besides the kernel's own watchdogs). */
BPC_API int bpc_stream_round(bpc_stream* s, const uint8_t* round_dets, uint8_t* residual, float* logits,
                             int64_t timeout_us);
/* n_rounds rounds in a row (rounds: n_rounds x 2 nh bytes); per-round results and the host wall-clock latency of
 * each round in ns (each output may be NULL). */
BPC_API int bpc_stream_run(bpc_stream* s, const uint8_t* rounds, int64_t n_rounds, uint8_t* residuals, float* logits,
                           int64_t* latency_ns, int64_t timeout_us);
/* Sends the stop command and waits (bounded) for the kernel to leave. */
BPC_API int bpc_stream_stop(bpc_stream* s);
/* The kernel's status word: 0 starting, 1 ready / serving, 2 stopped, 3 watchdog fired, 4 idle limit reached. */
BPC_API int bpc_stream_status(const bpc_stream* s);
/* The layout of the kernel that runs or ran last (BPC_STREAM_CLUSTERS or BPC_STREAM_ONE_CLUSTER; 0 before the first
 * start). */
BPC_API int bpc_stream_layout(const bpc_stream* s);
/* Tracing (set before bpc_stream_start): thread 0 of every CTA stamps the device global timer (ns) at the phase
 * boundaries of each step, overwritten round after round.  bpc_stream_trace_read (after bpc_stream_stop) copies the
 * stamps of the last round served: n >= 64 x 16 x 8 values, [CTA][slot][k]; slots 0 .. 2 L - 2 are the steps (k: 0
 * start, 1 weights / gathered rows ready, 2 MMAs issued, 3 accumulators ready, 4 partials exchanged, 5 epilogue
 * done, 6 past the barrier), slot 15 the round (0 waiting for the request, 1 request accepted, 2 window embedded --
 * in the 8-cluster layout the window's detectors taken in, the embedding overlapping the first step --, 3 past the
 * barrier after the embedding (one-cluster layout), 4 response published); 0 where a CTA did not pass. */
BPC_API int bpc_stream_trace(bpc_stream* s, int32_t on);
BPC_API int bpc_stream_trace_read(const bpc_stream* s, uint64_t* out, int64_t n);
BPC_API void bpc_stream_destroy(bpc_stream* s);

/* Routing to a fallback decoder and its hand-off (the reference's decoder.route / decode and the router's matcher
 * call: evaluation/convlines/decoder.py:116-142, evaluation/timing/d7/router.cc:142-168).  Per shot b of a
 * pre-decoded batch (logits (B, n_data, 2) fp32, residual (B, n_checks) uint8, device buffers):
 *   conf[b] = min |logits[b, :, :]|,  weight[b] = number of set residual bits,
 *   routed[b] = conf[b] < tau || (route_residual && weight[b] > 0)        (uint8, (B,))
 * and the routed shots in ascending order: index[i] (int64, room for B), their residual rows handoff[i, :] (uint8,
 * room for B x n_checks, or NULL), the count in *n_routed (a device int64).  conf / weight may be NULL.  workspace:
 * bpc_route_workspace_size(B) bytes of device memory, 8-byte aligned.  Every launch on `stream`. */
BPC_API int bpc_route(const float* logits, const uint8_t* residual, int64_t B, int32_t n_data, int32_t n_checks,
                      float tau, int32_t route_residual, uint8_t* routed, int64_t* index, uint8_t* handoff,
                      int64_t* n_routed, float* conf, int32_t* weight, void* workspace, size_t workspace_bytes,
                      bpc_stream_t stream);
BPC_API size_t bpc_route_workspace_size(int64_t B);

/* Size in bytes of the scratch array bpc_predecoder_forward_noalloc runs on. */
BPC_API size_t bpc_noalloc_scratch_bytes(void);

#ifdef __cplusplus
}
#endif

#endif /* BPC_H_ */
