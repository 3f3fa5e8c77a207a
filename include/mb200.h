/*
 * libmb200 — the C ABI of the MetalBench B200 backend.
 *
 * This library replaces the reference's native host dispatcher
 * (metal/scripts/main.mm:73-197, timing.mm:125-193, setup.cpp:116-136) and its
 * Metal kernels. Python (the harness, via ctypes) or any FFI binds these
 * symbols; no C++ types, exceptions or torch types cross the boundary.
 *
 * Conventions
 *   - Every function returns 0 on success or a negative MB_ERR_* code; the
 *     message of the last failure on the calling thread is mb_last_error().
 *   - Device-pointer entry points (mb_<kernel>_*) take plain device pointers,
 *     sizes and a cudaStream_t passed as void*; they only enqueue work.
 *   - mb_run is the manifest-style entry point: host (or device) buffers by
 *     reference binding index, timed warmup+iters launches, outputs copied back.
 *   - Calls are serialised per device by the caller; one process per GPU.
 */
#ifndef MB200_H
#define MB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define MB_OK 0
#define MB_ERR_BAD_ARG -1       /* wrong shape / size / alignment / dtype      */
#define MB_ERR_UNKNOWN_KERNEL -2 /* name not in the kernel table               */
#define MB_ERR_CUDA -3          /* a CUDA runtime/driver call failed           */
#define MB_ERR_NCCL -4          /* an NCCL call failed                          */
#define MB_ERR_TIMEOUT -5       /* a bounded device wait or comm init timed out */
#define MB_ERR_NOT_INIT -6      /* mb_init was not called                       */

/* ---- dtype tags (superset of mlx_helpers.py:83-89 "f32|f16|i32|u32") ---- */
#define MB_F32 0
#define MB_F16 1
#define MB_I32 2
#define MB_U32 3
#define MB_BF16 4

/* ---- buffer roles (manifest "role", mlx_helpers.py:301-313) ------------- */
#define MB_ROLE_INPUT 0
#define MB_ROLE_OUTPUT 1

/* ---- buffer flags -------------------------------------------------------- */
#define MB_DEVICE_PTR 1 /* ptr is already a device pointer (e.g. a torch tensor) */

typedef struct mb_buf {
  int binding; /* reference [[buffer(i)]] index                               */
  int role;    /* MB_ROLE_INPUT / MB_ROLE_OUTPUT                              */
  int dtype;   /* MB_F32 ...                                                  */
  int flags;   /* MB_DEVICE_PTR                                               */
  void* ptr;   /* host pointer (inputs read, outputs written) or device ptr  */
  size_t bytes;
} mb_buf;

typedef struct mb_scalar {
  int binding; /* reference scalar binding index (registry "scalars")         */
  int dtype;   /* MB_U32 / MB_I32 / MB_F32                                    */
  union {
    uint32_t u;
    int32_t i;
    float f;
  } v;
} mb_scalar;

/* Timing of mb_run, same statistics as timing.mm:150-159: per-launch device
 * times sorted, median = times[n/2]. */
typedef struct mb_timing {
  double min_ms;
  double median_ms;
  double mean_ms;
  int iters;
  int smem_bytes;      /* dynamic shared memory per CTA of the main kernel    */
  int threads_per_cta; /* threads per CTA of the main kernel                  */
  int launches_per_iter;
  double h2d_ms; /* host->device copy time of the inputs (0 for device ptrs) */
  double d2h_ms; /* device->host copy time of the outputs                    */
  /* config {"profile": true} (the reference's --profile, main.mm:98 and
   * timing.mm:163-190): one extra dispatch after the timed ones, inside the
   * NVTX range "mb_profile:<kernel>" for an outside profiler (ncu --nvtx
   * --nvtx-include "mb_profile:<kernel>/"); its CUDA-event time, else -1.
   * Every timed dispatch sits in an NVTX range "mb_timed:<kernel>". */
  double profile_ms;
} mb_timing;

/* Device description (replaces setup.cpp:116-136 chip detection). */
typedef struct mb_device {
  char name[128];
  char type[32];   /* "b200" on B200, else "sm<major><minor>"                 */
  char bucket[32]; /* results/<bucket>/ directory key                         */
  int sm_count;
  int cc_major;
  int cc_minor;
  int cpu_cores;
  uint64_t hbm_bytes;
  uint64_t ram_bytes;
  int l2_bytes;
  int smem_per_block_optin;
} mb_device;

/* ---- lifecycle / manifest API (replaces metal/scripts/main.mm) ---- */

/* Select the device for this process. rank/world/nccl_id_path are used by the
 * tensor-parallel entry points (world > 1); pass 0/1/NULL for one GPU.
 * timeout_ms bounds communicator set-up. */
int mb_init(int device, int rank, int world, const char* nccl_id_path, int timeout_ms);
void mb_shutdown(void);
const char* mb_last_error(void);
int mb_device_info(mb_device* out);

/* Names understood by mb_run, comma separated (static storage). */
const char* mb_kernel_names(void);

/* Run `kernel` warmup+iters times on the bound buffers and report per-launch
 * device time (main.mm:161-165 + timing.mm:125-193). config_json is an optional
 * flat JSON object of extra keys (e.g. {"padding":1,"flush_l2":true}). */
int mb_run(const char* kernel, const mb_buf* bufs, int nbufs, const mb_scalar* scalars, int nsc,
           const char* config_json, int warmup, int iters, mb_timing* out);

/* Status word that bounded device waits write on timeout; 0 = clean. There is
 * one word per device; both calls act on the current device. Reading it
 * synchronises the device. mb_clear_device_status resets it. The value also
 * includes the word mb_sqr_mm_f32_noalloc falls back to on a device that has
 * no shared word yet. */
int mb_device_status(uint32_t* out);
int mb_clear_device_status(void);

/* Failure-detection self-test (no counterpart in the reference, whose host
 * only has die()): one CTA waits on a barrier that never completes, gives up
 * after timeout_us, records a status bit and returns. Expected result:
 * MB_ERR_TIMEOUT with the context still usable (clear the status afterwards). */
int mb_selftest_bounded_wait(int timeout_us, void* stream);

/* ---- transpose_2d (metal/kernels/common/transpose_2d/default.metal:10-48;
 *      hook mlx/kernels/common/transpose_2d.py:10-11) -------------------- */

/* out[c][r] = in[r][c] for an fp32 rows x cols row-major matrix. */
int mb_transpose_2d_f32(const float* in, float* out, int64_t rows, int64_t cols, void* stream);

/* out[b][c][r] = in[b][r][c] for bf16 (raw uint16) tensors [batch, rows, cols]. */
int mb_transpose_batched_bf16(const uint16_t* in, uint16_t* out, int64_t batch, int64_t rows,
                              int64_t cols, void* stream);

/* Same for fp32 tensors [batch, rows, cols]. */
int mb_transpose_batched_f32(const float* in, float* out, int64_t batch, int64_t rows,
                             int64_t cols, void* stream);

/* ---- GEMM on the tcgen05 core (registry helper matmul,
 *      mlx/kernels/common/registry.py:44-61; sqr_mm hook
 *      mlx/kernels/common/sqr_mm.py:10-11; Metal kernel
 *      metal/kernels/common/sqr_mm.metal:19-111) ------------------------- */

/* C[M,N] (bf16) = A[M,K] (bf16, row-major) @ B, fp32 accumulation.
 * b_layout 0: B is [N,K] row-major (K contiguous, "weights" layout);
 * b_layout 1: B is [K,N] row-major (the reference's A @ B layout).
 * Needs K % 8 == 0, N % 8 == 0, 16-byte aligned pointers. */
int mb_gemm_bf16(const uint16_t* A, const uint16_t* B, uint16_t* C, int64_t M, int64_t N,
                 int64_t K, int b_layout, void* stream);

/* C[M,N] (fp32) = A[M,K] @ B[K,N], all fp32 row-major, fp32-accurate via
 * 3xTF32 on the tensor cores: a prepass writes tf32 hi/lo splits of A and of
 * B^T into `workspace` (mb_sqr_mm_f32_workspace_bytes, 256-byte aligned, caller
 * owned), then lo*hi + hi*lo + hi*hi accumulate in fp32 in TMEM.
 * Needs K % 4 == 0 and a 16-byte aligned A. */
size_t mb_sqr_mm_f32_workspace_bytes(int64_t M, int64_t N, int64_t K);
int mb_sqr_mm_f32(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                  void* workspace, size_t workspace_bytes, void* stream);

/* ---- conv2d (hook mlx/kernels/common/conv2d.py:7-12; registry
 *      mlx/kernels/common/registry.py:469-477; Metal kernel
 *      metal/kernels/common/conv2d/default.metal:31-217) ------------------ */

/* y = conv2d(x, w): x NHWC [N,H,W,Cin] bf16, w OHWI [Cout,KH,KW,Cin] bf16,
 * cross-correlation, symmetric zero padding `pad`, y NHWC [N,H2,W2,Cout] bf16
 * with fp32 accumulation. Needs stride 1, Cin % 64 == 0, Cout % 16 == 0,
 * Cout <= 256, pad < KH and pad < KW, 16-byte aligned pointers. */
int mb_conv2d_nhwc_bf16(const uint16_t* x, const uint16_t* w, uint16_t* y, int N, int H, int W,
                        int Cin, int Cout, int KH, int KW, int stride, int pad, void* stream);

/* fp32 conv2d for the reference's own conv2d_f32 entry (registry
 * mlx/kernels/common/registry.py:469-477: x (8,64,64,64), w (128,3,3,64),
 * pad 0, rtol = atol = 1e-3). Same layouts as the bf16 entry, fp32 buffers,
 * any stride >= 1 and pad >= 0, Cin % 4 == 0, 16-byte aligned x and w. The
 * products use 3xTF32 (fp32-accurate) on the tcgen05 GEMM: an im2col pass
 * writes the tf32-split patch matrix into `workspace`
 * (mb_conv2d_nhwc_f32_workspace_bytes, 256-byte aligned, caller owned). */
size_t mb_conv2d_nhwc_f32_workspace_bytes(int N, int H, int W, int Cin, int Cout, int KH, int KW,
                                          int stride, int pad);
int mb_conv2d_nhwc_f32(const float* x, const float* w, float* y, int N, int H, int W, int Cin,
                       int Cout, int KH, int KW, int stride, int pad, void* workspace,
                       size_t workspace_bytes, void* stream);

/* ---- GQA attention over a paged KV cache (hook
 *      mlx/kernels/full/llama_decoder_layer.py:30-37) ----------------------
 * Cache: k_cache, v_cache = [num_pages][Hkv][64][Dh] bf16; token p of
 * sequence b is in page block_table[b*max_pages + p/64], slot p%64. Query
 * head h reads kv head h / (Hq/Hkv). Dh must be 128. */

/* Decode: one query row per sequence (q [B, ldq]), keys 0..kv_len[b]-1.
 * Split-KV; needs mb_attention_decode_workspace_bytes of caller scratch. */
size_t mb_attention_decode_workspace_bytes(int B, int Hq, int Hkv, int max_kv_len);
int mb_attention_decode_bf16(const uint16_t* q, int ldq, const uint16_t* k_cache,
                             const uint16_t* v_cache, const int* block_table, int max_pages,
                             const int* kv_len, int max_kv_len, int B, int Hq, int Hkv, int Dh,
                             uint16_t* out, int ldo, void* workspace, size_t workspace_bytes,
                             void* stream);

/* Prefill: S query rows per sequence (row b*S+s at position start_pos[b]+s),
 * keys 0..kv_len[b]-1, optional causal mask (key position <= query position). */
int mb_attention_prefill_bf16(const uint16_t* q, int ldq, const uint16_t* k_cache,
                              const uint16_t* v_cache, const int* block_table, int max_pages,
                              const int* start_pos, const int* kv_len, int B, int S, int Hq,
                              int Hkv, int Dh, int causal, uint16_t* out, int ldo, void* stream);

/* ---- LLaMA decoder layer (hook mlx/kernels/full/llama_decoder_layer.py:17-64;
 *      registry mlx/kernels/full/registry.py:87-104; Metal kernel
 *      metal/kernels/full/llama_decoder_layer/default.metal:16-206) ------- */
typedef struct mb_decoder_config {
  int d_model;
  int n_heads;
  int n_kv_heads;
  int head_dim; /* must be 128 */
  int ffn;
  float rope_base;
  float eps;
} mb_decoder_config;

/* Pack the reference-layout weights (device pointers, bf16, (in, out)
 * row-major: W_qkv [D, D+2*Hkv*Dh], W_o [D, D], W_gu [D, 2*ffn] (gate | up),
 * W_down [ffn, D]) into this rank's tensor-parallel shard (tp_world = 1 for one
 * GPU). The layer owns its packed copies; the inputs may be freed after. */
int mb_decoder_layer_create(const mb_decoder_config* cfg, const uint16_t* W_qkv,
                            const uint16_t* W_o, const uint16_t* W_gu, const uint16_t* W_down,
                            int tp_rank, int tp_world, void** layer);
void mb_decoder_layer_destroy(void* layer);
size_t mb_decoder_layer_workspace_bytes(const void* layer, int B, int S, int max_kv_len);

/* y = layer(x) for B sequences of S new tokens (x, y [B*S, D] bf16, row b*S+s
 * at position start_pos[b]+s). The new tokens' rotated K and V are written into
 * the cache first; attention then reads keys 0..kv_len[b]-1 (= start_pos[b]+S),
 * causal or not (the reference hook is non-causal with start_pos 0). S == 1
 * uses the split-KV decode kernel. With tp_world > 1 (after mb_init with the
 * same world) the o-proj and down-proj outputs are summed with NCCL. */
int mb_decoder_layer_forward(const void* layer, const uint16_t* x, uint16_t* y, int B, int S,
                             const int* start_pos, const int* kv_len, int max_kv_len,
                             uint16_t* k_cache, uint16_t* v_cache, const int* block_table,
                             int max_pages, int causal, void* workspace, size_t workspace_bytes,
                             void* stream);

/* mb_decoder_layer_forward with the residual stream kept in fp32 between
 * layers (a stack of layers hands it on): x_res32 [B*S, D] fp32 is the layer
 * input's residual (x must hold its bf16 rounding; null = use x), and when
 * y_res32 is not null it receives the fp32 output beside the bf16 y. Inside
 * the layer the residual adds are fp32 in either case; under tensor
 * parallelism the ranks' fp32 partial products are summed in rank order over
 * NVLink peer memory together with the residual (messages above the peer
 * slot, i.e. prefill: a bf16 NCCL all-reduce, then the residual add). Same
 * reference as
 * mb_decoder_layer_forward (mlx/kernels/full/llama_decoder_layer.py:24-46,
 * whose x stays fp32 throughout). */
int mb_decoder_layer_forward_ex(const void* layer, const uint16_t* x, const float* x_res32,
                                uint16_t* y, float* y_res32, int B, int S, const int* start_pos,
                                const int* kv_len, int max_kv_len, uint16_t* k_cache,
                                uint16_t* v_cache, const int* block_table, int max_pages,
                                int causal, void* workspace, size_t workspace_bytes, void* stream);

/* mb_decoder_layer_forward_ex for layers chained in a stack: the input-side
 * RMSNorm factor of layer l+1, rstd = rsqrt(mean(y_res32^2) + eps) per row, is
 * written by layer l into rstd_out [B*S] fp32 (needs y_res32) from the kernel
 * that forms each output row, and layer l+1 takes it as rstd_in instead of
 * computing it again (null = compute it). Both layers must share eps. Same
 * reference as mb_decoder_layer_forward (the `_rms_norm` of the next layer's
 * input, mlx/kernels/full/llama_decoder_layer.py:48-50). */
int mb_decoder_layer_forward_chain(const void* layer, const uint16_t* x, const float* x_res32,
                                   const float* rstd_in, uint16_t* y, float* y_res32,
                                   float* rstd_out, int B, int S, const int* start_pos,
                                   const int* kv_len, int max_kv_len, uint16_t* k_cache,
                                   uint16_t* v_cache, const int* block_table, int max_pages,
                                   int causal, void* workspace, size_t workspace_bytes,
                                   void* stream);

/* fp32 decoder layer for the reference's own llama_decoder_layer_f32 entry
 * (mlx/kernels/full/llama_decoder_layer.py:24-64; registry
 * mlx/kernels/full/registry.py:87-104: S 64, D 128, H 4 / H_kv 2, head_dim 32,
 * FF 256, rtol = atol = 1e-2). x, y [B*S, D] fp32; weights fp32 in the
 * reference (in, out) layout; head_dim = D/H even and <= 256, D and FF
 * multiples of 4. Every sequence's tokens sit at positions 0..S-1; causal = 0
 * is the reference hook. Everything runs in fp32 (the GEMMs as fp32 FMA
 * tiles: with N(0,1) weights the softmax is nearly one-hot and magnifies any
 * product error). Scratch: mb_llama_decoder_f32_workspace_bytes,
 * 256-byte aligned, caller owned. */
size_t mb_llama_decoder_f32_workspace_bytes(int B, int S, int D, int H, int H_kv, int FF);
int mb_llama_decoder_f32(const float* x, const float* W_qkv, const float* W_o, const float* W_gu,
                         const float* W_down, float* y, int B, int S, int D, int H, int H_kv,
                         int FF, float rope_base, float eps, int causal, void* workspace,
                         size_t workspace_bytes, void* stream);

/* In-place bf16 sum all-reduce over the tensor-parallel communicator. */
int mb_tp_allreduce_bf16(uint16_t* buf, size_t count, void* stream);

/* ---- standard-set fused ops (mlx/kernels/standard/registry.py:26-42,
 *      103-132, 280-292, 382-396; hooks mlx/kernels/standard/*.py) -------- */

/* y[M,N] = rms_norm(x[M,K]) @ w^T with w [N, K] (rms_norm_linear.py); the
 * norm is a per-row scale of the GEMM epilogue. Workspace: M floats. */
size_t mb_rms_norm_linear_workspace_bytes(int64_t M);
int mb_rms_norm_linear_bf16(const uint16_t* x, const uint16_t* w, uint16_t* y, int64_t M, int64_t K,
                            int64_t N, float eps, void* workspace, size_t workspace_bytes,
                            void* stream);

/* y = rms_norm(x + residual), rows of D (fused_add_rms_norm.py). */
int mb_fused_add_rms_norm_bf16(const uint16_t* x, const uint16_t* residual, uint16_t* y, int64_t M,
                               int64_t D, float eps, void* stream);

/* Interleaved-pair RoPE of [S, D] at positions 0..S-1, omega_i = base^(-2i/D)
 * (rope_embedding.py). */
int mb_rope_bf16(const uint16_t* x, uint16_t* y, int64_t S, int64_t D, float base, void* stream);

/* out[M, FF] = silu(x @ w_gate) * (x @ w_up) (swiglu.py): pack the two
 * (in, out) [D, FF] weights once, then run the fused GEMM. */
size_t mb_swiglu_packed_bytes(int64_t D, int64_t FF);
int mb_swiglu_pack_bf16(const uint16_t* w_gate, const uint16_t* w_up, void* packed, int64_t D,
                        int64_t FF, void* stream);
int mb_swiglu_bf16(const uint16_t* x, const void* packed, uint16_t* out, int64_t M, int64_t D,
                   int64_t FF, void* stream);

/* O[S,128] = softmax(Q K^T / sqrt(128)) V, single head (scaled_dot_product.py). */
size_t mb_sdpa_workspace_bytes(int64_t S);
int mb_sdpa_bf16(const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* O, int64_t S,
                 int64_t d, void* workspace, size_t workspace_bytes, void* stream);

/* out[S, D] = GQA attention of x [S, D] (llama_attention.py:22-63): qkv =
 * x @ W_qkv (W_qkv (in, out) = [D, D + 2*Hkv*128]), per-head interleaved
 * RoPE on q and k at positions 0..S-1 with omega_i = base^(-2i/128), softmax
 * attention over all S keys (non-causal, H query heads sharing Hkv kv heads),
 * then @ W_o [D, D]. Head dim 128 (D = 128*H). */
size_t mb_llama_attention_workspace_bytes(int64_t S, int64_t D, int64_t H, int64_t Hkv);
int mb_llama_attention_bf16(const uint16_t* x, const uint16_t* w_qkv, const uint16_t* w_o,
                            uint16_t* out, int64_t S, int64_t D, int64_t H, int64_t Hkv, float base,
                            void* workspace, size_t workspace_bytes, void* stream);

/* out[S, D] = softmax((x Wq)(x Wk)^T / sqrt(128)) (x Wv) @ Wo per head, heads
 * of 128 (H = D/128), no mask, no RoPE (mlx/kernels/full/mha_attention.py:13-28);
 * all four weights (in, out) = [D, D]. */
size_t mb_mha_attention_workspace_bytes(int64_t S, int64_t D);
int mb_mha_attention_bf16(const uint16_t* x, const uint16_t* wq, const uint16_t* wk,
                          const uint16_t* wv, const uint16_t* wo, uint16_t* out, int64_t S,
                          int64_t D, void* workspace, size_t workspace_bytes, void* stream);

/* Pre-LN transformer block (mlx/kernels/full/transformer_block.py:22-52):
 * x1 = x + MHA(LN(x)) @ W_o with W_qkv [D, 3D], H heads of 128 (D = 128*H);
 * out = x1 + gelu(LN(x1) @ W_ff1) @ W_ff2 with W_ff1 [D, FF], W_ff2 [FF, D].
 * LN has no affine; gelu is the exact x*Phi(x). */
size_t mb_transformer_block_workspace_bytes(int64_t S, int64_t D, int64_t H, int64_t FF);
int mb_transformer_block_bf16(const uint16_t* x, const uint16_t* w_qkv, const uint16_t* w_o,
                              const uint16_t* w_ff1, const uint16_t* w_ff2, uint16_t* out,
                              int64_t S, int64_t D, int64_t H, int64_t FF, float eps,
                              void* workspace, size_t workspace_bytes, void* stream);

/* C[b] = A[b] @ B[b] for b < batch, fp32 row-major contiguous batches
 * (mlx/kernels/common/batch_mm.py:10-11, registry.py:61-77, 131), 3xTF32 like
 * mb_sqr_mm_f32. Workspace: mb_batch_mm_f32_workspace_bytes, 256-byte aligned. */
size_t mb_batch_mm_f32_workspace_bytes(int64_t batch, int64_t M, int64_t N, int64_t K);
int mb_batch_mm_f32(const float* A, const float* B, float* C, int64_t batch, int64_t M, int64_t N,
                    int64_t K, void* workspace, size_t workspace_bytes, void* stream);

/* sqr_mm for callers that cannot allocate device memory. This entry point
 * has no counterpart in the reference. It computes exactly what
 * mb_sqr_mm_f32 computes, but takes its scratch from a 64 MiB array compiled
 * into the library (held on every GPU that loads it, until exit) instead of a
 * caller workspace, and calls no allocator (no cudaMalloc, no torch).
 *  - Shapes whose scratch (mb_sqr_mm_f32_workspace_bytes) exceeds
 *    mb_sqr_mm_f32_noalloc_max_workspace_bytes() are rejected with
 *    MB_ERR_BAD_ARG; 2048^3 fits.
 *  - The first call on a device looks up the array's device address with
 *    cudaGetSymbolAddress, so make it before any stream capture.
 *  - All calls share the one array: calls that overlap on the GPU (different
 *    streams, or other processes' threads on the same context) race and give
 *    wrong results. Serialise them, e.g. on one stream.
 *  - Like the other device-pointer entry points it returns once the work is
 *    queued. A bounded device wait that runs out is reported afterwards by
 *    mb_device_status (non-zero) and cleared by mb_clear_device_status: the
 *    device's shared status word is used when it exists (after mb_init or any
 *    allocating entry point), else a word compiled into the library beside
 *    the scratch array, which mb_device_status also reads. */
size_t mb_sqr_mm_f32_noalloc_max_workspace_bytes(void);
int mb_sqr_mm_f32_noalloc(const float* A, const float* B, float* C, int64_t M, int64_t N,
                          int64_t K, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* MB200_H */
