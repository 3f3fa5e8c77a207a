// Kernel table behind mb_run: binds reference binding indices and scalars to
// the device-pointer entry points. Binding numbers follow the reference
// registry entries (mlx/kernels/common/registry.py, mlx/kernels/full/registry.py).
#include <mutex>
#include <initializer_list>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace mb {
namespace {

int need_buf(const RunArgs& a, int binding, int role, const RunArgs::Buf** out) {
  const RunArgs::Buf* b = a.buf(binding);
  MB_REQUIRE(b != nullptr, "binding %d missing", binding);
  MB_REQUIRE(b->role == role, "binding %d has role %d, expected %d", binding, b->role, role);
  *out = b;
  return MB_OK;
}

int need_scalar(const RunArgs& a, int binding, int64_t* out) {
  double v = 0;
  MB_REQUIRE(a.scalar(binding, &v), "scalar binding %d missing", binding);
  *out = (int64_t)v;
  return MB_OK;
}

#define TRY(x)          \
  do {                  \
    int _rc = (x);      \
    if (_rc) return _rc; \
  } while (0)

// transpose_2d: registry common/registry.py:165-179 — in@0, out@1, rows@2, cols@3.
int prep_transpose_2d(const RunArgs& a, KernelState& st, cudaStream_t) {
  const RunArgs::Buf *in, *out;
  int64_t rows, cols;
  TRY(need_buf(a, 0, MB_ROLE_INPUT, &in));
  TRY(need_buf(a, 1, MB_ROLE_OUTPUT, &out));
  TRY(need_scalar(a, 2, &rows));
  TRY(need_scalar(a, 3, &cols));
  const int esz = in->dtype == MB_BF16 ? 2 : 4;
  MB_REQUIRE(in->dtype == MB_F32 || in->dtype == MB_BF16, "transpose_2d: dtype must be f32 or bf16");
  MB_REQUIRE(in->bytes == (size_t)(rows * cols * esz) && out->bytes == in->bytes,
             "transpose_2d: buffer sizes do not match %lldx%lld", (long long)rows, (long long)cols);
  void* ip = in->dev;
  void* op = out->dev;
  const int dt = in->dtype;
  st.threads_per_cta = 256;
  st.smem_bytes = dt == MB_BF16 ? 16640 : 16384;
  st.launch = [=](cudaStream_t s) {
    return dt == MB_BF16 ? mb_transpose_batched_bf16((const uint16_t*)ip, (uint16_t*)op, 1, rows, cols, s)
                         : mb_transpose_2d_f32((const float*)ip, (float*)op, rows, cols, s);
  };
  return MB_OK;
}

// transpose_batched: in@0 [batch, rows, cols], out@1, batch@2, rows@3, cols@4.
int prep_transpose_batched(const RunArgs& a, KernelState& st, cudaStream_t) {
  const RunArgs::Buf *in, *out;
  int64_t batch, rows, cols;
  TRY(need_buf(a, 0, MB_ROLE_INPUT, &in));
  TRY(need_buf(a, 1, MB_ROLE_OUTPUT, &out));
  TRY(need_scalar(a, 2, &batch));
  TRY(need_scalar(a, 3, &rows));
  TRY(need_scalar(a, 4, &cols));
  MB_REQUIRE(in->dtype == MB_F32 || in->dtype == MB_BF16, "transpose_batched: dtype must be f32 or bf16");
  const int esz = in->dtype == MB_BF16 ? 2 : 4;
  MB_REQUIRE(in->bytes == (size_t)(batch * rows * cols * esz) && out->bytes == in->bytes,
             "transpose_batched: buffer sizes do not match");
  void* ip = in->dev;
  void* op = out->dev;
  const int dt = in->dtype;
  st.threads_per_cta = 256;
  st.smem_bytes = dt == MB_BF16 ? 16640 : 16384;
  st.launch = [=](cudaStream_t s) {
    return dt == MB_BF16
               ? mb_transpose_batched_bf16((const uint16_t*)ip, (uint16_t*)op, batch, rows, cols, s)
               : mb_transpose_batched_f32((const float*)ip, (float*)op, batch, rows, cols, s);
  };
  return MB_OK;
}

// sqr_mm: registry matmul helper common/registry.py:44-61 — A@0, B@1, C@2,
// M@3, N@4, K@5, fp32 row-major.
int prep_sqr_mm(const RunArgs& a, KernelState& st, cudaStream_t) {
  const RunArgs::Buf *A, *B, *Cb;
  int64_t M, N, K;
  TRY(need_buf(a, 0, MB_ROLE_INPUT, &A));
  TRY(need_buf(a, 1, MB_ROLE_INPUT, &B));
  TRY(need_buf(a, 2, MB_ROLE_OUTPUT, &Cb));
  TRY(need_scalar(a, 3, &M));
  TRY(need_scalar(a, 4, &N));
  TRY(need_scalar(a, 5, &K));
  MB_REQUIRE(A->bytes == (size_t)(M * K * 4) && B->bytes == (size_t)(K * N * 4) &&
                 Cb->bytes == (size_t)(M * N * 4),
             "sqr_mm: buffer sizes do not match M=%lld N=%lld K=%lld", (long long)M, (long long)N,
             (long long)K);
  const void *pa = A->dev, *pb = B->dev;
  void* pc = Cb->dev;
  const size_t wsb = mb_sqr_mm_f32_workspace_bytes(M, N, K);
  void* ws = nullptr;
  if (wsb) {
    MB_CUDA(cudaMalloc(&ws, wsb));
    st.scratch.push_back(ws);
  }
  st.threads_per_cta = 256;
  st.smem_bytes = 197752;
  st.launches_per_iter = 3;
  st.launch = [=](cudaStream_t s) {
    return mb_sqr_mm_f32((const float*)pa, (const float*)pb, (float*)pc, M, N, K, ws, wsb, s);
  };
  return MB_OK;
}

// batch_mm: registry batched_matmul helper common/registry.py:61-77 — A@0
// [batch, M, K], B@1 [batch, K, N], C@2 [batch, M, N], M@3, N@4, K@5 (the batch
// count follows from A's size), fp32.
int prep_batch_mm(const RunArgs& a, KernelState& st, cudaStream_t) {
  const RunArgs::Buf *A, *B, *Cb;
  int64_t M, N, K;
  TRY(need_buf(a, 0, MB_ROLE_INPUT, &A));
  TRY(need_buf(a, 1, MB_ROLE_INPUT, &B));
  TRY(need_buf(a, 2, MB_ROLE_OUTPUT, &Cb));
  TRY(need_scalar(a, 3, &M));
  TRY(need_scalar(a, 4, &N));
  TRY(need_scalar(a, 5, &K));
  MB_REQUIRE(M > 0 && K > 0 && A->bytes % (size_t)(M * K * 4) == 0, "batch_mm: A size");
  const int64_t batch = (int64_t)(A->bytes / (size_t)(M * K * 4));
  MB_REQUIRE(B->bytes == (size_t)(batch * K * N * 4) && Cb->bytes == (size_t)(batch * M * N * 4),
             "batch_mm: buffer sizes do not match batch=%lld M=%lld N=%lld K=%lld",
             (long long)batch, (long long)M, (long long)N, (long long)K);
  const void *pa = A->dev, *pb = B->dev;
  void* pc = Cb->dev;
  const size_t wsb = mb_batch_mm_f32_workspace_bytes(batch, M, N, K);
  void* ws = nullptr;
  if (wsb) {
    MB_CUDA(cudaMalloc(&ws, wsb));
    st.scratch.push_back(ws);
  }
  st.threads_per_cta = 256;
  st.smem_bytes = 197752;
  st.launches_per_iter = 3;
  st.launch = [=](cudaStream_t s) {
    return mb_batch_mm_f32((const float*)pa, (const float*)pb, (float*)pc, batch, M, N, K, ws,
                           wsb, s);
  };
  return MB_OK;
}

// gemm_bf16: same bindings with bf16 buffers; config "b_layout" 0/1 (default 1).
int prep_gemm_bf16(const RunArgs& a, KernelState& st, cudaStream_t) {
  const RunArgs::Buf *A, *B, *Cb;
  int64_t M, N, K;
  TRY(need_buf(a, 0, MB_ROLE_INPUT, &A));
  TRY(need_buf(a, 1, MB_ROLE_INPUT, &B));
  TRY(need_buf(a, 2, MB_ROLE_OUTPUT, &Cb));
  TRY(need_scalar(a, 3, &M));
  TRY(need_scalar(a, 4, &N));
  TRY(need_scalar(a, 5, &K));
  MB_REQUIRE(A->bytes == (size_t)(M * K * 2) && B->bytes == (size_t)(K * N * 2) &&
                 Cb->bytes == (size_t)(M * N * 2),
             "gemm_bf16: buffer sizes do not match");
  const int lay = (int)a.config.num("b_layout", 1);
  const void *pa = A->dev, *pb = B->dev;
  void* pc = Cb->dev;
  st.threads_per_cta = 256;
  st.smem_bytes = 197752;
  st.launch = [=](cudaStream_t s) {
    return mb_gemm_bf16((const uint16_t*)pa, (const uint16_t*)pb, (uint16_t*)pc, M, N, K, lay, s);
  };
  return MB_OK;
}

// conv2d: registry common/registry.py:469-477 — x@0, w@1, y@2, N@3, H@4, W@5,
// Cin@6, Cout@7, KH@8, KW@9, stride@10; padding from scalar 11 or config
// "padding" (the reference hook hard-codes 0).
int prep_conv2d(const RunArgs& a, KernelState& st, cudaStream_t) {
  const RunArgs::Buf *x, *w, *y;
  int64_t N, H, W, Ci, Co, KH, KW, stride;
  TRY(need_buf(a, 0, MB_ROLE_INPUT, &x));
  TRY(need_buf(a, 1, MB_ROLE_INPUT, &w));
  TRY(need_buf(a, 2, MB_ROLE_OUTPUT, &y));
  TRY(need_scalar(a, 3, &N));
  TRY(need_scalar(a, 4, &H));
  TRY(need_scalar(a, 5, &W));
  TRY(need_scalar(a, 6, &Ci));
  TRY(need_scalar(a, 7, &Co));
  TRY(need_scalar(a, 8, &KH));
  TRY(need_scalar(a, 9, &KW));
  TRY(need_scalar(a, 10, &stride));
  double padv = a.config.num("padding", 0);
  a.scalar(11, &padv);
  const int64_t pad = (int64_t)padv;
  if (x->dtype == MB_F32) {
    // the reference's own conv2d_f32 entry: fp32 buffers, 3xTF32 products
    MB_REQUIRE(w->dtype == MB_F32 && y->dtype == MB_F32, "conv2d: mixed f32/bf16 buffers");
    MB_REQUIRE(stride >= 1, "conv2d: stride must be >= 1");
    const int64_t H2 = (H + 2 * pad - KH) / stride + 1, W2 = (W + 2 * pad - KW) / stride + 1;
    MB_REQUIRE(x->bytes == (size_t)(N * H * W * Ci * 4) &&
                   w->bytes == (size_t)(Co * KH * KW * Ci * 4) &&
                   y->bytes == (size_t)(N * H2 * W2 * Co * 4),
               "conv2d: buffer sizes do not match the geometry");
    const size_t wsb = mb_conv2d_nhwc_f32_workspace_bytes((int)N, (int)H, (int)W, (int)Ci, (int)Co,
                                                          (int)KH, (int)KW, (int)stride, (int)pad);
    MB_REQUIRE(wsb > 0, "conv2d: unsupported f32 geometry (Cin must be a multiple of 4)");
    void* ws = nullptr;
    MB_CUDA(cudaMalloc(&ws, wsb));
    st.scratch.push_back(ws);
    const void *px = x->dev, *pw = w->dev;
    void* py = y->dev;
    st.threads_per_cta = 256;
    st.launches_per_iter = 3;
    st.launch = [=](cudaStream_t s) {
      return mb_conv2d_nhwc_f32((const float*)px, (const float*)pw, (float*)py, (int)N, (int)H,
                                (int)W, (int)Ci, (int)Co, (int)KH, (int)KW, (int)stride, (int)pad,
                                ws, wsb, s);
    };
    return MB_OK;
  }
  MB_REQUIRE(x->dtype == MB_BF16 && w->dtype == MB_BF16 && y->dtype == MB_BF16,
             "conv2d: buffers must be all bf16 or all f32");
  const int64_t H2 = H + 2 * pad - KH + 1, W2 = W + 2 * pad - KW + 1;
  MB_REQUIRE(x->bytes == (size_t)(N * H * W * Ci * 2) && w->bytes == (size_t)(Co * KH * KW * Ci * 2) &&
                 y->bytes == (size_t)(N * H2 * W2 * Co * 2),
             "conv2d: buffer sizes do not match the geometry");
  const void *px = x->dev, *pw = w->dev;
  void* py = y->dev;
  st.threads_per_cta = 256;
  st.launch = [=](cudaStream_t s) {
    return mb_conv2d_nhwc_bf16((const uint16_t*)px, (const uint16_t*)pw, (uint16_t*)py, (int)N,
                               (int)H, (int)W, (int)Ci, (int)Co, (int)KH, (int)KW, (int)stride,
                               (int)pad, s);
  };
  return MB_OK;
}

// llama_decoder_layer: registry full/registry.py:87-104 — x@0 [B*S, D],
// W_qkv@1, W_o@2, W_gu@3, W_down@4 (bf16, reference (in, out) layout), y@5;
// scalars S@6, D@7, H@8, H_kv@9, FF@10, base@11 (f32), eps@12 (f32).
// Extensions (config): "batch" (B, default 1), "causal" (default 0, as the
// reference hook), "past_len" (cached tokens before x, default 0) with the
// already-rotated cache as optional inputs k_past@13, v_past@14
// [B, H_kv, past_len, 128] bf16. Weight packing and cache set-up happen in
// prepare (untimed); each timed launch is one mb_decoder_layer_forward.
int prep_llama(const RunArgs& a, KernelState& st, cudaStream_t stream) {
  const RunArgs::Buf *x, *wq, *wo, *wg, *wd, *y;
  TRY(need_buf(a, 0, MB_ROLE_INPUT, &x));
  TRY(need_buf(a, 1, MB_ROLE_INPUT, &wq));
  TRY(need_buf(a, 2, MB_ROLE_INPUT, &wo));
  TRY(need_buf(a, 3, MB_ROLE_INPUT, &wg));
  TRY(need_buf(a, 4, MB_ROLE_INPUT, &wd));
  TRY(need_buf(a, 5, MB_ROLE_OUTPUT, &y));
  int64_t S, D, H, Hkv, FF;
  TRY(need_scalar(a, 6, &S));
  TRY(need_scalar(a, 7, &D));
  TRY(need_scalar(a, 8, &H));
  TRY(need_scalar(a, 9, &Hkv));
  TRY(need_scalar(a, 10, &FF));
  double base = 10000.0, eps = 1e-5;
  a.scalar(11, &base);
  a.scalar(12, &eps);
  const int B = (int)a.config.num("batch", 1);
  const int causal = (int)a.config.num("causal", 0);
  const int past = (int)a.config.num("past_len", 0);
  MB_REQUIRE(B >= 1 && S >= 1 && past >= 0, "llama_decoder_layer: bad batch/S/past_len");
  if (x->dtype == MB_F32) {
    // the reference's own llama_decoder_layer_f32 entry: fp32 buffers, any
    // even head_dim <= 256 (the registry's is 32), no KV cache
    for (const RunArgs::Buf* b : {wq, wo, wg, wd, y})
      MB_REQUIRE(b->dtype == MB_F32, "llama_decoder_layer: mixed f32/bf16 buffers");
    MB_REQUIRE(past == 0, "llama_decoder_layer: past_len needs the bf16 path");
    MB_REQUIRE(H > 0 && D % H == 0, "llama_decoder_layer: D must be a multiple of H");
    const int64_t Dh = D / H;
    MB_REQUIRE(x->bytes == (size_t)(B * S * D * 4) && y->bytes == x->bytes,
               "llama_decoder_layer: x/y must be [batch*S, D] f32");
    MB_REQUIRE(wq->bytes == (size_t)(D * (D + 2 * Hkv * Dh) * 4) &&
                   wo->bytes == (size_t)(D * D * 4) && wg->bytes == (size_t)(D * 2 * FF * 4) &&
                   wd->bytes == (size_t)(FF * D * 4),
               "llama_decoder_layer: weight sizes do not match D/H/H_kv/FF");
    const size_t wsb = mb_llama_decoder_f32_workspace_bytes(B, (int)S, (int)D, (int)H, (int)Hkv,
                                                            (int)FF);
    MB_REQUIRE(wsb > 0, "llama_decoder_layer: unsupported f32 geometry (head_dim even <= 256, "
                        "D and FF multiples of 4)");
    void* ws = nullptr;
    MB_CUDA(cudaMalloc(&ws, wsb));
    st.scratch.push_back(ws);
    const float *px = (const float*)x->dev, *pq = (const float*)wq->dev,
                *po = (const float*)wo->dev, *pg = (const float*)wg->dev,
                *pd = (const float*)wd->dev;
    float* py = (float*)y->dev;
    const float fb = (float)base, fe = (float)eps;
    st.threads_per_cta = 256;
    st.launches_per_iter = 0;
    st.launch = [=](cudaStream_t s) {
      return mb_llama_decoder_f32(px, pq, po, pg, pd, py, B, (int)S, (int)D, (int)H, (int)Hkv,
                                  (int)FF, fb, fe, causal, ws, wsb, s);
    };
    return MB_OK;
  }
  for (const RunArgs::Buf* b : {x, wq, wo, wg, wd, y})
    MB_REQUIRE(b->dtype == MB_BF16, "llama_decoder_layer: buffers must be all bf16 or all f32");
  const int Dh = (int)(D / H);
  MB_REQUIRE(x->bytes == (size_t)(B * S * D * 2) && y->bytes == x->bytes,
             "llama_decoder_layer: x/y must be [batch*S, D] bf16");
  MB_REQUIRE(wq->bytes == (size_t)(D * (D + 2 * Hkv * Dh) * 2) && wo->bytes == (size_t)(D * D * 2) &&
                 wg->bytes == (size_t)(D * 2 * FF * 2) && wd->bytes == (size_t)(FF * D * 2),
             "llama_decoder_layer: weight sizes do not match D/H/H_kv/FF");
  mb_decoder_config cfg{(int)D, (int)H, (int)Hkv, Dh, (int)FF, (float)base, (float)eps};
  void* layer = nullptr;
  int rc = mb_decoder_layer_create(&cfg, (const uint16_t*)wq->dev, (const uint16_t*)wo->dev,
                                   (const uint16_t*)wg->dev, (const uint16_t*)wd->dev, 0, 1, &layer);
  if (rc) return rc;
  st.cleanup.push_back([layer] { mb_decoder_layer_destroy(layer); });
  const int kv_total = past + (int)S;
  const int pages = (kv_total + 63) / 64;
  const size_t page_elems = (size_t)Hkv * 64 * Dh;
  auto alloc = [&](size_t bytes, void** p) -> int {
    MB_CUDA(cudaMalloc(p, bytes));
    st.scratch.push_back(*p);
    return MB_OK;
  };
  void *kc, *vc, *bt, *spos, *kvl;
  TRY(alloc((size_t)B * pages * page_elems * 2, &kc));
  TRY(alloc((size_t)B * pages * page_elems * 2, &vc));
  TRY(alloc((size_t)B * pages * 4, &bt));
  TRY(alloc((size_t)B * 4, &spos));
  TRY(alloc((size_t)B * 4, &kvl));
  std::vector<int> h_bt(B * pages), h_sp(B, past), h_kl(B, kv_total);
  for (int i = 0; i < B * pages; ++i) h_bt[i] = i;
  MB_CUDA(cudaMemcpy(bt, h_bt.data(), h_bt.size() * 4, cudaMemcpyHostToDevice));
  MB_CUDA(cudaMemcpy(spos, h_sp.data(), h_sp.size() * 4, cudaMemcpyHostToDevice));
  MB_CUDA(cudaMemcpy(kvl, h_kl.data(), h_kl.size() * 4, cudaMemcpyHostToDevice));
  MB_CUDA(cudaMemset(kc, 0, (size_t)B * pages * page_elems * 2));
  MB_CUDA(cudaMemset(vc, 0, (size_t)B * pages * page_elems * 2));
  if (past > 0) {
    const RunArgs::Buf *kp = a.buf(13), *vp = a.buf(14);
    MB_REQUIRE(kp && vp && kp->bytes == (size_t)B * Hkv * past * Dh * 2 && vp->bytes == kp->bytes,
               "llama_decoder_layer: past_len > 0 needs k_past@13 and v_past@14 [B, H_kv, past_len, Dh]");
    // [B][Hkv][past][Dh] -> pages [b*pages + p][Hkv][64][Dh], one 2-D copy per (b, page)
    for (int b = 0; b < B; ++b)
      for (int p = 0; p * 64 < past; ++p) {
        const int rows = past - p * 64 < 64 ? past - p * 64 : 64;
        const size_t src_off = (((size_t)b * Hkv) * past + (size_t)p * 64) * Dh * 2;
        const size_t dst_off = ((size_t)b * pages + p) * page_elems * 2;
        for (int which = 0; which < 2; ++which) {
          const uint8_t* src = (const uint8_t*)(which ? vp->dev : kp->dev) + src_off;
          uint8_t* dst = (uint8_t*)(which ? vc : kc) + dst_off;
          MB_CUDA(cudaMemcpy2DAsync(dst, (size_t)64 * Dh * 2, src, (size_t)past * Dh * 2,
                                    (size_t)rows * Dh * 2, (size_t)Hkv, cudaMemcpyDeviceToDevice,
                                    stream));
        }
      }
  }
  const size_t wsb = mb_decoder_layer_workspace_bytes(layer, B, (int)S, kv_total);
  void* ws = nullptr;
  TRY(alloc(wsb, &ws));
  MB_CUDA(cudaStreamSynchronize(stream));
  const void* px = x->dev;
  void* py = y->dev;
  st.threads_per_cta = 256;
  st.launches_per_iter = 0;  // several kernels; see the profiles
  st.launch = [=](cudaStream_t s) {
    return mb_decoder_layer_forward(layer, (const uint16_t*)px, (uint16_t*)py, B, (int)S,
                                    (const int*)spos, (const int*)kvl, kv_total, (uint16_t*)kc,
                                    (uint16_t*)vc, (const int*)bt, pages, causal, ws, wsb, s);
  };
  return MB_OK;
}

int bf16_all(const std::initializer_list<const RunArgs::Buf*>& bl, const char* what) {
  for (const RunArgs::Buf* b : bl)
    MB_REQUIRE(b->dtype == MB_BF16, "%s: buffers must be bf16", what);
  return MB_OK;
}

// rms_norm_linear: standard/registry.py:26-42 — x@0 [M,K], w@1 [N,K], y@2;
// M@3, N@4, K@5, eps@6 (f32).
int prep_rms_norm_linear(const RunArgs& a, KernelState& st, cudaStream_t) {
  const RunArgs::Buf *x, *w, *y;
  int64_t M, N, K;
  TRY(need_buf(a, 0, MB_ROLE_INPUT, &x));
  TRY(need_buf(a, 1, MB_ROLE_INPUT, &w));
  TRY(need_buf(a, 2, MB_ROLE_OUTPUT, &y));
  TRY(need_scalar(a, 3, &M));
  TRY(need_scalar(a, 4, &N));
  TRY(need_scalar(a, 5, &K));
  double eps = 1e-5;
  a.scalar(6, &eps);
  TRY(bf16_all({x, w, y}, "rms_norm_linear"));
  MB_REQUIRE(x->bytes == (size_t)(M * K * 2) && w->bytes == (size_t)(N * K * 2) &&
                 y->bytes == (size_t)(M * N * 2),
             "rms_norm_linear: buffer sizes do not match M/N/K");
  const size_t wsb = mb_rms_norm_linear_workspace_bytes(M);
  void* ws = nullptr;
  MB_CUDA(cudaMalloc(&ws, wsb));
  st.scratch.push_back(ws);
  const void *px = x->dev, *pw = w->dev;
  void* py = y->dev;
  st.launches_per_iter = 2;
  st.launch = [=](cudaStream_t s) {
    return mb_rms_norm_linear_bf16((const uint16_t*)px, (const uint16_t*)pw, (uint16_t*)py, M, K,
                                   N, (float)eps, ws, wsb, s);
  };
  return MB_OK;
}

// fused_add_rms_norm: standard/registry.py:280-292 — x@0, residual@1, y@2;
// D@3, eps@4 (f32); rows = size / D.
int prep_add_rms_norm(const RunArgs& a, KernelState& st, cudaStream_t) {
  const RunArgs::Buf *x, *r, *y;
  int64_t D;
  TRY(need_buf(a, 0, MB_ROLE_INPUT, &x));
  TRY(need_buf(a, 1, MB_ROLE_INPUT, &r));
  TRY(need_buf(a, 2, MB_ROLE_OUTPUT, &y));
  TRY(need_scalar(a, 3, &D));
  double eps = 1e-5;
  a.scalar(4, &eps);
  TRY(bf16_all({x, r, y}, "fused_add_rms_norm"));
  MB_REQUIRE(D > 0 && x->bytes % (size_t)(D * 2) == 0 && r->bytes == x->bytes &&
                 y->bytes == x->bytes,
             "fused_add_rms_norm: buffer sizes do not match D");
  const int64_t M = (int64_t)(x->bytes / (D * 2));
  const void *px = x->dev, *pr = r->dev;
  void* py = y->dev;
  st.launch = [=](cudaStream_t s) {
    return mb_fused_add_rms_norm_bf16((const uint16_t*)px, (const uint16_t*)pr, (uint16_t*)py, M,
                                      D, (float)eps, s);
  };
  return MB_OK;
}

// rope_embedding: standard/registry.py:103-116 — x@0 [S,D], y@1; S@2, D@3, base@4.
int prep_rope(const RunArgs& a, KernelState& st, cudaStream_t) {
  const RunArgs::Buf *x, *y;
  int64_t S, D;
  TRY(need_buf(a, 0, MB_ROLE_INPUT, &x));
  TRY(need_buf(a, 1, MB_ROLE_OUTPUT, &y));
  TRY(need_scalar(a, 2, &S));
  TRY(need_scalar(a, 3, &D));
  double base = 10000.0;
  a.scalar(4, &base);
  TRY(bf16_all({x, y}, "rope_embedding"));
  MB_REQUIRE(x->bytes == (size_t)(S * D * 2) && y->bytes == x->bytes,
             "rope_embedding: buffer sizes do not match S/D");
  const void* px = x->dev;
  void* py = y->dev;
  st.launch = [=](cudaStream_t s) {
    return mb_rope_bf16((const uint16_t*)px, (uint16_t*)py, S, D, (float)base, s);
  };
  return MB_OK;
}

// swiglu: standard/registry.py:119-132 — x@0 [M,D], w_gate@1 [D,FF], w_up@2,
// out@3 [M,FF]; M@4, D@5, FF@6. The weights are packed in prepare (untimed).
int prep_swiglu(const RunArgs& a, KernelState& st, cudaStream_t stream) {
  const RunArgs::Buf *x, *wg, *wu, *y;
  int64_t M, D, FF;
  TRY(need_buf(a, 0, MB_ROLE_INPUT, &x));
  TRY(need_buf(a, 1, MB_ROLE_INPUT, &wg));
  TRY(need_buf(a, 2, MB_ROLE_INPUT, &wu));
  TRY(need_buf(a, 3, MB_ROLE_OUTPUT, &y));
  TRY(need_scalar(a, 4, &M));
  TRY(need_scalar(a, 5, &D));
  TRY(need_scalar(a, 6, &FF));
  TRY(bf16_all({x, wg, wu, y}, "swiglu"));
  MB_REQUIRE(x->bytes == (size_t)(M * D * 2) && wg->bytes == (size_t)(D * FF * 2) &&
                 wu->bytes == wg->bytes && y->bytes == (size_t)(M * FF * 2),
             "swiglu: buffer sizes do not match M/D/FF");
  const size_t pb = mb_swiglu_packed_bytes(D, FF);
  void* packed = nullptr;
  MB_CUDA(cudaMalloc(&packed, pb));
  st.scratch.push_back(packed);
  TRY(mb_swiglu_pack_bf16((const uint16_t*)wg->dev, (const uint16_t*)wu->dev, packed, D, FF,
                          stream));
  MB_CUDA(cudaStreamSynchronize(stream));
  const void* px = x->dev;
  void* py = y->dev;
  st.threads_per_cta = 256;
  st.launch = [=](cudaStream_t s) {
    return mb_swiglu_bf16((const uint16_t*)px, packed, (uint16_t*)py, M, D, FF, s);
  };
  return MB_OK;
}

// scaled_dot_product: standard/registry.py:382-396 — Q@0, K@1, V@2 [S,d], O@3;
// S@4, d@5.
int prep_sdpa(const RunArgs& a, KernelState& st, cudaStream_t) {
  const RunArgs::Buf *q, *k, *v, *o;
  int64_t S, d;
  TRY(need_buf(a, 0, MB_ROLE_INPUT, &q));
  TRY(need_buf(a, 1, MB_ROLE_INPUT, &k));
  TRY(need_buf(a, 2, MB_ROLE_INPUT, &v));
  TRY(need_buf(a, 3, MB_ROLE_OUTPUT, &o));
  TRY(need_scalar(a, 4, &S));
  TRY(need_scalar(a, 5, &d));
  TRY(bf16_all({q, k, v, o}, "scaled_dot_product"));
  MB_REQUIRE(q->bytes == (size_t)(S * d * 2) && k->bytes == q->bytes && v->bytes == q->bytes &&
                 o->bytes == q->bytes,
             "scaled_dot_product: buffer sizes do not match S/d");
  const size_t wsb = mb_sdpa_workspace_bytes(S);
  void* ws = nullptr;
  MB_CUDA(cudaMalloc(&ws, wsb));
  st.scratch.push_back(ws);
  const void *pq = q->dev, *pk = k->dev, *pv = v->dev;
  void* po = o->dev;
  st.launches_per_iter = 2;
  st.launch = [=](cudaStream_t s) {
    return mb_sdpa_bf16((const uint16_t*)pq, (const uint16_t*)pk, (const uint16_t*)pv,
                        (uint16_t*)po, S, d, ws, wsb, s);
  };
  return MB_OK;
}

// llama_attention: standard/registry.py:398-413 — x@0 [S, D], W_qkv@1
// [D, D + 2*Hkv*Dh], W_o@2 [D, D], out@3; S@4, D@5, H@6, H_kv@7, base@8 (f32).
int prep_llama_attention(const RunArgs& a, KernelState& st, cudaStream_t) {
  const RunArgs::Buf *x, *wqkv, *wo, *o;
  int64_t S, D, H, Hkv;
  TRY(need_buf(a, 0, MB_ROLE_INPUT, &x));
  TRY(need_buf(a, 1, MB_ROLE_INPUT, &wqkv));
  TRY(need_buf(a, 2, MB_ROLE_INPUT, &wo));
  TRY(need_buf(a, 3, MB_ROLE_OUTPUT, &o));
  TRY(need_scalar(a, 4, &S));
  TRY(need_scalar(a, 5, &D));
  TRY(need_scalar(a, 6, &H));
  TRY(need_scalar(a, 7, &Hkv));
  double base = 10000.0;
  a.scalar(8, &base);
  TRY(bf16_all({x, wqkv, wo, o}, "llama_attention"));
  MB_REQUIRE(H > 0 && D == 128 * H, "llama_attention: head dim must be 128 (D = 128*H)");
  MB_REQUIRE(x->bytes == (size_t)(S * D * 2) && o->bytes == x->bytes &&
                 wqkv->bytes == (size_t)(D * (D + 2 * Hkv * 128) * 2) &&
                 wo->bytes == (size_t)(D * D * 2),
             "llama_attention: buffer sizes do not match S/D/H_kv");
  const size_t wsb = mb_llama_attention_workspace_bytes(S, D, H, Hkv);
  void* ws = nullptr;
  MB_CUDA(cudaMalloc(&ws, wsb));
  st.scratch.push_back(ws);
  const void *px = x->dev, *pq = wqkv->dev, *pw = wo->dev;
  void* po = o->dev;
  const float fb = (float)base;
  st.launches_per_iter = 5;
  st.launch = [=](cudaStream_t s) {
    return mb_llama_attention_bf16((const uint16_t*)px, (const uint16_t*)pq, (const uint16_t*)pw,
                                   (uint16_t*)po, S, D, H, Hkv, fb, ws, wsb, s);
  };
  return MB_OK;
}

// mha_attention: full/registry.py:107-130 — x@0 [S, D], wq@1, wk@2, wv@3,
// wo@4 [D, D], out@5; S@6, D@7, H@8, Dh@9, scale@10. Heads of 128: H = D/128.
int prep_mha(const RunArgs& a, KernelState& st, cudaStream_t) {
  const RunArgs::Buf *x, *wq, *wk, *wv, *wo, *o;
  int64_t S, D, H = 0;
  TRY(need_buf(a, 0, MB_ROLE_INPUT, &x));
  TRY(need_buf(a, 1, MB_ROLE_INPUT, &wq));
  TRY(need_buf(a, 2, MB_ROLE_INPUT, &wk));
  TRY(need_buf(a, 3, MB_ROLE_INPUT, &wv));
  TRY(need_buf(a, 4, MB_ROLE_INPUT, &wo));
  TRY(need_buf(a, 5, MB_ROLE_OUTPUT, &o));
  TRY(need_scalar(a, 6, &S));
  TRY(need_scalar(a, 7, &D));
  TRY(bf16_all({x, wq, wk, wv, wo, o}, "mha_attention"));
  double h = 0;
  if (a.scalar(8, &h)) H = (int64_t)h;
  MB_REQUIRE(D % 128 == 0 && (H == 0 || H == D / 128),
             "mha_attention: heads of 128 required (H = D/128)");
  MB_REQUIRE(x->bytes == (size_t)(S * D * 2) && o->bytes == x->bytes &&
                 wq->bytes == (size_t)(D * D * 2) && wk->bytes == wq->bytes &&
                 wv->bytes == wq->bytes && wo->bytes == wq->bytes,
             "mha_attention: buffer sizes do not match S/D");
  const size_t wsb = mb_mha_attention_workspace_bytes(S, D);
  void* ws = nullptr;
  MB_CUDA(cudaMalloc(&ws, wsb));
  st.scratch.push_back(ws);
  const void *px = x->dev, *pq = wq->dev, *pk = wk->dev, *pv = wv->dev, *pw = wo->dev;
  void* po = o->dev;
  st.launches_per_iter = 7;
  st.launch = [=](cudaStream_t s) {
    return mb_mha_attention_bf16((const uint16_t*)px, (const uint16_t*)pq, (const uint16_t*)pk,
                                 (const uint16_t*)pv, (const uint16_t*)pw, (uint16_t*)po, S, D,
                                 ws, wsb, s);
  };
  return MB_OK;
}

// transformer_block: full/registry.py:47-62 — x@0 [S, D], W_qkv@1 [D, 3D],
// W_o@2 [D, D], W_ff1@3 [D, FF], W_ff2@4 [FF, D], out@5; S@6, D@7, H@8, FF@9,
// eps@10 (f32).
int prep_transformer_block(const RunArgs& a, KernelState& st, cudaStream_t) {
  const RunArgs::Buf *x, *wqkv, *wo, *w1, *w2, *o;
  int64_t S, D, H, FF;
  TRY(need_buf(a, 0, MB_ROLE_INPUT, &x));
  TRY(need_buf(a, 1, MB_ROLE_INPUT, &wqkv));
  TRY(need_buf(a, 2, MB_ROLE_INPUT, &wo));
  TRY(need_buf(a, 3, MB_ROLE_INPUT, &w1));
  TRY(need_buf(a, 4, MB_ROLE_INPUT, &w2));
  TRY(need_buf(a, 5, MB_ROLE_OUTPUT, &o));
  TRY(need_scalar(a, 6, &S));
  TRY(need_scalar(a, 7, &D));
  TRY(need_scalar(a, 8, &H));
  TRY(need_scalar(a, 9, &FF));
  double eps = 1e-5;
  a.scalar(10, &eps);
  TRY(bf16_all({x, wqkv, wo, w1, w2, o}, "transformer_block"));
  MB_REQUIRE(H > 0 && D == 128 * H, "transformer_block: heads of 128 required (D = 128*H)");
  MB_REQUIRE(x->bytes == (size_t)(S * D * 2) && o->bytes == x->bytes &&
                 wqkv->bytes == (size_t)(3 * D * D * 2) && wo->bytes == (size_t)(D * D * 2) &&
                 w1->bytes == (size_t)(D * FF * 2) && w2->bytes == w1->bytes,
             "transformer_block: buffer sizes do not match S/D/FF");
  const size_t wsb = mb_transformer_block_workspace_bytes(S, D, H, FF);
  void* ws = nullptr;
  MB_CUDA(cudaMalloc(&ws, wsb));
  st.scratch.push_back(ws);
  const void *px = x->dev, *p1 = wqkv->dev, *p2 = wo->dev, *p3 = w1->dev, *p4 = w2->dev;
  void* po = o->dev;
  const float fe = (float)eps;
  st.launches_per_iter = 10;
  st.launch = [=](cudaStream_t s) {
    return mb_transformer_block_bf16((const uint16_t*)px, (const uint16_t*)p1,
                                     (const uint16_t*)p2, (const uint16_t*)p3,
                                     (const uint16_t*)p4, (uint16_t*)po, S, D, H, FF, fe, ws, wsb,
                                     s);
  };
  return MB_OK;
}

}  // namespace

void register_all_kernels() {
  static std::once_flag once;
  std::call_once(once, [] {
    register_kernel({"transpose_2d", prep_transpose_2d});
    register_kernel({"transpose_batched", prep_transpose_batched});
    register_kernel({"sqr_mm", prep_sqr_mm});
    register_kernel({"batch_mm", prep_batch_mm});
    register_kernel({"gemm_bf16", prep_gemm_bf16});
    register_kernel({"conv2d", prep_conv2d});
    register_kernel({"llama_decoder_layer", prep_llama});
    register_kernel({"rms_norm_linear", prep_rms_norm_linear});
    register_kernel({"fused_add_rms_norm", prep_add_rms_norm});
    register_kernel({"rope_embedding", prep_rope});
    register_kernel({"swiglu", prep_swiglu});
    register_kernel({"scaled_dot_product", prep_sdpa});
    register_kernel({"llama_attention", prep_llama_attention});
    register_kernel({"mha_attention", prep_mha});
    register_kernel({"transformer_block", prep_transformer_block});
  });
}

}  // namespace mb
