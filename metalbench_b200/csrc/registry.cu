// Kernel table behind mb_run: binds reference binding indices and scalars to
// the device-pointer entry points. Binding numbers follow the reference
// registry entries (mlx/kernels/common/registry.py, mlx/kernels/full/registry.py).
#include <mutex>

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
  MB_REQUIRE(x->dtype == MB_BF16 && w->dtype == MB_BF16 && y->dtype == MB_BF16,
             "conv2d: buffers must be bf16");
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

}  // namespace

void register_all_kernels() {
  static std::once_flag once;
  std::call_once(once, [] {
    register_kernel({"transpose_2d", prep_transpose_2d});
    register_kernel({"transpose_batched", prep_transpose_batched});
    register_kernel({"sqr_mm", prep_sqr_mm});
    register_kernel({"gemm_bf16", prep_gemm_bf16});
    register_kernel({"conv2d", prep_conv2d});
  });
}

}  // namespace mb
