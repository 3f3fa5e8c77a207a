// Plain GEMM entry points on the tcgen05 core:
//   mb_gemm_bf16  C(bf16) = A(bf16) @ B(bf16), fp32 accumulate in TMEM
//   mb_sqr_mm_f32 C(fp32) = A(fp32) @ B(fp32) with 3xTF32 (fp32-accurate)
//
// Reference: mlx/kernels/common/sqr_mm.py:10-11 (mx.matmul) and the registry
// matmul helper mlx/kernels/common/registry.py:44-61 (row-major A [M,K],
// B [K,N], C [M,N]); the Metal kernel metal/kernels/common/sqr_mm.metal:19-111
// is a 64x64x16 simdgroup-MMA tile loop that this replaces.
#include <mutex>

#include "gemm_core.cuh"
#include "gemm_epi.cuh"
#include "gemm_launch.cuh"

using namespace gemm;

namespace mb {
int gemm_bf16_ex(const uint16_t* A, const uint16_t* B, uint16_t* C, int64_t M, int64_t N,
                 int64_t K, int64_t ldc, int b_layout, const uint16_t* residual, int64_t ld_res,
                 int act, cudaStream_t s) {
  gemm::Epi<256, gemm::EpiStore> e{};
  e.M = (int)M;
  e.N = (int)N;
  e.out = C;
  e.ldo = ldc;
  e.alpha = 1.f;
  e.residual = residual;
  e.ld_res = ld_res;
  e.act = act;
  if (b_layout == 0) return launch_gemm<gemm::Mode::BF16, 256, 4, false>(A, B, e, M, N, K, 1, s);
  return launch_gemm<gemm::Mode::BF16, 256, 4, true>(A, B, e, M, N, K, 1, s);
}
}  // namespace mb

extern "C" int mb_gemm_bf16(const uint16_t* A, const uint16_t* B, uint16_t* C, int64_t M,
                            int64_t N, int64_t K, int b_layout, void* stream) {
  MB_REQUIRE(M >= 0 && N >= 0 && K >= 0, "mb_gemm_bf16: negative dimension");
  MB_REQUIRE(b_layout == 0 || b_layout == 1, "mb_gemm_bf16: b_layout must be 0 ([N,K]) or 1 ([K,N])");
  if (M == 0 || N == 0) return MB_OK;
  MB_REQUIRE(K > 0, "mb_gemm_bf16: K must be positive");
  MB_REQUIRE(N % 8 == 0, "mb_gemm_bf16: N must be a multiple of 8");
  return mb::gemm_bf16_ex(A, B, C, M, N, K, N, b_layout, nullptr, 0, 0,
                          static_cast<cudaStream_t>(stream));
}

// k-blocks (32 fp32 of K each) per tensor-core partial sum of the 3xTF32
// GEMM; the partial sums are added in fp32 registers (gemm_kernel PROMOTE).
constexpr int kTf32PromoteBlocks = 4;

namespace {

// tf32 "hi" = the fp32 value with its low 13 mantissa bits cleared (exactly
// representable in tf32, so the tensor core sees it unchanged); "lo" = the
// exact fp32 remainder x - hi.
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  lo = x - hi;
}

// A [M,K] -> A_hi, A_lo (same row-major layout), 16 bytes per thread step.
__global__ void split_a_kernel(const float4* __restrict__ a, float4* __restrict__ hi,
                               float4* __restrict__ lo, int64_t n4) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float4 x = a[i];
    float4 h, l;
    split_tf32(x.x, h.x, l.x);
    split_tf32(x.y, h.y, l.y);
    split_tf32(x.z, h.z, l.z);
    split_tf32(x.w, h.w, l.w);
    hi[i] = h;
    lo[i] = l;
  }
}

// B [K,N] -> Bt_hi, Bt_lo [N,K] (transposed so both GEMM operands are K-major);
// blockIdx.z = batch (strides K*N). 64 x 64 tiles through a padded shared
// tile: 16-byte loads along N and 16-byte stores along K when K and N are
// multiples of 4 (else element by element).
__global__ void __launch_bounds__(256) split_bt_kernel(const float* __restrict__ b,
                                                       float* __restrict__ hi,
                                                       float* __restrict__ lo, int64_t K,
                                                       int64_t N) {
  __shared__ float T[64][65];
  const int64_t z = blockIdx.z;
  b += z * K * N;
  hi += z * K * N;
  lo += z * K * N;
  const int64_t k0 = (int64_t)blockIdx.y * 64, n0 = (int64_t)blockIdx.x * 64;
  const bool vec = (K % 4 == 0) && (N % 4 == 0) && k0 + 64 <= K && n0 + 64 <= N;
  if (vec) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {  // 64 rows x 16 float4
      const int idx = threadIdx.x + i * 256, r = idx >> 4, c4 = (idx & 15) * 4;
      const float4 v = *reinterpret_cast<const float4*>(b + (k0 + r) * N + n0 + c4);
      T[r][c4] = v.x;
      T[r][c4 + 1] = v.y;
      T[r][c4 + 2] = v.z;
      T[r][c4 + 3] = v.w;
    }
  } else {
    for (int idx = threadIdx.x; idx < 64 * 64; idx += 256) {
      const int r = idx >> 6, c = idx & 63;
      if (k0 + r < K && n0 + c < N) T[r][c] = b[(k0 + r) * N + n0 + c];
    }
  }
  __syncthreads();
  if (vec) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {  // 64 output rows (n) x 16 float4 along k, 256 B per row
      const int idx = threadIdx.x + i * 256, n = idx >> 4, k4 = (idx & 15) * 4;
      float4 h, l;
      split_tf32(T[k4][n], h.x, l.x);
      split_tf32(T[k4 + 1][n], h.y, l.y);
      split_tf32(T[k4 + 2][n], h.z, l.z);
      split_tf32(T[k4 + 3][n], h.w, l.w);
      *reinterpret_cast<float4*>(hi + (n0 + n) * K + k0 + k4) = h;
      *reinterpret_cast<float4*>(lo + (n0 + n) * K + k0 + k4) = l;
    }
  } else {
    for (int idx = threadIdx.x; idx < 64 * 64; idx += 256) {
      const int n = idx >> 6, k = idx & 63;
      if (n0 + n < N && k0 + k < K) {
        float h, l;
        split_tf32(T[k][n], h, l);
        hi[(n0 + n) * K + k0 + k] = h;
        lo[(n0 + n) * K + k0 + k] = l;
      }
    }
  }
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

size_t tf32x3_workspace(int64_t batch, int64_t M, int64_t N, int64_t K) {
  return 2 * align256((size_t)batch * M * K * 4) + 2 * align256((size_t)batch * N * K * 4);
}

}  // namespace

namespace mb {

int tf32x3_split_rows(const float* src, float* hi, float* lo, int64_t n, cudaStream_t s) {
  MB_REQUIRE(n % 4 == 0, "tf32x3 split: element count must be a multiple of 4");
  MB_REQUIRE(reinterpret_cast<uintptr_t>(src) % 16 == 0, "tf32x3 split: source must be 16-byte aligned");
  if (n == 0) return MB_OK;
  const int sms = mb::num_sms();
  split_a_kernel<<<sms * 8, 256, 0, s>>>(reinterpret_cast<const float4*>(src),
                                         reinterpret_cast<float4*>(hi),
                                         reinterpret_cast<float4*>(lo), n / 4);
  MB_CUDA(cudaGetLastError());
  return MB_OK;
}

// C[b] = A[b] @ B[b] for b < batch from operands split already: A_hi/A_lo
// [batch*M, K] and B_hi/B_lo [batch*N, K], both K-major. M % 128 == 0 when
// batch > 1, so no 128-row tile straddles two batches; B rows of batch b
// start at b*N (GemmProducer::b_rows_per_batch).
int tf32x3_core(const float* a_hi, const float* a_lo, const float* b_hi, const float* b_lo,
                float* C, int64_t batch, int64_t M, int64_t N, int64_t K, uint32_t* status,
                cudaStream_t s) {
  const int sms = mb::num_sms();
  using P = GemmProducer<Mode::TF32X3, 128, false>;
  using S = Smem<P, 128, 3>;
  gemm::Epi<128, gemm::EpiStore> e{};
  e.M = (int)(batch * M);
  e.N = (int)N;
  e.out = C;
  e.ldo = N;
  e.out_f32 = 1;
  e.alpha = 1.f;
  P p;
  if (batch > 1) {
    p.a_tiles_per_batch = (int)(M / BM);
    p.b_rows_per_batch = (int)N;
  }
  const auto dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const auto sw = CU_TENSOR_MAP_SWIZZLE_128B;
  const int64_t rows_a = batch * M, rows_b = batch * N;
  int rc = mb::make_tmap_2d(&p.a, a_hi, dt, 4, K, rows_a, K * 4, P::KE, BM, sw);
  if (!rc) rc = mb::make_tmap_2d(&p.alo, a_lo, dt, 4, K, rows_a, K * 4, P::KE, BM, sw);
  if (!rc) rc = mb::make_tmap_2d(&p.b, b_hi, dt, 4, K, rows_b, K * 4, P::KE, 128, sw);
  if (!rc) rc = mb::make_tmap_2d(&p.blo, b_lo, dt, 4, K, rows_b, K * 4, P::KE, 128, sw);
  if (rc) return rc;
  Sched sc;
  sc.tiles_m = (int)((batch * M + BM - 1) / BM);
  sc.tiles_n = (int)((N + 127) / 128);
  sc.kblocks = (int)((K + P::KE - 1) / P::KE);
  sc.ksplit = 1;
  sc.kb_per_split = sc.kblocks;
  auto kern = gemm_kernel<128, 3, P, decltype(e), kTf32PromoteBlocks>;
  {
    const int arc = mb::ensure_smem_attr(reinterpret_cast<const void*>(kern), S::TOTAL);
    if (arc) return arc;
  }
  const int grid = sc.total() < sms ? sc.total() : sms;
  kern<<<grid, 256, S::TOTAL, s>>>(p, e, sc, status);
  MB_CUDA(cudaGetLastError());
  return MB_OK;
}

}  // namespace mb

namespace {

// C[b] = A[b] @ B[b] for b < batch (row-major, contiguous batches) with
// 3xTF32: split prepass into the workspace (B transposed to K-major), then
// one persistent GEMM launch whose tile rows run over all batches.
int tf32x3_gemm(const float* A, const float* B, float* C, int64_t batch, int64_t M, int64_t N,
                int64_t K, uint8_t* w, uint32_t* status, cudaStream_t s) {
  float* a_hi = reinterpret_cast<float*>(w);
  float* a_lo = reinterpret_cast<float*>(w + align256((size_t)batch * M * K * 4));
  float* b_hi = reinterpret_cast<float*>(w + 2 * align256((size_t)batch * M * K * 4));
  float* b_lo = reinterpret_cast<float*>(w + 2 * align256((size_t)batch * M * K * 4) +
                                         align256((size_t)batch * N * K * 4));
  int rc = mb::tf32x3_split_rows(A, a_hi, a_lo, batch * M * K, s);
  if (rc) return rc;
  dim3 g((unsigned)((N + 63) / 64), (unsigned)((K + 63) / 64), (unsigned)batch);
  MB_REQUIRE(g.y <= 65535 && g.z <= 65535, "tf32x3: K or batch too large");
  split_bt_kernel<<<g, 256, 0, s>>>(B, b_hi, b_lo, K, N);
  MB_CUDA(cudaGetLastError());
  return mb::tf32x3_core(a_hi, a_lo, b_hi, b_lo, C, batch, M, N, K, status, s);
}

int check_tf32x3_args(const char* fn, const float* A, int64_t batch, int64_t M, int64_t N,
                      int64_t K) {
  MB_REQUIRE(batch >= 0 && M >= 0 && N >= 0 && K >= 0, "%s: negative dimension", fn);
  if (batch == 0 || M == 0 || N == 0) return MB_OK;
  MB_REQUIRE(K > 0, "%s: K must be positive", fn);
  MB_REQUIRE(K % 4 == 0, "%s: K must be a multiple of 4", fn);
  MB_REQUIRE(reinterpret_cast<uintptr_t>(A) % 16 == 0, "%s: A must be 16-byte aligned", fn);
  return MB_OK;
}

}  // namespace

extern "C" size_t mb_sqr_mm_f32_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  return tf32x3_workspace(1, M, N, K);
}

extern "C" int mb_sqr_mm_f32(const float* A, const float* B, float* C, int64_t M, int64_t N,
                             int64_t K, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_tf32x3_args("mb_sqr_mm_f32", A, 1, M, N, K);
  if (rc || M == 0 || N == 0) return rc;
  const size_t need = mb_sqr_mm_f32_workspace_bytes(M, N, K);
  MB_REQUIRE(workspace != nullptr && workspace_bytes >= need &&
                 reinterpret_cast<uintptr_t>(workspace) % 256 == 0,
             "mb_sqr_mm_f32: workspace of %zu bytes (256-byte aligned) required, got %zu", need,
             workspace_bytes);
  return tf32x3_gemm(A, B, C, 1, M, N, K, static_cast<uint8_t*>(workspace),
                     mb::device_status_ptr(), static_cast<cudaStream_t>(stream));
}

extern "C" size_t mb_batch_mm_f32_workspace_bytes(int64_t batch, int64_t M, int64_t N,
                                                  int64_t K) {
  if (batch <= 0 || M <= 0 || N <= 0 || K <= 0) return 0;
  // one launch over all batches when M is a whole number of 128-row tiles,
  // else batch-by-batch through one batch's workspace
  return M % BM == 0 ? tf32x3_workspace(batch, M, N, K) : tf32x3_workspace(1, M, N, K);
}

extern "C" int mb_batch_mm_f32(const float* A, const float* B, float* C, int64_t batch, int64_t M,
                               int64_t N, int64_t K, void* workspace, size_t workspace_bytes,
                               void* stream) {
  int rc = check_tf32x3_args("mb_batch_mm_f32", A, batch, M, N, K);
  if (rc || batch == 0 || M == 0 || N == 0) return rc;
  const size_t need = mb_batch_mm_f32_workspace_bytes(batch, M, N, K);
  MB_REQUIRE(workspace != nullptr && workspace_bytes >= need &&
                 reinterpret_cast<uintptr_t>(workspace) % 256 == 0,
             "mb_batch_mm_f32: workspace of %zu bytes (256-byte aligned) required, got %zu", need,
             workspace_bytes);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M % BM == 0) return tf32x3_gemm(A, B, C, batch, M, N, K, w, mb::device_status_ptr(), s);
  MB_REQUIRE(((M * K) % 4) == 0, "mb_batch_mm_f32: M*K must be a multiple of 4");
  for (int64_t b = 0; b < batch; ++b) {
    rc = tf32x3_gemm(A + b * M * K, B + b * K * N, C + b * M * N, 1, M, N, K, w,
                     mb::device_status_ptr(), s);
    if (rc) return rc;
  }
  return MB_OK;
}

// ---------------------------------------------------------------------------
// sqr_mm without any allocation.
//
// Some callers cannot allocate device memory at all: a plugin that runs
// inside a host process which owns every allocation (a custom allocator or
// a memory pool it must not bypass), or code that must not call cudaMalloc
// because an allocation would synchronise the device or fail under a memory
// cap. They still need the scratch that mb_sqr_mm_f32 takes as `workspace`.
// This entry point takes it from a fixed array compiled into the library
// instead: every GPU that loads libmb200.so holds these 64 MiB until the
// process exits.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;  // 64 MiB: enough for 2048^3
static __device__ __align__(256) uint8_t g_sqr_mm_scratch[kNoAllocScratchBytes];
static __device__ uint32_t g_sqr_mm_scratch_status;

// Device addresses of the two arrays, looked up once per device (the names
// are host-side stand-ins, never device addresses).
struct NoAllocSlot {
  void* scratch = nullptr;
  uint32_t* status = nullptr;
};
constexpr int kMaxDevices = 64;
NoAllocSlot g_noalloc[kMaxDevices];
std::mutex g_noalloc_mu;

int noalloc_setup(int dev, NoAllocSlot* out) {
  MB_REQUIRE(dev >= 0 && dev < kMaxDevices, "mb_sqr_mm_f32_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoAllocSlot& s = g_noalloc[dev];
  if (!s.scratch) {
    void* p = nullptr;
    void* q = nullptr;
    MB_CUDA(cudaGetSymbolAddress(&p, g_sqr_mm_scratch));
    MB_CUDA(cudaGetSymbolAddress(&q, g_sqr_mm_scratch_status));
    s.status = static_cast<uint32_t*>(q);
    s.scratch = p;
  }
  *out = s;
  return MB_OK;
}

}  // namespace

namespace mb {
int noalloc_status(uint32_t* out, bool clear) {
  *out = 0;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MB_OK;
  uint32_t* st = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    st = g_noalloc[dev].status;
  }
  if (!st) return MB_OK;  // the entry point never ran on this device
  MB_CUDA(cudaDeviceSynchronize());
  MB_CUDA(cudaMemcpy(out, st, sizeof(uint32_t), cudaMemcpyDeviceToHost));
  if (clear) MB_CUDA(cudaMemset(st, 0, sizeof(uint32_t)));
  return MB_OK;
}
}  // namespace mb

extern "C" size_t mb_sqr_mm_f32_noalloc_max_workspace_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int mb_sqr_mm_f32_noalloc(const float* A, const float* B, float* C, int64_t M,
                                     int64_t N, int64_t K, void* stream) {
  MB_REQUIRE(M >= 0 && N >= 0 && K >= 0, "mb_sqr_mm_f32_noalloc: negative dimension");
  if (M == 0 || N == 0) return MB_OK;
  MB_REQUIRE(K > 0 && K % 4 == 0, "mb_sqr_mm_f32_noalloc: K must be a positive multiple of 4");
  MB_REQUIRE(reinterpret_cast<uintptr_t>(A) % 16 == 0,
             "mb_sqr_mm_f32_noalloc: A must be 16-byte aligned");
  const size_t need = mb_sqr_mm_f32_workspace_bytes(M, N, K);
  MB_REQUIRE(need <= kNoAllocScratchBytes,
             "mb_sqr_mm_f32_noalloc: M=%lld N=%lld K=%lld needs %zu bytes of scratch, more than "
             "the fixed %zu-byte array; use mb_sqr_mm_f32 with a caller workspace",
             (long long)M, (long long)N, (long long)K, need, kNoAllocScratchBytes);
  int dev = 0;
  MB_CUDA(cudaGetDevice(&dev));
  NoAllocSlot slot;
  int rc = noalloc_setup(dev, &slot);
  if (rc) return rc;
  // Bounded-wait timeouts go to the device's shared status word when mb_init
  // (or any other entry point) created it, else to the array-backed word;
  // mb_device_status reports both, mb_clear_device_status clears both.
  uint32_t* status = mb::existing_device_status_ptr();
  if (!status) status = slot.status;

  // The split prepass overwrites every scratch byte the GEMM reads, so nothing
  // has to be cleared first.
  return tf32x3_gemm(A, B, C, 1, M, N, K, static_cast<uint8_t*>(slot.scratch), status,
                     static_cast<cudaStream_t>(stream));
}
