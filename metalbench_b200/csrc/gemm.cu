// Plain GEMM entry points on the tcgen05 core:
//   mb_gemm_bf16  C(bf16) = A(bf16) @ B(bf16), fp32 accumulate in TMEM
//   mb_sqr_mm_f32 C(fp32) = A(fp32) @ B(fp32) with 3xTF32 (fp32-accurate)
//
// Reference: mlx/kernels/common/sqr_mm.py:10-11 (mx.matmul) and the registry
// matmul helper mlx/kernels/common/registry.py:44-61 (row-major A [M,K],
// B [K,N], C [M,N]); the Metal kernel metal/kernels/common/sqr_mm.metal:19-111
// is a 64x64x16 simdgroup-MMA tile loop that this replaces.
#include "gemm_core.cuh"
#include "gemm_epi.cuh"

namespace {

using namespace gemm;

template <Mode MODE, int BN, int STAGES, bool B_MN, class Epi>
int launch_gemm(const void* A, const void* B, const Epi& epi, int64_t M, int64_t N, int64_t K,
                int ksplit, cudaStream_t stream) {
  using S = Smem<MODE, BN, STAGES>;
  using P = GemmProducer<MODE, BN, B_MN>;
  const int esz = elem_bytes(MODE);
  const CUtensorMapDataType dt =
      MODE == Mode::BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  MB_REQUIRE((K * esz) % 16 == 0, "gemm: K*elem_size must be a multiple of 16 bytes (K=%lld)",
             (long long)K);
  MB_REQUIRE(reinterpret_cast<uintptr_t>(A) % 16 == 0 && reinterpret_cast<uintptr_t>(B) % 16 == 0,
             "gemm: operands must be 16-byte aligned");
  MB_REQUIRE(!B_MN || (N * esz) % 16 == 0, "gemm: N*elem_size must be a multiple of 16 bytes");
  P p;
  int rc = mb::make_tmap_2d(&p.a, A, dt, esz, K, M, K * esz, P::KE, BM,
                            CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (!B_MN)
    rc = mb::make_tmap_2d(&p.b, B, dt, esz, K, N, K * esz, P::KE, BN, CU_TENSOR_MAP_SWIZZLE_128B);
  else
    rc = mb::make_tmap_2d(&p.b, B, dt, esz, N, K, N * esz, P::KE, P::KE,
                          CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  Sched sc;
  sc.tiles_m = (int)((M + BM - 1) / BM);
  sc.tiles_n = (int)((N + BN - 1) / BN);
  sc.kblocks = (int)((K + P::KE - 1) / P::KE);
  sc.ksplit = ksplit < 1 ? 1 : (ksplit > sc.kblocks ? sc.kblocks : ksplit);
  sc.kb_per_split = (sc.kblocks + sc.ksplit - 1) / sc.ksplit;
  auto kern = gemm_kernel<MODE, BN, STAGES, B_MN, P, Epi>;
  static bool attr = false;  // one instantiation = one static
  if (!attr) {
    MB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::TOTAL));
    attr = true;
  }
  const int grid = sc.total() < mb::num_sms() ? sc.total() : mb::num_sms();
  kern<<<grid, num_warps(MODE) * 32, S::TOTAL, stream>>>(p, epi, sc, mb::device_status_ptr());
  MB_CUDA(cudaGetLastError());
  return MB_OK;
}

}  // namespace

extern "C" int mb_gemm_bf16(const uint16_t* A, const uint16_t* B, uint16_t* C, int64_t M,
                            int64_t N, int64_t K, int b_layout, void* stream) {
  MB_REQUIRE(M >= 0 && N >= 0 && K >= 0, "mb_gemm_bf16: negative dimension");
  MB_REQUIRE(b_layout == 0 || b_layout == 1, "mb_gemm_bf16: b_layout must be 0 ([N,K]) or 1 ([K,N])");
  if (M == 0 || N == 0) return MB_OK;
  MB_REQUIRE(K > 0, "mb_gemm_bf16: K must be positive");
  MB_REQUIRE(N % 8 == 0, "mb_gemm_bf16: N must be a multiple of 8");
  gemm::Epi<256, gemm::EpiStore> e{};
  e.M = (int)M;
  e.N = (int)N;
  e.out = C;
  e.ldo = N;
  e.alpha = 1.f;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (b_layout == 0) return launch_gemm<gemm::Mode::BF16, 256, 4, false>(A, B, e, M, N, K, 1, s);
  return launch_gemm<gemm::Mode::BF16, 256, 4, true>(A, B, e, M, N, K, 1, s);
}

extern "C" int mb_sqr_mm_f32(const float* A, const float* B, float* C, int64_t M, int64_t N,
                             int64_t K, void* stream) {
  MB_REQUIRE(M >= 0 && N >= 0 && K >= 0, "mb_sqr_mm_f32: negative dimension");
  if (M == 0 || N == 0) return MB_OK;
  MB_REQUIRE(K > 0, "mb_sqr_mm_f32: K must be positive");
  MB_REQUIRE(N % 4 == 0 && K % 4 == 0, "mb_sqr_mm_f32: N and K must be multiples of 4");
  gemm::Epi<128, gemm::EpiStore> e{};
  e.M = (int)M;
  e.N = (int)N;
  e.out = C;
  e.ldo = N;
  e.out_f32 = 1;
  e.alpha = 1.f;
  return launch_gemm<gemm::Mode::TF32X3, 128, 3, true>(A, B, e, M, N, K, 1,
                                                       static_cast<cudaStream_t>(stream));
}
