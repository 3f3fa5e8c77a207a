// Host-side launcher for the tcgen05 GEMM core with 2-D tensor-map operands.
#pragma once
#include "gemm_core.cuh"

namespace gemm {

// Stream-K plan for `tiles` output tiles of `kblocks` k-blocks on `sms` CTAs:
// k-blocks per CTA, CTAs used, and an upper bound on the segments one tile
// can be cut into (the size of the partial-sum buffer in tiles).
struct StreamK {
  int per, ctas, max_segs;
};
inline StreamK streamk_plan(int tiles, int kblocks, int sms) {
  const long long total = (long long)tiles * kblocks;
  StreamK p;
  p.per = (int)((total + sms - 1) / sms);
  if (p.per < 1) p.per = 1;
  p.ctas = (int)((total + p.per - 1) / p.per);
  p.max_segs = (kblocks + p.per - 1) / p.per + 1;
  return p;
}

template <Mode MODE, int BN, int STAGES, bool B_MN, class Epi>
inline int launch_gemm(const void* A, const void* B, const Epi& epi, int64_t M, int64_t N, int64_t K,
                int ksplit, cudaStream_t stream, bool streamk = false, bool b_tiled = false) {
  using P = GemmProducer<MODE, BN, B_MN>;
  using S = Smem<P, BN, STAGES>;
  const int esz = elem_bytes(MODE);
  const CUtensorMapDataType dt =
      MODE == Mode::BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  MB_REQUIRE((K * esz) % 16 == 0, "gemm: K*elem_size must be a multiple of 16 bytes (K=%lld)",
             (long long)K);
  MB_REQUIRE(reinterpret_cast<uintptr_t>(A) % 16 == 0 && reinterpret_cast<uintptr_t>(B) % 16 == 0,
             "gemm: operands must be 16-byte aligned");
  MB_REQUIRE(!B_MN || (N * esz) % 16 == 0, "gemm: N*elem_size must be a multiple of 16 bytes");
  P p;
  p.a_rows = M < BM ? (uint32_t)((M + 15) / 16 * 16) : (uint32_t)BM;
  int rc = mb::make_tmap_2d(&p.a, A, dt, esz, K, M, K * esz, P::KE, p.a_rows,
                            CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (b_tiled) {
    MB_REQUIRE(MODE == Mode::BF16 && !B_MN && K % P::KE == 0,
               "gemm: tiled B needs bf16, K-major and K %% 64 == 0");
    p.b_tiled = static_cast<const uint8_t*>(B);
    p.b_kblocks = (int)(K / P::KE);
  } else if (!B_MN)
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
  // no empty trailing split: every split owns at least one k-block
  sc.ksplit = (sc.kblocks + sc.kb_per_split - 1) / sc.kb_per_split;
  auto kern = gemm_kernel<BN, STAGES, P, Epi>;
  {
    const int arc = mb::ensure_smem_attr(reinterpret_cast<const void*>(kern), S::TOTAL);
    if (arc) return arc;
  }
  int grid = sc.total() < mb::num_sms() ? sc.total() : mb::num_sms();
  if (streamk) {
    const StreamK pl = streamk_plan(sc.tiles_m * sc.tiles_n, sc.kblocks, mb::num_sms());
    sc.ksplit = 1;
    sc.kb_per_split = sc.kblocks;
    sc.streamk = 1;
    sc.sk_per = pl.per;
    grid = pl.ctas;
  }
  MB_CUDA(mb::launch_pdl(kern, dim3(grid), dim3(256), S::TOTAL, stream, p, epi, sc,
                          mb::device_status_ptr()));
  MB_CUDA(cudaGetLastError());
  return MB_OK;
}


// Weight tiling: a K-major bf16 [N, K] matrix (K % 64 == 0) becomes
// ceil(N/BN) x K/64 tiles, tile (tn, kb) at ((tn * K/64) + kb) * BN * 128 bytes,
// each holding rows tn*BN.. and k kb*64.. exactly as the 128-byte-swizzled TMA
// box lands in shared memory: 16-byte chunk c of row r at r*128 + ((c ^ (r%8))*16).
// Rows past N are zero. A GEMM then streams each stage's B with one
// contiguous bulk copy. (The tiling kernel is decoder.cu's tile_weights_kernel.)
inline size_t tiled_weight_bytes(int64_t N, int64_t K, int BN) {
  return (size_t)((N + BN - 1) / BN) * (size_t)(K / 64) * BN * KBYTES;
}

// Stream-K GEMM for decode sizes (M <= 64): bf16, B K-major [N, K].
template <int BN, int STAGES, class Epi>
inline int launch_gemm_decode(const void* A, const void* B, const Epi& epi, int64_t M, int64_t N,
                              int64_t K, cudaStream_t stream, bool b_tiled = false) {
  using P = DecodeProducer<BN, 64>;
  using S = Smem<P, BN, STAGES>;
  static_assert(S::TOTAL <= 232448, "decode GEMM: shared memory over the sm_100 limit");
  MB_REQUIRE(M >= 1 && M <= 64, "decode GEMM: M must be in [1, 64]");
  MB_REQUIRE(K % 8 == 0, "decode GEMM: K must be a multiple of 8");
  P p;
  p.a_rows = (uint32_t)((M + 15) / 16 * 16);
  int rc = mb::make_tmap_2d(&p.a, A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, M, K * 2, 64,
                            p.a_rows, CU_TENSOR_MAP_SWIZZLE_128B);
  if (b_tiled) {
    MB_REQUIRE(K % 64 == 0, "decode GEMM: tiled B needs K %% 64 == 0");
    p.b_tiled = static_cast<const uint8_t*>(B);
    p.b_kblocks = (int)(K / 64);
  } else if (!rc) {
    rc = mb::make_tmap_2d(&p.b, B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, N, K * 2, 64, BN,
                          CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (rc) return rc;
  Sched sc;
  sc.tiles_m = 1;
  sc.tiles_n = (int)((N + BN - 1) / BN);
  sc.kblocks = (int)((K + 63) / 64);
  sc.ksplit = 1;
  sc.kb_per_split = sc.kblocks;
  const StreamK pl = streamk_plan(sc.tiles_n, sc.kblocks, mb::num_sms());
  sc.streamk = 1;
  sc.sk_per = pl.per;
  auto kern = gemm_kernel<BN, STAGES, P, Epi>;
  {
    const int arc = mb::ensure_smem_attr(reinterpret_cast<const void*>(kern), S::TOTAL);
    if (arc) return arc;
  }
  MB_CUDA(mb::launch_pdl(kern, dim3(pl.ctas), dim3(256), S::TOTAL, stream, p, epi, sc,
                          mb::device_status_ptr()));
  MB_CUDA(cudaGetLastError());
  return MB_OK;
}

}  // namespace gemm
