// NHWC conv2d (cross-correlation, OHWI weights) as an implicit GEMM on the
// tcgen05 core.
//
// Reference: hook mlx/kernels/common/conv2d.py:7-12 (mx.conv2d, NHWC x OHWI,
// stride, padding 0 in the hook; the north-star config uses padding 1), the
// registry entry mlx/kernels/common/registry.py:469-477 and the Metal kernel
// metal/kernels/common/conv2d/default.metal:31-217 (implicit im2col GEMM with
// M = N*H2*W2, K = KH*KW*Cin, simdgroup MMA).
//
//   GEMM M  = output pixels, tiled as TH output rows x TW output columns of one
//            image (TH*TW = 128; TW = 64 when W2 <= 64, else 128);
//   GEMM N  = Cout (one N tile of up to 256);
//   GEMM K  = (r, s, c): one k-block is one filter tap (r, s) x 64 channels.
// The A tile of a k-block is ONE 4-D TMA box {64 ch, TW, TH, 1} of x taken at
// (c0, w0 + s - pad, h0 + r - pad, n): TMA zero-fills coordinates outside the
// image, which is exactly the zero padding, and lands the box as 128 rows of
// 128 bytes in the same 128-byte swizzle as a K-major GEMM operand. The weight
// tensor [Cout, KH*KW*Cin] is the K-major B operand as stored (OHWI).
#include <stdlib.h>

#include "gemm_core.cuh"
#include "gemm_epi.cuh"

namespace {

using namespace gemm;

struct ConvGeom {
  int N, H, W, C, Co, KH, KW, pad, H2, W2, TH, TW, tiles_h, tiles_w, cchunks;
};

template <int BN>
struct ConvProducer {
  CUtensorMap x, w;
  ConvGeom g;
  static constexpr int KE = 64;
  static constexpr uint32_t BYTES = (BM + BN) * KBYTES;
  __device__ uint32_t stage_tx_bytes() const { return BYTES; }
  static constexpr int STAGE_BYTES = (BM + BN) * KBYTES;
  static constexpr int RESIDENT_BYTES = 0;
  __device__ uint32_t resident_tx_bytes() const { return 0; }
  static constexpr int KSTEPS = 4;
  __device__ void prefetch() const {
    mbd::prefetch_tmap(&x);
    mbd::prefetch_tmap(&w);
  }
  __device__ void load(uint8_t* st, uint64_t* bar, int tm, int tn, int kb) const {
    const int tw = tm % g.tiles_w;
    const int th = (tm / g.tiles_w) % g.tiles_h;
    const int n = tm / (g.tiles_w * g.tiles_h);
    const int tap = kb / g.cchunks, c0 = (kb % g.cchunks) * 64;
    const int r = tap / g.KW, s = tap % g.KW;
    mbd::tma_load_4d(st, &x, bar, c0, tw * g.TW + s - g.pad, th * g.TH + r - g.pad, n);
    mbd::tma_load_2d(st + BM * KBYTES, &w, bar, kb * 64, tn * BN);
  }
  __device__ static uint64_t a_desc(uint32_t sA, int kk) {
    return mbd::sw128_desc(sA + kk * 32, 16, 1024);
  }
  __device__ static uint64_t b_desc(uint32_t sB, int kk) {
    return mbd::sw128_desc(sB + kk * 32, 16, 1024);
  }
  __device__ void load_resident(uint8_t*, uint64_t*) const {}
  __device__ void issue(uint32_t d, uint32_t st, uint32_t, int, int, bool first) const {
    constexpr uint32_t idesc = mbd::make_idesc(1u, BM, BN, 0, 0);
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk)
      mbd::mma_f16(d, a_desc(st, kk), b_desc(st + BM * KBYTES, kk), idesc,
                   (!first || kk > 0) ? 1u : 0u);
  }
};

// Resident-weight variant (the weights of all taps fit in shared memory next
// to the ring; they are loaded once per CTA). Output pixels of one image are
// numbered as positions p = h*TWS + w in a grid TWS = W2 + KW - 1 slots wide
// (slots w >= W2 are padding), and a tile is 128 consecutive positions
// [p0, p0 + 128). Its A data is ONE TMA box {64 ch, TWS, ROWS, 1} of x taken
// at (c0, -pad, h0 - pad, n), h0 = p0 / TWS: input row h0 - pad + j lands as
// box rows [j*TWS, (j+1)*TWS), zero-filled outside the image. Position
// p0 + m under tap (r, s) reads input pixel (h + r - pad, w + s - pad), which
// is box row (p0 - h0*TWS) + m + r*TWS + s, so the A operand of every tap is
// the same box seen from a descriptor that starts off + r*TWS + s rows in
// (the swizzle follows the shared-memory address, so any 128-byte row start
// works). One load serves all KH*KW taps; rows read past the box land in
// the stage's slack and only reach positions whose slot is >= W2.
// k-block kb = channel chunk.
template <int BN, int KH>
struct ConvResProducer {
  CUtensorMap x, w;
  ConvGeom g;
  int box_rows;  // ROWS = (TWS - 1 + 127) / TWS + KH
  int tiles_per_img;
  FastDiv fd_tpi, fd_tw;  // / tiles_per_img, / TWS
  static constexpr int MAX_BOX_SLOTS = 384;  // ROWS*TWS <= 127 + TWS + KH*TWS for TWS <= 64
  static constexpr int STAGE_BYTES = MAX_BOX_SLOTS * KBYTES + 1024;  // + 8 rows of slack
  static constexpr int MAX_TAPS_CHUNKS = 9;  // KH*KW*cchunks served resident
  static constexpr int RESIDENT_BYTES = MAX_TAPS_CHUNKS * BN * KBYTES;
  uint32_t box_tx;       // ROWS * TWS * 128
  uint32_t resident_tx;  // bytes of the resident weight load
  __device__ uint32_t stage_tx_bytes() const { return box_tx; }
  __device__ uint32_t resident_tx_bytes() const { return resident_tx; }
  __device__ void prefetch() const {
    mbd::prefetch_tmap(&x);
    mbd::prefetch_tmap(&w);
  }
  __device__ void load_resident(uint8_t* res, uint64_t* bar) const {
    const int chunks = g.KH * g.KW * g.cchunks;
    for (int j = 0; j < chunks; ++j) mbd::tma_load_2d(res + j * BN * KBYTES, &w, bar, j * 64, 0);
  }
  __device__ void load(uint8_t* st, uint64_t* bar, int tm, int, int kb) const {
    const int n = fd_tpi.div(tm);
    const int h0 = fd_tw.div((tm - n * tiles_per_img) * BM);
    mbd::tma_load_4d(st, &x, bar, kb * 64, -g.pad, h0 - g.pad, n);
  }
  // One thread issues KH*KW*4 MMAs of N = 64 per stage, each only ~25 ns of
  // tensor work, so the issue loop is kept to two 64-bit adds per MMA: the
  // descriptors' start-address fields (address >> 4 in the low bits) are
  // advanced in 16-byte units from two base descriptors.
  __device__ void issue(uint32_t d, uint32_t st, uint32_t res, int tm, int kb, bool first) const {
    constexpr uint32_t idesc = mbd::make_idesc(1u, BM, BN, 0, 0);
    constexpr uint64_t kRow = KBYTES / 16, kChunk = BN * KBYTES / 16;
    const int off = fd_tw.mod(fd_tpi.mod(tm) * BM);  // p0 - h0*TWS
    const uint64_t a0 = mbd::sw128_desc(st, 16, 1024) + (uint64_t)off * kRow;
    const uint64_t b0 = mbd::sw128_desc(res, 16, 1024) + (uint64_t)kb * kChunk;
    const uint64_t a_row = (uint64_t)g.TW * kRow, b_tap = (uint64_t)g.cchunks * kChunk;
#pragma unroll
    for (int r = 0; r < KH; ++r) {
#pragma unroll
      for (int s = 0; s < 3; ++s) {
        if (s >= g.KW) break;
        const uint64_t ad = a0 + r * a_row + s * kRow;
        const uint64_t bd = b0 + (uint64_t)(r * g.KW + s) * b_tap;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mbd::mma_f16(d, ad + 2 * kk, bd + 2 * kk, idesc,
                       (!first || r > 0 || s > 0 || kk > 0) ? 1u : 0u);
      }
    }
  }
};

// Position p0 + m of tile tm is output pixel (n, p / TWS, p % TWS); slots past
// W2 and rows past H2 are dropped.
template <int BN>
struct EpiConvFlat {
  static constexpr bool kEarlyRelease = true;
  static_assert(BN == 64, "one 128-byte bf16 row per accumulator row");
  int M;  // tiles * 128: every accumulator row is "in range" for the core
  ConvGeom g;
  int tiles_per_img;
  FastDiv fd_tpi, fd_tw;
  uint16_t* y;
  // Each warp stages its 32 rows (bf16, 128 B each, 16-byte chunk j of row r
  // at chunk j ^ (r & 7): conflict-free both ways) and writes them back as
  // 4 whole pixels (4 * 2*Cout contiguous bytes) per store instruction instead of
  // 32 scattered 16-byte pieces, which keeps the SM's load/store pipe, and
  // with it the MMA thread's barrier polls, from backing up.
  __device__ void operator()(const EpiCtx& c) const {
    __shared__ alignas(128) uint4 stage_buf[4][32][8];
    uint32_t r[BN / 16][16];
#pragma unroll
    for (int q = 0; q < BN / 16; ++q) mbd::tmem_ld16(c.taddr + q * 16, r[q]);
    mbd::tmem_ld_wait();
    release_acc(c);
    const int lane = threadIdx.x & 31, wq = (threadIdx.x >> 5) & 3;
    uint4(&sb)[32][8] = stage_buf[wq];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint4 u;
      u.x = pack_bf16(__uint_as_float(r[j >> 1][(j & 1) * 8 + 0]), __uint_as_float(r[j >> 1][(j & 1) * 8 + 1]));
      u.y = pack_bf16(__uint_as_float(r[j >> 1][(j & 1) * 8 + 2]), __uint_as_float(r[j >> 1][(j & 1) * 8 + 3]));
      u.z = pack_bf16(__uint_as_float(r[j >> 1][(j & 1) * 8 + 4]), __uint_as_float(r[j >> 1][(j & 1) * 8 + 5]));
      u.w = pack_bf16(__uint_as_float(r[j >> 1][(j & 1) * 8 + 6]), __uint_as_float(r[j >> 1][(j & 1) * 8 + 7]));
      sb[lane][j ^ (lane & 7)] = u;
    }
    __syncwarp();
    const int tm = c.row / BM;
    const int n = fd_tpi.div(tm);
    const int p_warp = (tm - n * tiles_per_img) * BM + wq * 32;  // position of this warp's row 0
    const int sub = lane >> 3, ch = lane & 7;
    int h = fd_tw.div(p_warp + sub), wo = p_warp + sub - h * g.TW;  // walked 4 positions a step
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int rr = it * 4 + sub;  // staged row
      const uint4 u = sb[rr][ch ^ (rr & 7)];
      if (h < g.H2 && wo < g.W2 && ch * 8 < g.Co) {
        uint4* out = reinterpret_cast<uint4*>(y + (((int64_t)n * g.H2 + h) * g.W2 + wo) * g.Co);
        out[ch] = u;
      }
      wo += 4;
      while (wo >= g.TW) {
        wo -= g.TW;
        ++h;
      }
    }
    __syncwarp();
  }
};

// Accumulator row (hh * TW + ww) of tile tm is output pixel
// (n, th*TH + hh, tw*TW + ww); rows past the image edge are dropped.
template <int BN>
struct EpiConv {
  int M;  // tiles_m * 128: every accumulator row is "in range" for the core
  ConvGeom g;
  uint16_t* y;
  __device__ void operator()(const EpiCtx& c) const {
    const int tm = c.row / BM, local = c.row % BM;
    const int tw = tm % g.tiles_w;
    const int th = (tm / g.tiles_w) % g.tiles_h;
    const int n = tm / (g.tiles_w * g.tiles_h);
    const int h = th * g.TH + local / g.TW, wo = tw * g.TW + local % g.TW;
    const bool ok = h < g.H2 && wo < g.W2;
    const int64_t pix = ((int64_t)n * g.H2 + h) * g.W2 + wo;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      float v[32];
      tmem_ld32(c.taddr + c0, v);
      const int nn = c.n0 + c0;
      if (!ok || nn >= g.Co) continue;
      store_row32(y, g.Co, 0, (int)pix, nn, g.Co, v);
    }
  }
};

template <int BN, int STAGES>
int launch_conv(const uint16_t* x, const uint16_t* w, uint16_t* y, const ConvGeom& g,
                cudaStream_t stream) {
  using P = ConvProducer<BN>;
  using S = Smem<P, BN, STAGES>;
  using E = EpiConv<BN>;
  P p;
  p.g = g;
  const uint64_t dims[4] = {(uint64_t)g.C, (uint64_t)g.W, (uint64_t)g.H, (uint64_t)g.N};
  const uint64_t strides[3] = {(uint64_t)g.C * 2, (uint64_t)g.W * g.C * 2,
                               (uint64_t)g.H * g.W * g.C * 2};
  const uint32_t box[4] = {64, (uint32_t)g.TW, (uint32_t)g.TH, 1};
  int rc = mb::make_tmap_nd(&p.x, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, dims, strides, box,
                            CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const int64_t Kt = (int64_t)g.KH * g.KW * g.C;
  rc = mb::make_tmap_2d(&p.w, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, Kt, g.Co, Kt * 2, 64, BN,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  Sched sc;
  sc.tiles_m = g.N * g.tiles_h * g.tiles_w;
  sc.tiles_n = (g.Co + BN - 1) / BN;
  sc.kblocks = g.KH * g.KW * g.cchunks;
  sc.ksplit = 1;
  sc.kb_per_split = sc.kblocks;
  E e;
  e.M = sc.tiles_m * BM;
  e.g = g;
  e.y = y;
  auto kern = gemm_kernel<BN, STAGES, P, E>;
  {
    const int arc = mb::ensure_smem_attr(reinterpret_cast<const void*>(kern), S::TOTAL);
    if (arc) return arc;
  }
  const int grid = sc.total() < mb::num_sms() ? sc.total() : mb::num_sms();
  kern<<<grid, 256, S::TOTAL, stream>>>(p, e, sc, mb::device_status_ptr());
  MB_CUDA(cudaGetLastError());
  return MB_OK;
}

template <int BN, int KH, int STAGES>
int launch_conv_res(const uint16_t* x, const uint16_t* w, uint16_t* y, const ConvGeom& g0,
                    cudaStream_t stream) {
  using P = ConvResProducer<BN, KH>;
  using S = Smem<P, BN, STAGES>;
  using E = EpiConvFlat<BN>;
  static_assert(S::TOTAL + 16384 <= 232448, "conv: shared memory over the sm_100 limit");
  ConvGeom g = g0;
  g.TW = g.W2 + g.KW - 1;  // TWS: position-grid width in slots
  P p;
  p.g = g;
  p.box_rows = (g.TW - 1 + BM - 1) / g.TW + KH;
  p.tiles_per_img = (g.H2 * g.TW + BM - 1) / BM;
  p.fd_tpi.set(p.tiles_per_img);
  p.fd_tw.set(g.TW);
  MB_REQUIRE(g.TW <= 64 && p.box_rows * g.TW <= P::MAX_BOX_SLOTS, "conv: resident box too large");
  p.box_tx = (uint32_t)(p.box_rows * g.TW * KBYTES);
  const int chunks = g.KH * g.KW * g.cchunks;
  p.resident_tx = (uint32_t)(chunks * BN * KBYTES);
  const uint64_t dims[4] = {(uint64_t)g.C, (uint64_t)g.W, (uint64_t)g.H, (uint64_t)g.N};
  const uint64_t strides[3] = {(uint64_t)g.C * 2, (uint64_t)g.W * g.C * 2,
                               (uint64_t)g.H * g.W * g.C * 2};
  const uint32_t box[4] = {64, (uint32_t)g.TW, (uint32_t)p.box_rows, 1};
  int rc = mb::make_tmap_nd(&p.x, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, dims, strides, box,
                            CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const int64_t Kt = (int64_t)g.KH * g.KW * g.C;
  rc = mb::make_tmap_2d(&p.w, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, Kt, g.Co, Kt * 2, 64, BN,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  Sched sc;
  sc.tiles_m = g.N * p.tiles_per_img;
  sc.tiles_n = 1;
  sc.kblocks = g.cchunks;
  sc.ksplit = 1;
  sc.kb_per_split = sc.kblocks;
  E e;
  e.M = sc.tiles_m * BM;
  e.g = g;
  e.tiles_per_img = p.tiles_per_img;
  e.fd_tpi = p.fd_tpi;
  e.fd_tw = p.fd_tw;
  e.y = y;
  auto kern = gemm_kernel<BN, STAGES, P, E>;
  {
    const int arc = mb::ensure_smem_attr(reinterpret_cast<const void*>(kern), S::TOTAL);
    if (arc) return arc;
  }
  const int grid = sc.total() < mb::num_sms() ? sc.total() : mb::num_sms();
  kern<<<grid, 256, S::TOTAL, stream>>>(p, e, sc, mb::device_status_ptr());
  MB_CUDA(cudaGetLastError());
  return MB_OK;
}

}  // namespace

extern "C" int mb_conv2d_nhwc_bf16(const uint16_t* x, const uint16_t* w, uint16_t* y, int N, int H,
                                   int W, int Cin, int Cout, int KH, int KW, int stride, int pad,
                                   void* stream) {
  MB_REQUIRE(N >= 0 && H > 0 && W > 0 && KH > 0 && KW > 0 && pad >= 0,
             "mb_conv2d_nhwc_bf16: bad geometry");
  MB_REQUIRE(stride == 1, "mb_conv2d_nhwc_bf16: only stride 1 is implemented (got %d)", stride);
  MB_REQUIRE(Cin > 0 && Cin % 64 == 0, "mb_conv2d_nhwc_bf16: Cin must be a multiple of 64");
  MB_REQUIRE(Cout > 0 && Cout % 16 == 0 && Cout <= 256,
             "mb_conv2d_nhwc_bf16: Cout must be a multiple of 16 and at most 256");
  MB_REQUIRE(pad < KH && pad < KW, "mb_conv2d_nhwc_bf16: padding must be smaller than the kernel");
  ConvGeom g;
  g.N = N; g.H = H; g.W = W; g.C = Cin; g.Co = Cout; g.KH = KH; g.KW = KW; g.pad = pad;
  g.H2 = H + 2 * pad - KH + 1;
  g.W2 = W + 2 * pad - KW + 1;
  MB_REQUIRE(g.H2 > 0 && g.W2 > 0, "mb_conv2d_nhwc_bf16: empty output");
  if (N == 0) return MB_OK;
  g.TW = g.W2 <= 64 ? 64 : 128;
  g.TH = BM / g.TW;
  g.tiles_w = (g.W2 + g.TW - 1) / g.TW;
  g.tiles_h = (g.H2 + g.TH - 1) / g.TH;
  g.cchunks = Cin / 64;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Resident-weight path: position-grid rows of at most 64 slots (W2+KW-1),
  // 3 filter rows, all weight chunks (KH*KW*Cin/64 <= 9) in shared memory,
  // Cout <= 64.
  // (its epilogue stores 16-byte pieces of y, so y must be 16-byte aligned).
  if (g.W2 + KW - 1 <= 64 && KH == 3 && KW <= 3 && KH * KW * g.cchunks <= 9 && Cout <= 64 &&
      (reinterpret_cast<uintptr_t>(y) & 15) == 0 &&
      getenv("MB_CONV_NO_RESIDENT") == nullptr)
    return launch_conv_res<64, 3, 2>(x, w, y, g, s);
  if (Cout <= 64) return launch_conv<64, 8>(x, w, y, g, s);
  if (Cout <= 128) return launch_conv<128, 6>(x, w, y, g, s);
  return launch_conv<256, 4>(x, w, y, g, s);
}

