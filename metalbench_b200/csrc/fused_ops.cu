// Standalone fused ops: the sub-steps of the decoder as their own registry
// kernels (reference standard set, mlx/kernels/standard/registry.py).
//
//   mb_rms_norm_linear_bf16     y = rms_norm(x) @ w^T   (rms_norm_linear.py; w [N, K])
//   mb_fused_add_rms_norm_bf16  y = rms_norm(x + r)     (fused_add_rms_norm.py)
//   mb_rope_bf16                interleaved-pair RoPE over the full width
//                               (rope_embedding.py: omega_i = base^(-2i/D))
//   mb_swiglu_*                 silu(x @ Wg) * (x @ Wu)   (swiglu.py)
//   mb_sdpa_bf16                softmax(Q K^T / sqrt(d)) V  (scaled_dot_product.py)
//
// They reuse the decoder's pieces: the row-norm kernel, the tcgen05 GEMM core
// with its row-scale and SwiGLU epilogues, and the paged attention kernel (a
// contiguous [S, 128] K or V is a valid page sequence with an identity page
// table).
#include <algorithm>

#include "decoder_epi.cuh"
#include "gemm_launch.cuh"
#include "kernels.h"

namespace {

using namespace gemm;

// y = (x + r) * rsqrt(mean((x + r)^2) + eps), one warp per row, fp32 math.
__global__ void add_rms_norm_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ r,
                                    uint16_t* __restrict__ y, int M, int D, float eps) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= M) return;
  const uint4* xp = reinterpret_cast<const uint4*>(x + (int64_t)row * D);
  const uint4* rp = reinterpret_cast<const uint4*>(r + (int64_t)row * D);
  float ss = 0.f;
  for (int c = lane; c < D / 8; c += 32) {
    const uint4 a = xp[c], b = rp[c];
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const float s0 = __uint_as_float(aw[m] << 16) + __uint_as_float(bw[m] << 16);
      const float s1 = __uint_as_float(aw[m] & 0xFFFF0000u) + __uint_as_float(bw[m] & 0xFFFF0000u);
      ss += s0 * s0 + s1 * s1;
    }
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float rs = rsqrtf(ss / (float)D + eps);
  uint4* yp = reinterpret_cast<uint4*>(y + (int64_t)row * D);
  for (int c = lane; c < D / 8; c += 32) {
    const uint4 a = xp[c], b = rp[c];
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
    uint32_t o[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const float s0 = (__uint_as_float(aw[m] << 16) + __uint_as_float(bw[m] << 16)) * rs;
      const float s1 =
          (__uint_as_float(aw[m] & 0xFFFF0000u) + __uint_as_float(bw[m] & 0xFFFF0000u)) * rs;
      o[m] = gemm::pack_bf16(s0, s1);
    }
    yp[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// fused_add_rms_norm for D <= 8192: one 256-thread block per row, the row's
// x + r kept in registers (at most 4 16-byte units of each per thread), so x
// and r are read once.
__global__ void __launch_bounds__(256) add_rms_norm_row_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ r, uint16_t* __restrict__ y,
    int D, float eps) {
  __shared__ float part[8];
  const int64_t row = blockIdx.x;
  const uint4* xp = reinterpret_cast<const uint4*>(x + row * D);
  const uint4* rp = reinterpret_cast<const uint4*>(r + row * D);
  const int units = D / 8;
  float v[4][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int u = threadIdx.x + k * 256;
    if (u < units) {
      const uint4 a = xp[u], b = rp[u];
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        v[k][2 * m] = __uint_as_float(aw[m] << 16) + __uint_as_float(bw[m] << 16);
        v[k][2 * m + 1] = __uint_as_float(aw[m] & 0xFFFF0000u) + __uint_as_float(bw[m] & 0xFFFF0000u);
        ss += v[k][2 * m] * v[k][2 * m] + v[k][2 * m + 1] * v[k][2 * m + 1];
      }
    }
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) tot += part[w];
  const float rs = rsqrtf(tot / (float)D + eps);
  uint4* yp = reinterpret_cast<uint4*>(y + row * D);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int u = threadIdx.x + k * 256;
    if (u < units)
      yp[u] = make_uint4(gemm::pack_bf16(v[k][0] * rs, v[k][1] * rs),
                         gemm::pack_bf16(v[k][2] * rs, v[k][3] * rs),
                         gemm::pack_bf16(v[k][4] * rs, v[k][5] * rs),
                         gemm::pack_bf16(v[k][6] * rs, v[k][7] * rs));
  }
}

// RoPE over the full width, 8 pairs (16 elements) per thread for D % 16 == 0:
// omega_i from a per-block table, the angle s*omega_i reduced to [-pi, pi]
// (two-term 2*pi, the angle itself being an fp32 product as in the
// reference) and sin/cos on the SFU.
__global__ void __launch_bounds__(256) rope_fast_kernel(const uint16_t* __restrict__ x,
                                                        uint16_t* __restrict__ y, int S, int D,
                                                        float neg_log2_base_over_half) {
  extern __shared__ float omega[];  // [D/2]
  const int half = D / 2;
  for (int i = threadIdx.x; i < half; i += blockDim.x)
    omega[i] = exp2f(neg_log2_base_over_half * (float)i);
  __syncthreads();
  const int per_row = D / 16;
  const int64_t n = (int64_t)S * per_row;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int s = (int)(t / per_row), i0 = (int)(t % per_row) * 8;
    const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)s * D + 2 * i0);
    uint4 in[2] = {src[0], src[1]};
    uint4 out[2];
    const uint32_t* iw = reinterpret_cast<const uint32_t*>(in);
    uint32_t* ow = reinterpret_cast<uint32_t*>(out);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float a = (float)s * omega[i0 + k];
      const float q = rintf(a * 0.15915494309189535f);
      const float rr = fmaf(-q, -1.7484555e-7f, fmaf(-q, 6.28318548202514648f, a));
      float sn, cs;
      __sincosf(rr, &sn, &cs);
      const float e0 = __uint_as_float(iw[k] << 16), e1 = __uint_as_float(iw[k] & 0xFFFF0000u);
      ow[k] = gemm::pack_bf16(e0 * cs - e1 * sn, e0 * sn + e1 * cs);
    }
    uint4* dst = reinterpret_cast<uint4*>(y + (int64_t)s * D + 2 * i0);
    dst[0] = out[0];
    dst[1] = out[1];
  }
}

// y = (x - mean(x)) * rsqrt(var(x) + eps) per row of D (no affine), one warp
// per row; mean first, then the variance of (x - mean), both in fp32.
__global__ void layer_norm_kernel(const uint16_t* __restrict__ x, uint16_t* __restrict__ y, int M,
                                  int D, float eps) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= M) return;
  const uint4* xp = reinterpret_cast<const uint4*>(x + (int64_t)row * D);
  auto lo = [](uint32_t w) { return __uint_as_float(w << 16); };
  auto hi = [](uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); };
  float s1 = 0.f;
  for (int c = lane; c < D / 8; c += 32) {
    const uint4 a = xp[c];
    s1 += lo(a.x) + hi(a.x) + lo(a.y) + hi(a.y) + lo(a.z) + hi(a.z) + lo(a.w) + hi(a.w);
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) s1 += __shfl_xor_sync(0xffffffffu, s1, off);
  const float mean = s1 / (float)D;
  float s2 = 0.f;
  for (int c = lane; c < D / 8; c += 32) {
    const uint4 a = xp[c];
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const float d0 = lo(aw[m]) - mean, d1 = hi(aw[m]) - mean;
      s2 += d0 * d0 + d1 * d1;
    }
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, off);
  const float rs = rsqrtf(s2 / (float)D + eps);
  uint4* yp = reinterpret_cast<uint4*>(y + (int64_t)row * D);
  for (int c = lane; c < D / 8; c += 32) {
    const uint4 a = xp[c];
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
    uint32_t o[4];
#pragma unroll
    for (int m = 0; m < 4; ++m)
      o[m] = gemm::pack_bf16((lo(aw[m]) - mean) * rs, (hi(aw[m]) - mean) * rs);
    yp[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// RoPE over the full width: thread per (position s, pair i).
__global__ void rope_kernel(const uint16_t* __restrict__ x, uint16_t* __restrict__ y, int S, int D,
                            float neg_log2_base_over_half) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int half = D / 2;
  if (t >= (int64_t)S * half) return;
  const int s = (int)(t / half), i = (int)(t % half);
  const uint32_t w = *reinterpret_cast<const uint32_t*>(x + (int64_t)s * D + 2 * i);
  const float a = __uint_as_float(w << 16), b = __uint_as_float(w & 0xFFFF0000u);
  float sn, cs;
  sincosf((float)s * exp2f(neg_log2_base_over_half * (float)i), &sn, &cs);
  *reinterpret_cast<uint32_t*>(y + (int64_t)s * D + 2 * i) =
      gemm::pack_bf16(a * cs - b * sn, a * sn + b * cs);
}

// Pack W_gate, W_up (both [D, FF], reference (in, out) layout) into the tiled,
// pre-swizzled K-major layout of the decoder's gate/up GEMM: column block t of
// 256 packed rows = gate features t*128.. then the matching up features.
__global__ void swiglu_pack_kernel(const uint16_t* __restrict__ wg, const uint16_t* __restrict__ wu,
                                   int D, int FF, uint8_t* __restrict__ out) {
  const int64_t kblocks = D / 64, tiles_n = (2 * (int64_t)FF + 255) / 256;
  const int64_t chunks = tiles_n * kblocks * 256 * 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < chunks;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tile = i / (256 * 8);
    const int r = (int)((i / 8) % 256), c = (int)(i % 8);
    const int64_t tn = tile / kblocks, kb = tile % kblocks;
    const uint16_t* src = r < 128 ? wg : wu;
    const int64_t col = tn * 128 + (r % 128);
    const int64_t k0 = kb * 64 + c * 8;
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      w[j] = (uint32_t)src[(k0 + 2 * j) * FF + col] | ((uint32_t)src[(k0 + 2 * j + 1) * FF + col] << 16);
    *reinterpret_cast<uint4*>(out + tile * (256 * KBYTES) + r * KBYTES + ((c ^ (r & 7)) * 16)) =
        make_uint4(w[0], w[1], w[2], w[3]);
  }
}

__global__ void sdpa_tables_kernel(int* bt, int pages, int* start_pos, int* kv_len, int S) {
  for (int i = threadIdx.x; i < pages; i += blockDim.x) bt[i] = i;
  if (threadIdx.x == 0) {
    start_pos[0] = 0;
    kv_len[0] = S;
  }
}

// Attention step 2 (use_rope = 0: no rotation, the multi-head attention of
// transformer_block / mha_attention): per-head interleaved-pair RoPE (omega_i =
// base^(-2i/Dh), positions 0..S-1) on q in place inside qkv [S, ld], and on k
// into the paged cache layout [S/64 pages][Hkv][64][Dh] of the attention
// kernels, together with v (copied). One thread per (s, head, pair); heads
// 0..H-1 are q, H..H+Hkv-1 k, H+Hkv.. v.
__global__ void attn_rope_scatter_kernel(uint16_t* __restrict__ qkv, int64_t ld, int S, int H,
                                         int Hkv, int use_rope, float neg_log2_base_over_half,
                                         uint16_t* __restrict__ kc, uint16_t* __restrict__ vc) {
  constexpr int Dh = 128, half = Dh / 2;
  const int heads = H + 2 * Hkv;
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= (int64_t)S * heads * half) return;
  const int i = (int)(t % half);
  const int hd = (int)((t / half) % heads);
  const int s = (int)(t / ((int64_t)half * heads));
  uint16_t* src = qkv + (int64_t)s * ld + (int64_t)hd * Dh + 2 * i;
  uint32_t w = *reinterpret_cast<const uint32_t*>(src);
  if (use_rope && hd < H + Hkv) {
    const float a = __uint_as_float(w << 16), b = __uint_as_float(w & 0xFFFF0000u);
    float sn, cs;
    sincosf((float)s * exp2f(neg_log2_base_over_half * (float)i), &sn, &cs);
    w = gemm::pack_bf16(a * cs - b * sn, a * sn + b * cs);
  }
  if (hd < H) {
    *reinterpret_cast<uint32_t*>(src) = w;
    return;
  }
  const int kh = hd < H + Hkv ? hd - H : hd - H - Hkv;
  uint16_t* dst = (hd < H + Hkv ? kc : vc) +
                  (((int64_t)(s / 64) * Hkv + kh) * 64 + (s % 64)) * Dh + 2 * i;
  *reinterpret_cast<uint32_t*>(dst) = w;
}

}  // namespace

extern "C" size_t mb_rms_norm_linear_workspace_bytes(int64_t M) {
  return M > 0 ? (size_t)((M * 4 + 255) / 256 * 256) : 0;
}

extern "C" int mb_rms_norm_linear_bf16(const uint16_t* x, const uint16_t* w, uint16_t* y, int64_t M,
                                       int64_t K, int64_t N, float eps, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  MB_REQUIRE(M >= 0 && K > 0 && N >= 0, "rms_norm_linear: bad sizes");
  if (M == 0 || N == 0) return MB_OK;
  MB_REQUIRE(K % 8 == 0 && N % 8 == 0, "rms_norm_linear: K and N must be multiples of 8");
  MB_REQUIRE(workspace && workspace_bytes >= mb_rms_norm_linear_workspace_bytes(M),
             "rms_norm_linear: workspace of %zu bytes required",
             mb_rms_norm_linear_workspace_bytes(M));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* rstd = static_cast<float*>(workspace);
  int rc = mb::rownorm(x, (int)M, (int)K, eps, rstd, s);
  if (rc) return rc;
  Epi<256, EpiStore> e{};
  e.M = (int)M;
  e.N = (int)N;
  e.out = y;
  e.ldo = N;
  e.alpha = 1.f;
  e.row_scale = rstd;
  return launch_gemm<Mode::BF16, 256, 4, false>(x, w, e, M, N, K, 1, s);
}

extern "C" int mb_fused_add_rms_norm_bf16(const uint16_t* x, const uint16_t* residual,
                                          uint16_t* y, int64_t M, int64_t D, float eps,
                                          void* stream) {
  MB_REQUIRE(M >= 0 && D > 0 && D % 8 == 0, "fused_add_rms_norm: D must be a multiple of 8");
  if (M == 0) return MB_OK;
  if (D <= 8192 && M <= 0x7FFFFFFF)
    add_rms_norm_row_kernel<<<(unsigned)M, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        x, residual, y, (int)D, eps);
  else
    add_rms_norm_kernel<<<(unsigned)((M + 7) / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        x, residual, y, (int)M, (int)D, eps);
  MB_CUDA(cudaGetLastError());
  return MB_OK;
}

extern "C" int mb_rope_bf16(const uint16_t* x, uint16_t* y, int64_t S, int64_t D, float base,
                            void* stream) {
  MB_REQUIRE(S >= 0 && D > 0 && D % 2 == 0, "rope: D must be even");
  if (S == 0) return MB_OK;
  const int64_t n = S * (D / 2);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (D % 16 == 0 && D <= 16384) {
    const int64_t units = S * (D / 16);
    const int64_t blocks = std::min<int64_t>((units + 255) / 256, (int64_t)mb::num_sms() * 8);
    rope_fast_kernel<<<(unsigned)blocks, 256, (size_t)(D / 2) * 4, s>>>(
        x, y, (int)S, (int)D, -log2f(base) / (float)(D / 2));
  } else {
    rope_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, y, (int)S, (int)D,
                                                           -log2f(base) / (float)(D / 2));
  }
  MB_CUDA(cudaGetLastError());
  return MB_OK;
}

extern "C" size_t mb_swiglu_packed_bytes(int64_t D, int64_t FF) {
  if (D <= 0 || FF <= 0) return 0;
  return gemm::tiled_weight_bytes(2 * FF, D, 256);
}

extern "C" int mb_swiglu_pack_bf16(const uint16_t* w_gate, const uint16_t* w_up, void* packed,
                                   int64_t D, int64_t FF, void* stream) {
  MB_REQUIRE(D > 0 && D % 64 == 0 && FF > 0 && FF % 128 == 0,
             "swiglu pack: D %% 64 == 0 and FF %% 128 == 0 required");
  swiglu_pack_kernel<<<1024, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      w_gate, w_up, (int)D, (int)FF, static_cast<uint8_t*>(packed));
  MB_CUDA(cudaGetLastError());
  return MB_OK;
}

extern "C" int mb_swiglu_bf16(const uint16_t* x, const void* packed, uint16_t* out, int64_t M,
                              int64_t D, int64_t FF, void* stream) {
  MB_REQUIRE(M >= 0 && D % 64 == 0 && FF % 128 == 0, "swiglu: D %% 64 and FF %% 128 required");
  if (M == 0) return MB_OK;
  dec::EpiSwiGLU e;
  e.M = (int)M;
  e.p.M = (int)M;
  e.p.FF = (int)FF;
  e.p.rstd = nullptr;
  e.p.act = out;
  return launch_gemm<Mode::BF16, 256, 4, false>(x, packed, e, M, 2 * FF, D, 1,
                                                static_cast<cudaStream_t>(stream), false, true);
}

namespace {
struct SdpaWs {
  int splits;
  size_t tables, part_o, part_ml, total;
};
SdpaWs sdpa_ws(int64_t S) {
  auto al = [](size_t x) { return (x + 255) / 256 * 256; };
  SdpaWs w;
  // one head: ceil(S/128) query tiles alone leave most SMs idle, so the keys
  // are split across CTAs (partials + a combine kernel)
  w.splits = mb::attention_split_plan(1, S, 1, S);
  w.tables = al((size_t)((S + 63) / 64 + 2) * 4);
  w.part_o = w.splits > 1 ? al((size_t)S * w.splits * 128 * 4) : 0;
  w.part_ml = w.splits > 1 ? al((size_t)S * w.splits * 2 * 4) : 0;
  w.total = w.tables + w.part_o + w.part_ml;
  return w;
}
}  // namespace

extern "C" size_t mb_sdpa_workspace_bytes(int64_t S) {
  if (S <= 0) return 0;
  return sdpa_ws(S).total;
}

extern "C" int mb_sdpa_bf16(const uint16_t* Q, const uint16_t* K, const uint16_t* V, uint16_t* O,
                            int64_t S, int64_t d, void* workspace, size_t workspace_bytes,
                            void* stream) {
  MB_REQUIRE(d == 128, "sdpa: head dimension must be 128");
  MB_REQUIRE(S >= 0 && S <= (1 << 24), "sdpa: bad S");
  if (S == 0) return MB_OK;
  const SdpaWs wl = sdpa_ws(S);
  MB_REQUIRE(workspace && workspace_bytes >= wl.total, "sdpa: workspace of %zu bytes required",
             wl.total);
  const int pages = (int)((S + 63) / 64);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  int* bt = reinterpret_cast<int*>(w);
  int* sp = bt + pages;
  int* kl = sp + 1;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  sdpa_tables_kernel<<<1, 256, 0, s>>>(bt, pages, sp, kl, (int)S);
  MB_CUDA(cudaGetLastError());
  // [S, 128] rows are pages of 64 keys for one kv head: an identity page table
  if (wl.splits > 1 && mb::attention_prefill_tc_ok(Q, 128, K, V, O, 128))
    return mb::attention_prefill_tc(Q, 128, K, V, bt, pages, sp, kl, 1, (int)S, 1, 1, 0, O, 128, s,
                                    wl.splits, (int)S,
                                    reinterpret_cast<float*>(w + wl.tables),
                                    reinterpret_cast<float*>(w + wl.tables + wl.part_o));
  return mb_attention_prefill_bf16(Q, 128, K, V, bt, pages, sp, kl, 1, (int)S, 1, 1, 128, 0, O,
                                   128, stream);
}

// ---- llama_attention (mlx/kernels/standard/llama_attention.py:22-63) ------
namespace {
struct LlamaAttnWs {
  size_t qkv, kc, o, tables, total;
};
LlamaAttnWs llama_attn_ws(int64_t S, int64_t D, int64_t Hkv) {
  auto al = [](size_t x) { return (x + 255) / 256 * 256; };
  const int64_t pages = (S + 63) / 64;
  LlamaAttnWs w;
  w.qkv = al((size_t)S * (D + 2 * Hkv * 128) * 2);
  w.kc = al((size_t)pages * Hkv * 64 * 128 * 2);
  w.o = al((size_t)S * D * 2);
  w.tables = al((size_t)(pages + 2) * 4);
  w.total = w.qkv + 2 * w.kc + w.o + w.tables;
  return w;
}
}  // namespace

extern "C" size_t mb_llama_attention_workspace_bytes(int64_t S, int64_t D, int64_t H,
                                                     int64_t Hkv) {
  if (S <= 0 || D <= 0 || H <= 0 || Hkv <= 0) return 0;
  return llama_attn_ws(S, D, Hkv).total;
}

extern "C" int mb_llama_attention_bf16(const uint16_t* x, const uint16_t* w_qkv,
                                       const uint16_t* w_o, uint16_t* out, int64_t S, int64_t D,
                                       int64_t H, int64_t Hkv, float base, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  MB_REQUIRE(S >= 0 && H > 0 && Hkv > 0 && H % Hkv == 0 && D == H * 128,
             "llama_attention: need D = 128 * H and H a multiple of H_kv");
  if (S == 0) return MB_OK;
  MB_REQUIRE(S <= (1 << 24), "llama_attention: S too large");
  const LlamaAttnWs wl = llama_attn_ws(S, D, Hkv);
  MB_REQUIRE(workspace && workspace_bytes >= wl.total,
             "llama_attention: workspace of %zu bytes required", wl.total);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  uint16_t* qkv = reinterpret_cast<uint16_t*>(w);
  uint16_t* kc = reinterpret_cast<uint16_t*>(w + wl.qkv);
  uint16_t* vc = reinterpret_cast<uint16_t*>(w + wl.qkv + wl.kc);
  uint16_t* o = reinterpret_cast<uint16_t*>(w + wl.qkv + 2 * wl.kc);
  int* bt = reinterpret_cast<int*>(w + wl.qkv + 2 * wl.kc + wl.o);
  const int pages = (int)((S + 63) / 64);
  int* sp = bt + pages;
  int* kl = sp + 1;
  const int64_t nqkv = D + 2 * Hkv * 128;
  // 1. qkv = x @ W_qkv (W in the reference's (in, out) layout)
  int rc = mb_gemm_bf16(x, w_qkv, qkv, S, nqkv, D, 1, stream);
  if (rc) return rc;
  // 2. RoPE on q (in place) and k, K/V into pages; identity page table
  const int64_t n = S * (H + 2 * Hkv) * 64;
  attn_rope_scatter_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
      qkv, nqkv, (int)S, (int)H, (int)Hkv, 1, -log2f(base) / 64.f, kc, vc);
  MB_CUDA(cudaGetLastError());
  sdpa_tables_kernel<<<1, 256, 0, s>>>(bt, pages, sp, kl, (int)S);
  MB_CUDA(cudaGetLastError());
  // 3. non-causal GQA attention over all S keys
  rc = mb_attention_prefill_bf16(qkv, (int)nqkv, kc, vc, bt, pages, sp, kl, 1, (int)S, (int)H,
                                 (int)Hkv, 128, 0, o, (int)D, stream);
  if (rc) return rc;
  // 4. out = o @ W_o
  return mb_gemm_bf16(o, w_o, out, S, D, D, 1, stream);
}

// ---- multi-head attention without RoPE: mha_attention
//      (mlx/kernels/full/mha_attention.py:13-28) and transformer_block
//      (mlx/kernels/full/transformer_block.py:22-52) --------------------------
namespace {
struct MhaWs {
  size_t qkv, kc, o, tables, total;
};
MhaWs mha_ws(int64_t S, int64_t D, int64_t H) {
  auto al = [](size_t x) { return (x + 255) / 256 * 256; };
  const int64_t pages = (S + 63) / 64;
  MhaWs w;
  w.qkv = al((size_t)S * 3 * D * 2);
  w.kc = al((size_t)pages * H * 64 * 128 * 2);
  w.o = al((size_t)S * D * 2);
  w.tables = al((size_t)(pages + 2) * 4);
  w.total = w.qkv + 2 * w.kc + w.o + w.tables;
  return w;
}

// attention of the packed qkv [S, 3D] (q | k | v, H heads of 128 each, no
// RoPE, no mask) into o [S, D]; kc, vc, tables from the workspace layout above
int mha_core(uint16_t* qkv, uint8_t* w, const MhaWs& wl, int64_t S, int64_t D, int64_t H,
             uint16_t* o, cudaStream_t s) {
  uint16_t* kc = reinterpret_cast<uint16_t*>(w + wl.qkv);
  uint16_t* vc = reinterpret_cast<uint16_t*>(w + wl.qkv + wl.kc);
  int* bt = reinterpret_cast<int*>(w + wl.qkv + 2 * wl.kc + wl.o);
  const int pages = (int)((S + 63) / 64);
  int* sp = bt + pages;
  int* kl = sp + 1;
  const int64_t n = S * 3 * H * 64;
  attn_rope_scatter_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
      qkv, 3 * D, (int)S, (int)H, (int)H, 0, 0.f, kc, vc);
  MB_CUDA(cudaGetLastError());
  sdpa_tables_kernel<<<1, 256, 0, s>>>(bt, pages, sp, kl, (int)S);
  MB_CUDA(cudaGetLastError());
  return mb_attention_prefill_bf16(qkv, (int)(3 * D), kc, vc, bt, pages, sp, kl, 1, (int)S,
                                   (int)H, (int)H, 128, 0, o, (int)D, s);
}
}  // namespace

extern "C" size_t mb_mha_attention_workspace_bytes(int64_t S, int64_t D) {
  if (S <= 0 || D <= 0 || D % 128) return 0;
  return mha_ws(S, D, D / 128).total;
}

extern "C" int mb_mha_attention_bf16(const uint16_t* x, const uint16_t* wq, const uint16_t* wk,
                                     const uint16_t* wv, const uint16_t* wo, uint16_t* out,
                                     int64_t S, int64_t D, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  MB_REQUIRE(S >= 0 && D > 0 && D % 128 == 0, "mha_attention: D must be a multiple of 128");
  if (S == 0) return MB_OK;
  MB_REQUIRE(S <= (1 << 24), "mha_attention: S too large");
  const int64_t H = D / 128;
  const MhaWs wl = mha_ws(S, D, H);
  MB_REQUIRE(workspace && workspace_bytes >= wl.total,
             "mha_attention: workspace of %zu bytes required", wl.total);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  uint16_t* qkv = reinterpret_cast<uint16_t*>(w);
  uint16_t* o = reinterpret_cast<uint16_t*>(w + wl.qkv + 2 * wl.kc);
  // q | k | v side by side in one [S, 3D] buffer
  const uint16_t* ws3[3] = {wq, wk, wv};
  for (int j = 0; j < 3; ++j) {
    const int rc = mb::gemm_bf16_ex(x, ws3[j], qkv + j * D, S, D, D, 3 * D, 1, nullptr, 0, 0, s);
    if (rc) return rc;
  }
  const int rc = mha_core(qkv, w, wl, S, D, H, o, s);
  if (rc) return rc;
  return mb::gemm_bf16_ex(o, wo, out, S, D, D, D, 1, nullptr, 0, 0, s);
}

namespace {
size_t tb_extra(int64_t S, int64_t D, int64_t FF) {  // ln, x1, ffn hidden
  auto al = [](size_t x) { return (x + 255) / 256 * 256; };
  return 2 * al((size_t)S * D * 2) + al((size_t)S * FF * 2);
}
}  // namespace

extern "C" size_t mb_transformer_block_workspace_bytes(int64_t S, int64_t D, int64_t H,
                                                       int64_t FF) {
  if (S <= 0 || D <= 0 || H <= 0 || FF <= 0 || D != 128 * H) return 0;
  return mha_ws(S, D, H).total + tb_extra(S, D, FF);
}

extern "C" int mb_transformer_block_bf16(const uint16_t* x, const uint16_t* w_qkv,
                                         const uint16_t* w_o, const uint16_t* w_ff1,
                                         const uint16_t* w_ff2, uint16_t* out, int64_t S,
                                         int64_t D, int64_t H, int64_t FF, float eps,
                                         void* workspace, size_t workspace_bytes, void* stream) {
  MB_REQUIRE(S >= 0 && H > 0 && D == 128 * H && D % 8 == 0 && FF > 0 && FF % 8 == 0,
             "transformer_block: need D = 128 * H and FF a multiple of 8");
  if (S == 0) return MB_OK;
  MB_REQUIRE(S <= (1 << 24), "transformer_block: S too large");
  const MhaWs wl = mha_ws(S, D, H);
  const size_t need = wl.total + tb_extra(S, D, FF);
  MB_REQUIRE(workspace && workspace_bytes >= need,
             "transformer_block: workspace of %zu bytes required", need);
  auto al = [](size_t v) { return (v + 255) / 256 * 256; };
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  uint16_t* qkv = reinterpret_cast<uint16_t*>(w);
  uint16_t* o = reinterpret_cast<uint16_t*>(w + wl.qkv + 2 * wl.kc);
  uint16_t* ln = reinterpret_cast<uint16_t*>(w + wl.total);
  uint16_t* x1 = reinterpret_cast<uint16_t*>(w + wl.total + al((size_t)S * D * 2));
  uint16_t* hdn = reinterpret_cast<uint16_t*>(w + wl.total + 2 * al((size_t)S * D * 2));
  const unsigned ln_grid = (unsigned)((S + 7) / 8);
  // attention sub-block: x1 = x + MHA(LN(x)) @ W_o
  layer_norm_kernel<<<ln_grid, 256, 0, s>>>(x, ln, (int)S, (int)D, eps);
  MB_CUDA(cudaGetLastError());
  int rc = mb::gemm_bf16_ex(ln, w_qkv, qkv, S, 3 * D, D, 3 * D, 1, nullptr, 0, 0, s);
  if (!rc) rc = mha_core(qkv, w, wl, S, D, H, o, s);
  if (!rc) rc = mb::gemm_bf16_ex(o, w_o, x1, S, D, D, D, 1, x, D, 0, s);
  if (rc) return rc;
  // FFN sub-block: out = x1 + gelu(LN(x1) @ W_ff1) @ W_ff2
  layer_norm_kernel<<<ln_grid, 256, 0, s>>>(x1, ln, (int)S, (int)D, eps);
  MB_CUDA(cudaGetLastError());
  rc = mb::gemm_bf16_ex(ln, w_ff1, hdn, S, FF, D, FF, 1, nullptr, 0, 1, s);
  if (!rc) rc = mb::gemm_bf16_ex(hdn, w_ff2, out, S, D, FF, D, 1, x1, D, 0, s);
  return rc;
}
