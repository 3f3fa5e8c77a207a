// Fused decoder epilogues, shared by the tcgen05 GEMM epilogue warps (values
// straight from TMEM) and by the split-K reduce kernel (values summed from
// fp32 partials). Every function handles one row and one 32-column chunk.
//
// Reference op order (mlx/kernels/full/llama_decoder_layer.py:24-64):
//   h = x * rsqrt(mean(x^2)+eps)             -> folded in as a per-row scale
//   qkv = h @ W_qkv; RoPE(q), RoPE(k)         -> EpiQKV (scale, rotate, scatter
//                                               q to [T, D] and k, v into the
//                                               paged KV cache)
//   x1 = x + attn @ W_o                       -> EpiStore with residual
//   gu = rms(x1) @ W_gu; silu(g) * u          -> EpiSwiGLU (scale, gate*up)
//   y  = x1 + act @ W_down                    -> EpiStore with residual
#pragma once
#include "gemm_epi.cuh"

namespace dec {

// Paged KV cache: k and v are [num_pages][Hkv][page][Dh] bf16; sequence b's
// token at position p lives in page block_table[b * max_pages + p / page],
// slot p % page.
struct KvCache {
  uint16_t* k;
  uint16_t* v;
  const int* block_table;
  int max_pages;
  int page;
};

// Rows are b * S + s: S new tokens of sequence b at positions start_pos[b] + s.
struct QkvParams {
  int M;        // rows (tokens)
  int S;        // new tokens per sequence
  int Hq, Hkv;  // heads held by this rank
  int Dh;
  float neg_log2_base_over_half;  // -log2(base) / (Dh/2)
  const float* rstd;              // per-row RMSNorm scale
  const int* start_pos;           // [B]
  uint16_t* q_out;                // [M, Hq*Dh]
  KvCache kv;

  // Rotate adjacent pairs (2i, 2i+1) of head-local dims d0..d0+W-1.
  template <int W>
  __device__ __forceinline__ void rope(float (&v)[W], int pos, int d0) const {
#pragma unroll
    for (int j = 0; j < W; j += 2) {
      const int i = (d0 + j) >> 1;
      const float inv_freq = exp2f(neg_log2_base_over_half * (float)i);
      float sn, cs;
      sincosf((float)pos * inv_freq, &sn, &cs);
      const float a = v[j], b = v[j + 1];
      v[j] = a * cs - b * sn;
      v[j + 1] = a * sn + b * cs;
    }
  }

  template <int W>
  __device__ void apply(int row, int col, float (&v)[W]) const {
    const float sc = rstd ? rstd[row] : 1.f;
#pragma unroll
    for (int j = 0; j < W; ++j) v[j] *= sc;
    const int b = row / S, s = row % S;
    const int pos = start_pos[b] + s;
    const int Dq = Hq * Dh, Dk = Hkv * Dh;
    if (col < Dq) {
      rope<W>(v, pos, col % Dh);
      gemm::store_rowW<W>(q_out, Dq, 0, row, col, Dq, v);
      return;
    }
    const bool is_k = col < Dq + Dk;
    const int c = is_k ? col - Dq : col - Dq - Dk;
    const int head = c / Dh, d = c % Dh;
    if (is_k) rope<W>(v, pos, d);
    const int pg = kv.block_table[b * kv.max_pages + pos / kv.page];
    const int64_t off = (((int64_t)pg * Hkv + head) * kv.page + pos % kv.page) * Dh + d;
    gemm::storeW_bf16<W>((is_k ? kv.k : kv.v) + off, v);
  }
};

// SwiGLU over a packed gate/up weight: packed column block t (256 wide) holds
// gate features t*128..t*128+127 then the matching up features. Output
// act[row, f] = silu(rstd*g) * (rstd*u), f = t*128 + j.
struct SwigluParams {
  int M, FF;
  const float* rstd;
  uint16_t* act;  // [M, FF]
  template <int W>
  __device__ void apply(int row, int f, float (&g)[W], const float (&u)[W]) const {
    const float sc = rstd ? rstd[row] : 1.f;
#pragma unroll
    for (int j = 0; j < W; ++j) {
      const float a = g[j] * sc, b = u[j] * sc;
      g[j] = a / (1.f + __expf(-a)) * b;
    }
    gemm::store_rowW<W>(act, FF, 0, row, f, FF, g);
  }
};

// ---------------------------------------------------------------------------
// TMEM-side functors for the GEMM core.
// ---------------------------------------------------------------------------
template <int BN>
struct EpiQKV {
  int M;
  int N;  // total qkv columns
  QkvParams q;
  __device__ void operator()(const gemm::EpiCtx& c) const {
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      float v[32];
      gemm::tmem_ld32(c.taddr + c0, v);
      if (!c.row_ok || c.n0 + c0 >= N) continue;
      q.apply(c.row, c.n0 + c0, v);
    }
  }
};

// BN must be 256: 128 gate columns then 128 up columns.
struct EpiSwiGLU {
  int M;
  SwigluParams p;
  __device__ void operator()(const gemm::EpiCtx& c) const {
    const int f0 = (c.n0 / 256) * 128;
#pragma unroll 1
    for (int c0 = 0; c0 < 128; c0 += 32) {
      float g[32], u[32];
      gemm::tmem_ld32(c.taddr + c0, g);
      gemm::tmem_ld32(c.taddr + 128 + c0, u);
      if (!c.row_ok || f0 + c0 >= p.FF) continue;
      p.apply(c.row, f0 + c0, g, u);
    }
  }
};

// Split-K: raw fp32 partial sums to ws[ks][row][n] (M x N per split).
template <int BN>
struct EpiPartial {
  int M, N;
  float* ws;
  __device__ void operator()(const gemm::EpiCtx& c) const {
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      float v[32];
      gemm::tmem_ld32(c.taddr + c0, v);
      if (!c.row_ok || c.n0 + c0 >= N) continue;
      gemm::store_row32(ws + (int64_t)c.ks * M * N, N, 1, c.row, c.n0 + c0, N, v);
    }
  }
};

}  // namespace dec
