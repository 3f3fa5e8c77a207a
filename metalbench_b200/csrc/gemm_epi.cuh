// Epilogue functors for the tcgen05 GEMM core. Each runs in the four
// epilogue warps; thread (warp w, lane l) owns accumulator row 32*(w%4)+l and
// reads it from TMEM 32 columns at a time. tcgen05.ld is warp-collective, so
// every lane issues the loads and only the stores are predicated.
#pragma once
#include "gemm_core.cuh"

namespace gemm {

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[16], s[16];
  mbd::tmem_ld16(taddr, r);
  mbd::tmem_ld16(taddr + 16, s);
  mbd::tmem_ld_wait();
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    v[j] = __uint_as_float(r[j]);
    v[16 + j] = __uint_as_float(s[j]);
  }
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);  // .x = a (low half)
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(((uint32_t)b) << 16);
}

// Store W consecutive values of one row (bf16 or fp32): vectorised when fully
// in range and 16-byte aligned, element-wise with bounds checks otherwise.
template <int W>
__device__ __forceinline__ void store_rowW(void* out, int64_t ldo, int out_f32, int row, int n,
                                           int N, const float (&v)[W]) {
  if (out_f32) {
    float* p = reinterpret_cast<float*>(out) + (int64_t)row * ldo + n;
    if (n + W <= N && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
#pragma unroll
      for (int j = 0; j < W; j += 4)
        *reinterpret_cast<float4*>(p + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < W; ++j)
        if (n + j < N) p[j] = v[j];
    }
  } else {
    uint16_t* p = reinterpret_cast<uint16_t*>(out) + (int64_t)row * ldo + n;
    if (n + W <= N && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
#pragma unroll
      for (int j = 0; j < W; j += 8) {
        uint4 w;
        w.x = pack_bf16(v[j], v[j + 1]);
        w.y = pack_bf16(v[j + 2], v[j + 3]);
        w.z = pack_bf16(v[j + 4], v[j + 5]);
        w.w = pack_bf16(v[j + 6], v[j + 7]);
        *reinterpret_cast<uint4*>(p + j) = w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < W; ++j)
        if (n + j < N) {
          __nv_bfloat16 h = __float2bfloat16_rn(v[j]);
          p[j] = *reinterpret_cast<uint16_t*>(&h);
        }
    }
  }
}

__device__ __forceinline__ void store_row32(void* out, int64_t ldo, int out_f32, int row, int n,
                                            int N, const float (&v)[32]) {
  store_rowW<32>(out, ldo, out_f32, row, n, N, v);
}

// W bf16 values to p (vectorised when 16-byte aligned).
template <int W>
__device__ __forceinline__ void storeW_bf16(uint16_t* p, const float (&v)[W]) {
  if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
#pragma unroll
    for (int j = 0; j < W; j += 8) {
      uint4 w;
      w.x = pack_bf16(v[j], v[j + 1]);
      w.y = pack_bf16(v[j + 2], v[j + 3]);
      w.z = pack_bf16(v[j + 4], v[j + 5]);
      w.w = pack_bf16(v[j + 6], v[j + 7]);
      *reinterpret_cast<uint4*>(p + j) = w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < W; ++j) {
      __nv_bfloat16 h = __float2bfloat16_rn(v[j]);
      p[j] = *reinterpret_cast<uint16_t*>(&h);
    }
  }
}

// out[row, n] = act(alpha * row_scale[row] * acc[row, n]) (+ residual[row, n]),
// stored as bf16 or fp32. row_scale and residual are optional (null).
struct EpiStore {
  int M, N;
  void* out;
  int64_t ldo;
  int out_f32;
  float alpha;
  const float* row_scale;
  const uint16_t* residual;  // bf16 [M, ld_res]
  int64_t ld_res;
  int act;  // 0: none; 1: exact GELU x*Phi(x), applied after the scale, before the residual
  // fp32 residual stream (optional): residual_f32 [M, ld_res] is added instead
  // of the bf16 residual, and out_f32_copy [M, ldo] receives the fp32 result
  // beside the (bf16) out.
  const float* residual_f32;
  float* out_f32_copy;
  // Scale, add the residual and store 32 accumulator values of row c.row
  // starting at column n.
  __device__ void finish32(const EpiCtx& c, float sc, int n, float (&v)[32]) const {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] *= sc;
    if (act == 1) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = 0.5f * v[j] * (1.f + erff(v[j] * 0.70710678118654752f));
    }
    if (residual_f32) {
      const float* r = residual_f32 + (int64_t)c.row * ld_res + n;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n + j < N) v[j] += r[j];
    } else if (residual) {
      const uint16_t* r = residual + (int64_t)c.row * ld_res + n;
      if (n + 32 <= N && (reinterpret_cast<uintptr_t>(r) & 15) == 0) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          const uint4 w = *reinterpret_cast<const uint4*>(r + j);
          const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            v[j + 2 * m] += __uint_as_float(ws[m] << 16);
            v[j + 2 * m + 1] += __uint_as_float(ws[m] & 0xFFFF0000u);
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (n + j < N) v[j] += bf16_bits_to_f32(r[j]);
      }
    }
    store_row32(out, ldo, out_f32, c.row, n, N, v);
    if (out_f32_copy) store_row32(out_f32_copy, ldo, 1, c.row, n, N, v);
  }
  __device__ float scale(const EpiCtx& c) const {
    return (c.row_ok && row_scale) ? row_scale[c.row] * alpha : alpha;
  }
  template <int BN>
  __device__ void run(const EpiCtx& c) const {
    const float sc = scale(c);
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      float v[32];
      tmem_ld32(c.taddr + c0, v);
      const int n = c.n0 + c0;
      if (!c.row_ok || n >= N) continue;
      finish32(c, sc, n, v);
    }
  }
  // Same, from an accumulator the kernel summed in registers (PROMOTE mode).
  template <int BN>
  __device__ void run_acc(const EpiCtx& c, const float (&acc)[BN]) const {
    if (!c.row_ok) return;
    const float sc = scale(c);
#pragma unroll
    for (int c0 = 0; c0 < BN; c0 += 32) {
      const int n = c.n0 + c0;
      if (n < N) {
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = acc[c0 + j];
        finish32(c, sc, n, v);
      }
    }
  }
};

// Adapter: the kernel calls epi(ctx); BN is fixed per instantiation.
template <int BN, class E>
struct Epi : E {
  __device__ void operator()(const EpiCtx& c) const { E::template run<BN>(c); }
  __device__ void store_acc(const EpiCtx& c, const float (&acc)[BN]) const {
    E::template run_acc<BN>(c, acc);
  }
};

}  // namespace gemm
