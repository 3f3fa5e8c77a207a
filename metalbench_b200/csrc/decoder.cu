// LLaMA decoder layer on B200: packed weights, fused tcgen05 GEMM epilogues,
// paged-KV attention, optional tensor parallelism over NCCL.
//
// Reference: mlx/kernels/full/llama_decoder_layer.py:24-64 (hook) and
// metal/kernels/full/llama_decoder_layer/default.metal:16-206 (one
// threadgroup computing the whole layer). Here one layer forward is:
//
//   rstd1   = rownorm(x)                      (1 small kernel)
//   q, K, V = RoPE((x @ Wqkv) * rstd1)         (GEMM + QKV epilogue: q -> [T, Dq],
//                                               k, v scattered into the paged cache)
//   a       = attention(q, cache)              (prefill: flash tiles; decode: split-KV)
//   x1      = x + a @ Wo                       (GEMM + residual epilogue; TP: all-reduce)
//   rstd2   = rownorm(x1)
//   act     = silu(g) * u, [g|u] = (x1 @ Wgu) * rstd2   (GEMM + SwiGLU epilogue)
//   y       = x1 + act @ Wdown                 (GEMM + residual epilogue; TP: all-reduce)
//
// The RMSNorm has no gain vector in the reference, so h @ W = rstd * (x @ W)
// and the normalised activations never touch HBM. Weights are packed once, at
// layer creation, into K-major [out, in] bf16 (both tcgen05 operands K-major);
// the gate/up weight is interleaved in blocks of 128 gate + 128 up features so
// that one 256-column tile holds matching gate and up columns. When the GEMM
// has too few output tiles to fill the 148 SMs (decode: 32 rows), it is split
// along K into fp32 partials and a reduce kernel applies the same epilogue.
#include <vector>

#include "decoder_epi.cuh"
#include "gemm_launch.cuh"
#include "kernels.h"

namespace {

// rstd[row] = 1 / sqrt(mean(x[row]^2) + eps); one warp per row, 16-byte loads.
__global__ void rownorm_kernel(const uint16_t* __restrict__ x, int M, int D, float eps,
                               float* __restrict__ rstd) {
  mbd::pdl_trigger();
  mbd::pdl_wait();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const uint4* p = reinterpret_cast<const uint4*>(x + (int64_t)row * D);
  float acc = 0.f;
  for (int c = lane; c < D / 8; c += 32) {
    const uint4 w = p[c];
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const float a = __uint_as_float(ws[m] << 16), b = __uint_as_float(ws[m] & 0xFFFF0000u);
      acc += a * a + b * b;
    }
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) rstd[row] = rsqrtf(acc / (float)D + eps);
}

// Same from an fp32 residual stream (16-byte loads).
__global__ void rownorm_f32_kernel(const float* __restrict__ x, int M, int D, float eps,
                                   float* __restrict__ rstd) {
  mbd::pdl_trigger();
  mbd::pdl_wait();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const float4* p = reinterpret_cast<const float4*>(x + (int64_t)row * D);
  float acc = 0.f;
  for (int c = lane; c < D / 4; c += 32) {
    const float4 w = p[c];
    acc += w.x * w.x + w.y * w.y + w.z * w.z + w.w * w.w;
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) rstd[row] = rsqrtf(acc / (float)D + eps);
}

// Tensor-parallel residual step, one CTA per row: io (bf16) holds the
// all-reduced sum of the ranks' partial outputs; out32 = residual + io in fp32
// (residual from res32, else from the bf16 res16), io = bf16(out32), and with
// rstd_out, rstd_out[row] = rsqrt(mean(out32^2) + eps).
__global__ void residual_add_kernel(uint16_t* __restrict__ io, const float* __restrict__ res32,
                                    const uint16_t* __restrict__ res16, float* __restrict__ out32,
                                    int D, float* __restrict__ rstd_out, float eps) {
  mbd::pdl_trigger();
  mbd::pdl_wait();
  const int64_t row = blockIdx.x;
  float ss = 0.f;
  for (int c = threadIdx.x * 8; c < D; c += blockDim.x * 8) {
    const int64_t off = row * D + c;
    const uint4 a = *reinterpret_cast<const uint4*>(io + off);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
    float v[8];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      v[2 * m] = __uint_as_float(aw[m] << 16);
      v[2 * m + 1] = __uint_as_float(aw[m] & 0xFFFF0000u);
    }
    if (res32) {
      const float4 r0 = *reinterpret_cast<const float4*>(res32 + off);
      const float4 r1 = *reinterpret_cast<const float4*>(res32 + off + 4);
      v[0] += r0.x; v[1] += r0.y; v[2] += r0.z; v[3] += r0.w;
      v[4] += r1.x; v[5] += r1.y; v[6] += r1.z; v[7] += r1.w;
    } else {
      const uint4 r = *reinterpret_cast<const uint4*>(res16 + off);
      const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        v[2 * m] += __uint_as_float(rw[m] << 16);
        v[2 * m + 1] += __uint_as_float(rw[m] & 0xFFFF0000u);
      }
    }
    if (out32) {
      *reinterpret_cast<float4*>(out32 + off) = make_float4(v[0], v[1], v[2], v[3]);
      *reinterpret_cast<float4*>(out32 + off + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
    *reinterpret_cast<uint4*>(io + off) =
        make_uint4(gemm::pack_bf16(v[0], v[1]), gemm::pack_bf16(v[2], v[3]),
                   gemm::pack_bf16(v[4], v[5]), gemm::pack_bf16(v[6], v[7]));
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
  }
  if (!rstd_out) return;
#pragma unroll
  for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  __shared__ float wsum[32];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) wsum[w] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < (int)(blockDim.x + 31) / 32; ++i) t += wsum[i];
    rstd_out[row] = rsqrtf(t / (float)D + eps);
  }
}

// How the fp32 partial slots of a column are summed: split-K (per <= 0): the
// same `slots` splits for every column; stream-K (per > 0): column block
// col/256 was cut into segments by CTAs first..last (first = t*kblocks/per).
struct PartSum {
  int slots;
  int kblocks, per;
  int64_t stride;  // elements per slot (M * N)
  __device__ int count(int col) const {
    if (per <= 0) return slots;
    const int t = col / 256;
    const int first = (int)(((long long)t * kblocks) / per);
    const int last = (int)(((long long)(t + 1) * kblocks - 1) / per);
    return last - first + 1;
  }
};

constexpr int RW = 8;  // columns per thread in the reduce kernels (16-byte bf16 stores)

__device__ __forceinline__ void sum_slots(const float* __restrict__ part, const PartSum& ps, int N,
                                          int row, int col, float (&v)[RW]) {
#pragma unroll
  for (int j = 0; j < RW; ++j) v[j] = 0.f;
  const int n = ps.count(col);
  const float* p0 = part + (int64_t)row * N + col;
  // Whole batches of eight slots: all sixteen 16-byte loads are issued before
  // any add (stream-K at tensor-parallel sizes leaves ~30 slots per column of
  // a narrow GEMM, and these kernels run few threads). The adds stay in slot
  // order 0..n-1 in every case.
  int k0 = 0;
  for (; k0 + 8 <= n; k0 += 8) {
    float4 t[8][RW / 4];
#pragma unroll
    for (int k = 0; k < 8; ++k)
#pragma unroll
      for (int j = 0; j < RW / 4; ++j)
        t[k][j] = __ldcg(reinterpret_cast<const float4*>(p0 + (k0 + k) * ps.stride) + j);
#pragma unroll
    for (int k = 0; k < 8; ++k)
#pragma unroll
      for (int j = 0; j < RW / 4; ++j) {
        v[4 * j] += t[k][j].x;
        v[4 * j + 1] += t[k][j].y;
        v[4 * j + 2] += t[k][j].z;
        v[4 * j + 3] += t[k][j].w;
      }
  }
  for (; k0 < n; k0 += 4) {
    float4 t[4][RW / 4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int j = 0; j < RW / 4; ++j)
        t[k][j] = k0 + k < n ? __ldcg(reinterpret_cast<const float4*>(p0 + (k0 + k) * ps.stride) + j)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int j = 0; j < RW / 4; ++j) {
        v[4 * j] += t[k][j].x;
        v[4 * j + 1] += t[k][j].y;
        v[4 * j + 2] += t[k][j].z;
        v[4 * j + 3] += t[k][j].w;
      }
  }
}

// Split-K / stream-K epilogue: out = scale * sum + residual, one thread per
// (row, 8 columns). With rstd_out, the grid is one CTA per row (N/8 threads)
// and the CTA also writes rstd_out[row] = rsqrt(mean(out^2) + eps) of the
// bf16 values it stored: the next RMSNorm without another pass.
__global__ void reduce_store_kernel(const float* __restrict__ part, PartSum ps, int M, int N,
                                    gemm::EpiStore e, float* __restrict__ rstd_out, float eps) {
  mbd::pdl_trigger();
  mbd::pdl_wait();
  int row, col;
  if (rstd_out) {
    row = blockIdx.x;
    col = threadIdx.x * RW;
  } else {
    const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int chunks = N / RW;
    if (t >= (int64_t)M * chunks) return;
    row = (int)(t / chunks);
    col = (int)(t % chunks) * RW;
  }
  float v[RW];
  sum_slots(part, ps, N, row, col, v);
  const float sc = e.row_scale ? e.row_scale[row] * e.alpha : e.alpha;
#pragma unroll
  for (int j = 0; j < RW; ++j) v[j] *= sc;
  if (e.residual_f32) {
    const float4* r = reinterpret_cast<const float4*>(e.residual_f32 + (int64_t)row * e.ld_res + col);
#pragma unroll
    for (int j = 0; j < RW / 4; ++j) {
      const float4 t = r[j];
      v[4 * j] += t.x;
      v[4 * j + 1] += t.y;
      v[4 * j + 2] += t.z;
      v[4 * j + 3] += t.w;
    }
  } else if (e.residual) {
    const uint4 w = *reinterpret_cast<const uint4*>(e.residual + (int64_t)row * e.ld_res + col);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      v[2 * m] += __uint_as_float(ws[m] << 16);
      v[2 * m + 1] += __uint_as_float(ws[m] & 0xFFFF0000u);
    }
  }
  gemm::store_rowW<RW>(e.out, e.ldo, e.out_f32, row, col, e.N, v);
  if (e.out_f32_copy) gemm::store_rowW<RW>(e.out_f32_copy, e.ldo, 1, row, col, e.N, v);
  if (!rstd_out) return;
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < RW; ++j) {
    // the norm of the residual stream: fp32 when it is kept, else the stored bf16
    const float q = e.out_f32_copy ? v[j] : __bfloat162float(__float2bfloat16_rn(v[j]));
    ss += q * q;
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  __shared__ float wsum[32];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) wsum[w] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < (int)(blockDim.x + 31) / 32; ++i) t += wsum[i];
    rstd_out[row] = rsqrtf(t / (float)N + eps);
  }
}

__global__ void reduce_qkv_kernel(const float* __restrict__ part, PartSum ps, int M, int N,
                                  dec::QkvParams qp) {
  mbd::pdl_trigger();
  mbd::pdl_wait();
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int chunks = N / RW;
  if (t >= (int64_t)M * chunks) return;
  const int row = (int)(t / chunks), col = (int)(t % chunks) * RW;
  float v[RW];
  sum_slots(part, ps, N, row, col, v);
  qp.apply<RW>(row, col, v);
}

// N = 2*FF packed columns; thread per (row, 8 output features).
__global__ void reduce_swiglu_kernel(const float* __restrict__ part, PartSum ps, int M, int N,
                                     dec::SwigluParams sp) {
  mbd::pdl_trigger();
  mbd::pdl_wait();
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int chunks = sp.FF / RW;
  if (t >= (int64_t)M * chunks) return;
  const int row = (int)(t / chunks), f = (int)(t % chunks) * RW;
  const int gcol = (f / 128) * 256 + f % 128;
  float g[RW], u[RW];
  sum_slots(part, ps, N, row, gcol, g);
  sum_slots(part, ps, N, row, gcol + 128, u);
  sp.apply<RW>(row, f, g, u);
}

// Tile a K-major bf16 [N, K] weight for bulk-copy streaming (layout: see
// tiled_weight_bytes in gemm_launch.cuh).
__global__ void tile_weights_kernel(const uint16_t* __restrict__ w, int64_t N, int64_t K, int BN,
                                    uint8_t* __restrict__ out) {
  const int64_t kblocks = K / 64;
  const int64_t tiles_n = (N + BN - 1) / BN;
  const int64_t chunks = tiles_n * kblocks * BN * 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < chunks;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tile = i / (BN * 8);
    const int r = (int)((i / 8) % BN), c = (int)(i % 8);
    const int64_t tn = tile / kblocks, kb = tile % kblocks;
    const int64_t n = tn * BN + r;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (n < N) v = *reinterpret_cast<const uint4*>(w + n * K + kb * 64 + c * 8);
    *reinterpret_cast<uint4*>(out + tile * (BN * gemm::KBYTES) + r * gemm::KBYTES + ((c ^ (r & 7)) * 16)) = v;
  }
}


// Direct pack into the tiled, pre-swizzled layout: 16-byte chunk c of row r of
// tile (tn, kb) gathers in[(kb*64 + c*8 + j) * ld_in + col_idx[tn*256 + r]],
// j = 0..7 (rows past Nout are zero). One-time weight preparation.
__global__ void pack_tiled_kernel(const uint16_t* __restrict__ in, int64_t ld_in, int K,
                                  const int* __restrict__ col_idx, int Nout,
                                  uint8_t* __restrict__ out) {
  const int64_t kblocks = K / 64, tiles_n = (Nout + 255) / 256;
  const int64_t chunks = tiles_n * kblocks * 256 * 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < chunks;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tile = i / (256 * 8);
    const int r = (int)((i / 8) % 256), c = (int)(i % 8);
    const int64_t tn = tile / kblocks, kb = tile % kblocks;
    const int64_t n = tn * 256 + r;
    uint32_t w[4] = {0, 0, 0, 0};
    if (n < Nout) {
      const int64_t col = col_idx[n];
      const int64_t k0 = kb * 64 + c * 8;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        w[j] = (uint32_t)in[(k0 + 2 * j) * ld_in + col] |
               ((uint32_t)in[(k0 + 2 * j + 1) * ld_in + col] << 16);
    }
    *reinterpret_cast<uint4*>(out + tile * (256 * gemm::KBYTES) + r * gemm::KBYTES +
                              ((c ^ (r & 7)) * 16)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// out[n][k] = in[k * ld_in + col_idx[n]] for k < K: packs selected columns of a
// row-major (in, out) weight into a K-major [n, K] operand (32x32 smem tiles).
__global__ void pack_cols_kernel(const uint16_t* __restrict__ in, int64_t ld_in, int K,
                                 const int* __restrict__ col_idx, int Nout,
                                 uint16_t* __restrict__ out) {
  __shared__ uint16_t T[32][34];
  const int k0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int r = ty; r < 32; r += 8)
    if (k0 + r < K && n0 + tx < Nout) T[r][tx] = in[(int64_t)(k0 + r) * ld_in + col_idx[n0 + tx]];
  __syncthreads();
  for (int r = ty; r < 32; r += 8)
    if (n0 + r < Nout && k0 + tx < K) out[(int64_t)(n0 + r) * K + k0 + tx] = T[tx][r];
}

}  // namespace

namespace {

using namespace gemm;

struct Layer {
  mb_decoder_config cfg;
  int rank, world;
  int Hq, Hkv, Dq, Dkv, FF;  // per-rank
  uint16_t *wqkv, *wo, *wgu, *wdown;  // packed K-major
};

int upload_idx(const std::vector<int>& v, int** d) {
  MB_CUDA(cudaMalloc(d, v.size() * sizeof(int)));
  MB_CUDA(cudaMemcpy(*d, v.data(), v.size() * sizeof(int), cudaMemcpyHostToDevice));
  return MB_OK;
}

// Selected columns of a reference (in, out) weight -> K-major [N, K] -> the
// tiled, pre-swizzled layout every decoder GEMM streams (256-row tiles).
int pack(const uint16_t* in, int64_t ld_in, int K, const std::vector<int>& cols, uint16_t** out) {
  int* idx = nullptr;
  int rc = upload_idx(cols, &idx);
  if (rc) return rc;
  const int N = (int)cols.size();
  MB_REQUIRE(K % 64 == 0, "decoder: GEMM inner dimension %d is not a multiple of 64", K);
  uint16_t* kmajor = nullptr;
  MB_CUDA(cudaMalloc(&kmajor, (size_t)N * K * 2));
  dim3 g((N + 31) / 32, (K + 31) / 32);
  pack_cols_kernel<<<g, 256>>>(in, ld_in, K, idx, N, kmajor);
  MB_CUDA(cudaGetLastError());
  MB_CUDA(cudaMalloc(out, tiled_weight_bytes(N, K, 256)));
  tile_weights_kernel<<<1024, 256>>>(kmajor, N, K, 256, reinterpret_cast<uint8_t*>(*out));
  MB_CUDA(cudaGetLastError());
  MB_CUDA(cudaDeviceSynchronize());
  MB_CUDA(cudaFree(idx));
  MB_CUDA(cudaFree(kmajor));
  return MB_OK;
}

// Decode-size GEMMs (one tile row, fewer than two tiles per SM) run
// stream-K: every SM streams the same number of weight k-blocks instead of
// whole tiles (e.g. 112 gate/up tiles would leave 36 of 148 SMs idle).
bool use_streamk(int64_t M, int64_t N) {
  return M <= BM && ((N + 255) / 256) < 2 * mb::num_sms();
}

int choose_ksplit(int64_t M, int64_t N, int64_t K) {
  const int sms = mb::num_sms();
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + 255) / 256);
  const int kb = (int)((K + 63) / 64);
  if (tiles * 2 > sms) return 1;
  int ks = (int)(sms / tiles);
  if (ks > kb / 4) ks = kb / 4;  // keep at least 4 k-blocks per split
  if (ks <= 1) return 1;
  const int per = (kb + ks - 1) / ks;  // same normalisation as launch_gemm
  return (kb + per - 1) / per;
}

struct Plan {
  int64_t T;
  int ks_qkv, ks_o, ks_gu, ks_down;
  size_t off_rstd1, off_rstd2, off_q, off_attn, off_x1, off_x1f, off_p32, off_act, off_part,
      off_attn_ws, total;
  size_t attn_ws;
};

size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

Plan make_plan(const Layer& L, int B, int S, int max_kv_len) {
  Plan p;
  const int D = L.cfg.d_model;
  p.T = (int64_t)B * S;
  const int64_t T = p.T;
  const int Nqkv = L.Dq + 2 * L.Dkv;
  p.ks_qkv = choose_ksplit(T, Nqkv, D);
  p.ks_o = choose_ksplit(T, D, L.Dq);
  p.ks_gu = choose_ksplit(T, 2 * L.FF, D);
  p.ks_down = choose_ksplit(T, D, L.FF);
  size_t part = 0;
  auto upd = [&](int ks, int64_t N) {
    if (ks > 1) part = std::max(part, (size_t)ks * T * N * 4);
  };
  auto upd_sk = [&](int64_t N, int64_t K) {
    if (!use_streamk(T, N)) return;
    const StreamK pl = streamk_plan((int)((N + 255) / 256), (int)((K + 63) / 64), mb::num_sms());
    part = std::max(part, (size_t)pl.max_segs * T * N * 4);
  };
  upd_sk(Nqkv, D);
  upd_sk(D, L.Dq);
  upd_sk(2 * L.FF, D);
  upd_sk(D, L.FF);
  upd(p.ks_qkv, Nqkv);
  upd(p.ks_o, D);
  upd(p.ks_gu, 2 * L.FF);
  upd(p.ks_down, D);
  p.attn_ws = S == 1 ? mb_attention_decode_workspace_bytes(B, L.Hq, L.Hkv, max_kv_len) : 0;
  size_t o = 0;
  p.off_rstd1 = o; o += a256(T * 4);
  p.off_rstd2 = o; o += a256(T * 4);
  p.off_q = o; o += a256(T * L.Dq * 2);
  p.off_attn = o; o += a256(T * L.Dq * 2);
  p.off_x1 = o; o += a256(T * D * 2);
  p.off_x1f = o; o += a256(T * D * 4);
  p.off_p32 = o; o += L.world > 1 ? a256(T * D * 4) : 0;  // this rank's fp32 partial product
  p.off_act = o; o += a256(T * L.FF * 2);
  p.off_part = o; o += a256(part);
  p.off_attn_ws = o; o += a256(p.attn_ws);
  p.total = o;
  return p;
}

template <class Epi>
int gemm_call(const uint16_t* A, const uint16_t* Bw, const Epi& e, int64_t M, int64_t N, int64_t K,
              cudaStream_t s) {
  return launch_gemm<Mode::BF16, 256, 4, false>(A, Bw, e, M, N, K, 1, s, false, true);
}

// Partial sums of A @ Bw^T into fp32 slots of part ([slot][M][N]): stream-K
// for decode sizes, else split-K with `ks` splits. *ps tells the epilogue
// kernels how many slots each column sums.
int gemm_partial(const uint16_t* A, const uint16_t* Bw, float* part, int64_t M, int64_t N,
                 int64_t K, int ks, cudaStream_t s, PartSum* ps) {
  dec::EpiPartial<256> e;
  e.M = (int)M;
  e.N = (int)N;
  e.ws = part;
  ps->stride = M * N;
  ps->kblocks = (int)((K + 63) / 64);
  if (use_streamk(M, N)) {
    const StreamK pl = streamk_plan((int)((N + 255) / 256), ps->kblocks, mb::num_sms());
    ps->per = pl.per;
    ps->slots = 0;
    if (M <= 64) return launch_gemm_decode<256, 5>(A, Bw, e, M, N, K, s, true);
    return launch_gemm<Mode::BF16, 256, 4, false>(A, Bw, e, M, N, K, 1, s, true, true);
  }
  ps->per = 0;
  ps->slots = ks;
  return launch_gemm<Mode::BF16, 256, 4, false>(A, Bw, e, M, N, K, ks, s, false, true);
}

unsigned blocks_for(int64_t threads) { return (unsigned)((threads + 255) / 256); }



}  // namespace

namespace mb {
// Shared with the standalone fused ops (fused_ops.cu).
int rownorm(const uint16_t* x, int M, int D, float eps, float* rstd, cudaStream_t s) {
  MB_REQUIRE(D % 8 == 0, "rownorm: D must be a multiple of 8");
  rownorm_kernel<<<(unsigned)((M + 7) / 8), 256, 0, s>>>(x, M, D, eps, rstd);
  MB_CUDA(cudaGetLastError());
  return MB_OK;
}
int pack_tiled_weight(const uint16_t* in, int64_t ld_in, int K, const int* col_idx_dev, int Nout,
                      uint8_t* out, cudaStream_t s) {
  MB_REQUIRE(K % 64 == 0, "weight packing: K must be a multiple of 64");
  pack_tiled_kernel<<<1024, 256, 0, s>>>(in, ld_in, K, col_idx_dev, Nout, out);
  MB_CUDA(cudaGetLastError());
  return MB_OK;
}
}  // namespace mb

extern "C" int mb_decoder_layer_create(const mb_decoder_config* cfg, const uint16_t* W_qkv,
                                       const uint16_t* W_o, const uint16_t* W_gu,
                                       const uint16_t* W_down, int tp_rank, int tp_world,
                                       void** layer) {
  MB_REQUIRE(cfg && layer && W_qkv && W_o && W_gu && W_down, "decoder create: null argument");
  const int D = cfg->d_model, H = cfg->n_heads, Hkv = cfg->n_kv_heads, Dh = cfg->head_dim,
            FF = cfg->ffn;
  MB_REQUIRE(Dh == 128, "decoder: head_dim must be 128");
  MB_REQUIRE(H * Dh == D, "decoder: n_heads * head_dim must equal d_model");
  MB_REQUIRE(Hkv > 0 && H % Hkv == 0, "decoder: n_heads must be a multiple of n_kv_heads");
  MB_REQUIRE(tp_world >= 1 && tp_rank >= 0 && tp_rank < tp_world, "decoder: bad tp rank/world");
  MB_REQUIRE(Hkv % tp_world == 0, "decoder: n_kv_heads must be divisible by the TP size");
  MB_REQUIRE(FF % (128 * tp_world) == 0, "decoder: ffn must be a multiple of 128 * TP size");
  MB_REQUIRE(D % 256 == 0, "decoder: d_model must be a multiple of 256");
  Layer* L = new Layer();
  L->cfg = *cfg;
  L->rank = tp_rank;
  L->world = tp_world;
  L->Hq = H / tp_world;
  L->Hkv = Hkv / tp_world;
  L->Dq = L->Hq * Dh;
  L->Dkv = L->Hkv * Dh;
  L->FF = FF / tp_world;
  const int Ntot = D + 2 * Hkv * Dh;
  std::vector<int> cols;
  for (int c = 0; c < L->Dq; ++c) cols.push_back(tp_rank * L->Dq + c);
  for (int c = 0; c < L->Dkv; ++c) cols.push_back(D + tp_rank * L->Dkv + c);
  for (int c = 0; c < L->Dkv; ++c) cols.push_back(D + Hkv * Dh + tp_rank * L->Dkv + c);
  int rc = pack(W_qkv, Ntot, D, cols, &L->wqkv);
  std::vector<int> ident(D);
  for (int c = 0; c < D; ++c) ident[c] = c;
  if (!rc) rc = pack(W_o + (int64_t)tp_rank * L->Dq * D, D, L->Dq, ident, &L->wo);
  std::vector<int> gu;
  for (int p = 0; p < 2 * L->FF; ++p) {
    const int t = p / 256, w = p % 256;
    const int f = tp_rank * L->FF + t * 128 + (w % 128);
    gu.push_back(w < 128 ? f : FF + f);
  }
  if (!rc) rc = pack(W_gu, 2 * FF, D, gu, &L->wgu);
  if (!rc) rc = pack(W_down + (int64_t)tp_rank * L->FF * D, D, L->FF, ident, &L->wdown);
  if (rc) {
    delete L;
    return rc;
  }
  *layer = L;
  return MB_OK;
}

extern "C" void mb_decoder_layer_destroy(void* layer) {
  Layer* L = static_cast<Layer*>(layer);
  if (!L) return;
  cudaFree(L->wqkv);
  cudaFree(L->wo);
  cudaFree(L->wgu);
  cudaFree(L->wdown);
  delete L;
}

extern "C" size_t mb_decoder_layer_workspace_bytes(const void* layer, int B, int S,
                                                   int max_kv_len) {
  if (!layer || B <= 0 || S <= 0) return 0;
  return make_plan(*static_cast<const Layer*>(layer), B, S, max_kv_len).total;
}

namespace {
int decoder_forward(const void* layer, const uint16_t* x, const float* x_res32, uint16_t* y,
                    float* y_res32, const float* rstd_in, float* rstd_out, int B, int S,
                    const int* start_pos, const int* kv_len, int max_kv_len, uint16_t* k_cache,
                    uint16_t* v_cache, const int* block_table, int max_pages, int causal,
                    void* workspace, size_t workspace_bytes, void* stream) {
  MB_REQUIRE(layer && x && y && start_pos && kv_len && k_cache && v_cache && block_table,
             "decoder forward: null argument");
  MB_REQUIRE(!rstd_out || y_res32, "decoder forward: rstd_out needs the fp32 output y_res32");
  MB_REQUIRE(B >= 0 && S >= 0, "decoder forward: negative size");
  if (B == 0 || S == 0) return MB_OK;
  const Layer& L = *static_cast<const Layer*>(layer);
  MB_REQUIRE(max_kv_len >= S && max_kv_len <= max_pages * 64,
             "decoder forward: max_kv_len must be in [S, max_pages*64]");
  MB_REQUIRE((reinterpret_cast<uintptr_t>(x_res32) | reinterpret_cast<uintptr_t>(y_res32)) % 16 == 0,
             "decoder forward: fp32 residual buffers must be 16-byte aligned");
  const Plan p = make_plan(L, B, S, max_kv_len);
  MB_REQUIRE(workspace && workspace_bytes >= p.total &&
                 reinterpret_cast<uintptr_t>(workspace) % 256 == 0,
             "decoder forward: workspace of %zu bytes (256-byte aligned) required", p.total);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  float* rstd1 = reinterpret_cast<float*>(w + p.off_rstd1);
  float* rstd2 = reinterpret_cast<float*>(w + p.off_rstd2);
  uint16_t* q = reinterpret_cast<uint16_t*>(w + p.off_q);
  uint16_t* attn = reinterpret_cast<uint16_t*>(w + p.off_attn);
  uint16_t* x1 = reinterpret_cast<uint16_t*>(w + p.off_x1);
  float* x1f = reinterpret_cast<float*>(w + p.off_x1f);  // fp32 residual stream after attention
  float* p32 = reinterpret_cast<float*>(w + p.off_p32);
  uint16_t* act = reinterpret_cast<uint16_t*>(w + p.off_act);
  float* part = reinterpret_cast<float*>(w + p.off_part);
  const int D = L.cfg.d_model, Dh = L.cfg.head_dim;
  const int64_t T = p.T;
  const int Nqkv = L.Dq + 2 * L.Dkv;
  const bool tp = L.world > 1;
  // tensor parallel: fp32 partials summed over NVLink peer memory together
  // with the residual step (else a bf16 NCCL all-reduce, then the residual)
  const bool fused = tp && mb::tp_fused_ready((size_t)T, D);
  if (fused) p32 = mb::tp_partial_slot();  // the partial goes straight to peer-mapped memory
  int rc;

  // 1. rstd1 (of the fp32 residual stream when the caller keeps one), unless
  // the previous layer of a stack already produced it
  if (rstd_in)
    rstd1 = const_cast<float*>(rstd_in);
  else if (x_res32)
    MB_CUDA(mb::launch_pdl(rownorm_f32_kernel, dim3((unsigned)((T + 7) / 8)), dim3(256), 0, s,
                            x_res32, (int)T, D, L.cfg.eps, rstd1));
  else
    MB_CUDA(mb::launch_pdl(rownorm_kernel, dim3((unsigned)((T + 7) / 8)), dim3(256), 0, s, x,
                            (int)T, D, L.cfg.eps, rstd1));

  // 2. QKV + RoPE + KV-cache write
  dec::QkvParams qp;
  qp.M = (int)T;
  qp.S = S;
  qp.Hq = L.Hq;
  qp.Hkv = L.Hkv;
  qp.Dh = Dh;
  qp.neg_log2_base_over_half = -log2f(L.cfg.rope_base) / (float)(Dh / 2);
  qp.rstd = rstd1;
  qp.start_pos = start_pos;
  qp.q_out = q;
  qp.kv = dec::KvCache{k_cache, v_cache, block_table, max_pages, 64};
  if (p.ks_qkv > 1 || use_streamk(T, Nqkv)) {
    PartSum ps;
    rc = gemm_partial(x, L.wqkv, part, T, Nqkv, D, p.ks_qkv, s, &ps);
    if (rc) return rc;
    MB_CUDA(mb::launch_pdl(reduce_qkv_kernel, dim3(blocks_for(T * Nqkv / RW)), dim3(256), 0, s,
                            part, ps, (int)T, Nqkv, qp));
  } else {
    dec::EpiQKV<256> e;
    e.M = (int)T;
    e.N = Nqkv;
    e.q = qp;
    rc = gemm_call(x, L.wqkv, e, T, Nqkv, D, s);
    if (rc) return rc;
  }
  MB_CUDA(cudaGetLastError());

  // 3. attention
  if (S == 1)
    rc = mb_attention_decode_bf16(q, L.Dq, k_cache, v_cache, block_table, max_pages, kv_len,
                                  max_kv_len, B, L.Hq, L.Hkv, Dh, attn, L.Dq, w + p.off_attn_ws,
                                  p.attn_ws, s);
  else
    rc = mb_attention_prefill_bf16(q, L.Dq, k_cache, v_cache, block_table, max_pages, start_pos,
                                   kv_len, B, S, L.Hq, L.Hkv, Dh, causal, attn, L.Dq, s);
  if (rc) return rc;

  // The residual stream is added in fp32 and kept in fp32 (x1f); its bf16
  // copy x1 is the next GEMM's operand. One GPU: the o-proj epilogue adds
  // it. Tensor parallel: the ranks' fp32 partial products (no residual) are
  // summed over NVLink peer memory by tp_reduce_residual, which also adds
  // the residual (messages too large for its slots: bf16 NCCL all-reduce,
  // then residual_add_kernel).
  bool rstd2_done = false;
  // 4. x1 = x + attn @ Wo
  EpiStore eo{};
  eo.M = (int)T;
  eo.N = D;
  eo.out = x1;
  eo.ldo = D;
  eo.alpha = 1.f;
  eo.ld_res = D;
  if (!tp) {
    eo.residual = x_res32 ? nullptr : x;
    eo.residual_f32 = x_res32;
    eo.out_f32_copy = x1f;
  } else if (fused) {
    eo.out = p32;
    eo.out_f32 = 1;
  }
  if (p.ks_o > 1 || use_streamk(T, D)) {
    PartSum ps;
    rc = gemm_partial(attn, L.wo, part, T, D, L.Dq, p.ks_o, s, &ps);
    if (rc) return rc;
    if (!tp && D / RW <= 1024) {  // the reduce also yields rstd2 (one CTA per row)
      MB_CUDA(mb::launch_pdl(reduce_store_kernel, dim3((unsigned)T), dim3(D / RW), 0, s, part, ps,
                              (int)T, D, eo, rstd2, L.cfg.eps));
      rstd2_done = true;
    } else {
      MB_CUDA(mb::launch_pdl(reduce_store_kernel, dim3(blocks_for(T * D / RW)), dim3(256), 0, s,
                              part, ps, (int)T, D, eo, (float*)nullptr, 0.f));
    }
  } else {
    Epi<256, EpiStore> e{};
    static_cast<EpiStore&>(e) = eo;
    rc = gemm_call(attn, L.wo, e, T, D, L.Dq, s);
    if (rc) return rc;
  }
  MB_CUDA(cudaGetLastError());
  if (fused) {
    rc = mb::tp_reduce_residual(p32, T, D, x_res32, x, x1f, x1, rstd2, L.cfg.eps, s);
    if (rc) return rc;
    rstd2_done = true;
  } else if (tp) {
    rc = mb::tp_allreduce_sum(x1, (size_t)T * D, s);
    if (rc) return rc;
    MB_CUDA(mb::launch_pdl(residual_add_kernel, dim3((unsigned)T), dim3(256), 0, s, x1, x_res32,
                            x, x1f, D, rstd2, L.cfg.eps));
    rstd2_done = true;
  }

  // 5. rstd2 (unless produced above), 6. SwiGLU MLP up
  if (!rstd2_done) {
    MB_CUDA(mb::launch_pdl(rownorm_f32_kernel, dim3((unsigned)((T + 7) / 8)), dim3(256), 0, s,
                            (const float*)x1f, (int)T, D, L.cfg.eps, rstd2));
  }
  dec::SwigluParams sp;
  sp.M = (int)T;
  sp.FF = L.FF;
  sp.rstd = rstd2;
  sp.act = act;
  if (p.ks_gu > 1 || use_streamk(T, 2 * L.FF)) {
    PartSum ps;
    rc = gemm_partial(x1, L.wgu, part, T, 2 * L.FF, D, p.ks_gu, s, &ps);
    if (rc) return rc;
    MB_CUDA(mb::launch_pdl(reduce_swiglu_kernel, dim3(blocks_for(T * L.FF / RW)), dim3(256), 0, s,
                            part, ps, (int)T, 2 * L.FF, sp));
  } else {
    dec::EpiSwiGLU e;
    e.M = (int)T;
    e.p = sp;
    rc = gemm_call(x1, L.wgu, e, T, 2 * L.FF, D, s);
    if (rc) return rc;
  }
  MB_CUDA(cudaGetLastError());

  // 7. y = x1 + act @ Wdown
  EpiStore ed{};
  ed.M = (int)T;
  ed.N = D;
  ed.out = y;
  ed.ldo = D;
  ed.alpha = 1.f;
  ed.ld_res = D;
  if (!tp) {
    ed.residual_f32 = x1f;
    ed.out_f32_copy = y_res32;
  } else if (fused) {
    ed.out = p32;
    ed.out_f32 = 1;
  }
  if (p.ks_down > 1 || use_streamk(T, D)) {
    PartSum ps;
    rc = gemm_partial(act, L.wdown, part, T, D, L.FF, p.ks_down, s, &ps);
    if (rc) return rc;
    // (one CTA per row could also yield the next rstd1, but at T = 64 that
    // leaves most SMs idle in a latency-bound reduce: rownorm follows instead)
    MB_CUDA(mb::launch_pdl(reduce_store_kernel, dim3(blocks_for(T * D / RW)), dim3(256), 0, s,
                            part, ps, (int)T, D, ed, (float*)nullptr, 0.f));
  } else {
    Epi<256, EpiStore> e{};
    static_cast<EpiStore&>(e) = ed;
    rc = gemm_call(act, L.wdown, e, T, D, L.FF, s);
    if (rc) return rc;
  }
  MB_CUDA(cudaGetLastError());
  // rstd_out: the next layer's rstd1, rsqrt(mean(y_res32^2) + eps), from the
  // kernel that forms the output row under tensor parallelism (the peer
  // reduce, the residual add); on one GPU by rownorm_f32_kernel, the same
  // launch on the same input that the next layer would otherwise make
  if (fused) {
    rc = mb::tp_reduce_residual(p32, T, D, x1f, nullptr, y_res32, y, rstd_out, L.cfg.eps, s);
    if (rc) return rc;
  } else if (tp) {
    rc = mb::tp_allreduce_sum(y, (size_t)T * D, s);
    if (rc) return rc;
    MB_CUDA(mb::launch_pdl(residual_add_kernel, dim3((unsigned)T), dim3(256), 0, s, y,
                            (const float*)x1f, (const uint16_t*)nullptr, y_res32, D, rstd_out,
                            L.cfg.eps));
  } else if (rstd_out) {
    MB_CUDA(mb::launch_pdl(rownorm_f32_kernel, dim3((unsigned)((T + 7) / 8)), dim3(256), 0, s,
                            (const float*)y_res32, (int)T, D, L.cfg.eps, rstd_out));
  }
  return MB_OK;
}
}  // namespace

extern "C" int mb_decoder_layer_forward_ex(const void* layer, const uint16_t* x,
                                           const float* x_res32, uint16_t* y, float* y_res32,
                                           int B, int S, const int* start_pos, const int* kv_len,
                                           int max_kv_len, uint16_t* k_cache, uint16_t* v_cache,
                                           const int* block_table, int max_pages, int causal,
                                           void* workspace, size_t workspace_bytes,
                                           void* stream) {
  return decoder_forward(layer, x, x_res32, y, y_res32, nullptr, nullptr, B, S, start_pos, kv_len,
                         max_kv_len, k_cache, v_cache, block_table, max_pages, causal, workspace,
                         workspace_bytes, stream);
}

extern "C" int mb_decoder_layer_forward_chain(const void* layer, const uint16_t* x,
                                              const float* x_res32, const float* rstd_in,
                                              uint16_t* y, float* y_res32, float* rstd_out, int B,
                                              int S, const int* start_pos, const int* kv_len,
                                              int max_kv_len, uint16_t* k_cache,
                                              uint16_t* v_cache, const int* block_table,
                                              int max_pages, int causal, void* workspace,
                                              size_t workspace_bytes, void* stream) {
  return decoder_forward(layer, x, x_res32, y, y_res32, rstd_in, rstd_out, B, S, start_pos,
                         kv_len, max_kv_len, k_cache, v_cache, block_table, max_pages, causal,
                         workspace, workspace_bytes, stream);
}

extern "C" int mb_decoder_layer_forward(const void* layer, const uint16_t* x, uint16_t* y, int B,
                                        int S, const int* start_pos, const int* kv_len,
                                        int max_kv_len, uint16_t* k_cache, uint16_t* v_cache,
                                        const int* block_table, int max_pages, int causal,
                                        void* workspace, size_t workspace_bytes, void* stream) {
  return mb_decoder_layer_forward_ex(layer, x, nullptr, y, nullptr, B, S, start_pos, kv_len,
                                     max_kv_len, k_cache, v_cache, block_table, max_pages, causal,
                                     workspace, workspace_bytes, stream);
}
