// Out-of-place transpose for sm_100a: 64x64 tiles staged through an
// XOR-swizzled shared-memory tile, 16-byte global loads and stores.
//
// Reference: metal/kernels/common/transpose_2d/default.metal:10-48 (64x64 tile,
// float4 row loads, padded tile[64][65]); hook mlx/kernels/common/transpose_2d.py.
//
// Layout in shared memory: the tile is stored already transposed, T[c][r]
// (one 32-bit word per fp32 element; one word per PAIR of input rows for bf16),
// with the word index XOR-ed by 4*((c/G)%8). That swizzle makes both the
// scalar word stores (lanes spread over 8 column chunks x 4 rows) and the
// 16-byte row reads hit 32 distinct banks, with no padding, so every phase
// moves 16 B per thread per instruction on the global side.
#include "common.cuh"

namespace {

constexpr int TILE = 64;
constexpr int THREADS = 256;

// ---------------------------------------------------------------------------
// fp32: T is 64 (out rows c) x 64 (words r) = 16 KiB.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(THREADS) transpose_f32_kernel(const float* __restrict__ in,
                                                                float* __restrict__ out,
                                                                int64_t rows, int64_t cols,
                                                                int vec_ok) {
  __shared__ __align__(16) uint32_t T[TILE * TILE];
  const int64_t b = blockIdx.z;
  const float* src = in + b * rows * cols;
  float* dst = out + b * rows * cols;
  const int64_t r0 = (int64_t)blockIdx.y * TILE, c0 = (int64_t)blockIdx.x * TILE;
  const int t = threadIdx.x, w = t >> 5, l = t & 31;
  const bool full = vec_ok && (r0 + TILE <= rows) && (c0 + TILE <= cols);

  if (full) {
    const int q = l & 7, i = l >> 3;
    float4 v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {  // issue all four 16-byte loads first
      const int g = w * 4 + k, r = (g >> 1) * 4 + i, c = (g & 1) * 32 + q * 4;
      v[k] = __ldcs(reinterpret_cast<const float4*>(src + (r0 + r) * cols + c0 + c));
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int g = w * 4 + k, r = (g >> 1) * 4 + i, c = (g & 1) * 32 + q * 4;
      const int rs = r ^ (4 * q);  // swizzle of columns c..c+3 (all share (c/4)%8 == q)
      T[(c + 0) * TILE + rs] = __float_as_uint(v[k].x);
      T[(c + 1) * TILE + rs] = __float_as_uint(v[k].y);
      T[(c + 2) * TILE + rs] = __float_as_uint(v[k].z);
      T[(c + 3) * TILE + rs] = __float_as_uint(v[k].w);
    }
    __syncthreads();
    const int u = l & 7, ci = l >> 3;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int g = w * 4 + k, cg = g >> 1, c = cg * 4 + ci, uu = (g & 1) * 8 + u;
      const int phys = (4 * uu) ^ (4 * (cg & 7));
      const uint4 x = *reinterpret_cast<const uint4*>(&T[c * TILE + phys]);
      __stcs(reinterpret_cast<float4*>(dst + (c0 + c) * rows + r0 + 4 * uu),
             make_float4(__uint_as_float(x.x), __uint_as_float(x.y), __uint_as_float(x.z),
                         __uint_as_float(x.w)));
    }
  } else {
    // Edge or unaligned tile: element-wise with bounds checks, same swizzle.
    for (int e = t; e < TILE * TILE; e += THREADS) {
      const int r = e / TILE, c = e % TILE;
      if (r0 + r < rows && c0 + c < cols)
        T[c * TILE + (r ^ (4 * ((c >> 2) & 7)))] = __float_as_uint(src[(r0 + r) * cols + c0 + c]);
    }
    __syncthreads();
    for (int e = t; e < TILE * TILE; e += THREADS) {
      const int c = e / TILE, r = e % TILE;
      if (r0 + r < rows && c0 + c < cols)
        dst[(c0 + c) * rows + r0 + r] = __uint_as_float(T[c * TILE + (r ^ (4 * ((c >> 2) & 7)))]);
    }
  }
}

// ---------------------------------------------------------------------------
// bf16: a word holds the elements of two consecutive input rows for one
// column, so T is 64 (out rows c) x 32 (row pairs p) words = 8 KiB and an
// output 16-byte chunk is 4 consecutive words = 8 consecutive bf16.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(THREADS) transpose_bf16_kernel(const uint16_t* __restrict__ in,
                                                                 uint16_t* __restrict__ out,
                                                                 int64_t rows, int64_t cols,
                                                                 int vec_ok) {
  __shared__ __align__(16) uint32_t T[TILE * (TILE / 2)];
  __shared__ uint16_t E[TILE][TILE + 2];  // edge-tile staging
  const int64_t b = blockIdx.z;
  const uint16_t* src = in + b * rows * cols;
  uint16_t* dst = out + b * rows * cols;
  const int64_t r0 = (int64_t)blockIdx.y * TILE, c0 = (int64_t)blockIdx.x * TILE;
  const int t = threadIdx.x, w = t >> 5, l = t & 31;
  const bool full = vec_ok && (r0 + TILE <= rows) && (c0 + TILE <= cols);

  if (full) {
    const int q = l & 7, pi = l >> 3, p = w * 4 + pi;
    const uint4 x = __ldcs(reinterpret_cast<const uint4*>(src + (r0 + 2 * p) * cols + c0 + 8 * q));
    const uint4 y =
        __ldcs(reinterpret_cast<const uint4*>(src + (r0 + 2 * p + 1) * cols + c0 + 8 * q));
    const int ps = p ^ (4 * q);  // swizzle of columns 8q..8q+7
    const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      T[(8 * q + 2 * m) * 32 + ps] = __byte_perm(xs[m], ys[m], 0x5410);      // low halves
      T[(8 * q + 2 * m + 1) * 32 + ps] = __byte_perm(xs[m], ys[m], 0x7632);  // high halves
    }
    __syncthreads();
    const int u = l & 7, ci = l >> 3;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int c = (w * 2 + k) * 4 + ci;
      const int phys = (4 * u) ^ (4 * ((c >> 3) & 7));
      const uint4 o = *reinterpret_cast<const uint4*>(&T[c * 32 + phys]);
      __stcs(reinterpret_cast<uint4*>(dst + (c0 + c) * rows + r0 + 8 * u), o);
    }
  } else {
    for (int e = t; e < TILE * TILE; e += THREADS) {
      const int r = e / TILE, c = e % TILE;
      if (r0 + r < rows && c0 + c < cols) E[c][r] = src[(r0 + r) * cols + c0 + c];
    }
    __syncthreads();
    for (int e = t; e < TILE * TILE; e += THREADS) {
      const int c = e / TILE, r = e % TILE;
      if (r0 + r < rows && c0 + c < cols) dst[(c0 + c) * rows + r0 + r] = E[c][r];
    }
  }
}

int check_dims(int64_t batch, int64_t rows, int64_t cols) {
  MB_REQUIRE(batch >= 0 && rows >= 0 && cols >= 0, "transpose: negative dimension");
  MB_REQUIRE(batch <= 65535, "transpose: batch %lld exceeds 65535", (long long)batch);
  MB_REQUIRE((rows + TILE - 1) / TILE <= 65535, "transpose: rows %lld too large", (long long)rows);
  return MB_OK;
}

template <typename T>
int launch(void (*kern)(const T*, T*, int64_t, int64_t, int), const T* in, T* out, int64_t batch,
           int64_t rows, int64_t cols, int vec_elems, void* stream) {
  int rc = check_dims(batch, rows, cols);
  if (rc) return rc;
  if (batch == 0 || rows == 0 || cols == 0) return MB_OK;
  MB_REQUIRE(in != nullptr && out != nullptr, "transpose: null pointer");
  MB_REQUIRE(reinterpret_cast<uintptr_t>(in) != reinterpret_cast<uintptr_t>(out),
             "transpose: in-place transpose is not supported");
  const int vec_ok = (rows % vec_elems == 0) && (cols % vec_elems == 0) &&
                     (reinterpret_cast<uintptr_t>(in) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(out) % 16 == 0);
  dim3 grid((unsigned)((cols + TILE - 1) / TILE), (unsigned)((rows + TILE - 1) / TILE),
            (unsigned)batch);
  kern<<<grid, THREADS, 0, static_cast<cudaStream_t>(stream)>>>(in, out, rows, cols, vec_ok);
  MB_CUDA(cudaGetLastError());
  return MB_OK;
}

}  // namespace

extern "C" int mb_transpose_2d_f32(const float* in, float* out, int64_t rows, int64_t cols,
                                   void* stream) {
  return launch<float>(transpose_f32_kernel, in, out, 1, rows, cols, 4, stream);
}

extern "C" int mb_transpose_batched_f32(const float* in, float* out, int64_t batch, int64_t rows,
                                        int64_t cols, void* stream) {
  return launch<float>(transpose_f32_kernel, in, out, batch, rows, cols, 4, stream);
}

extern "C" int mb_transpose_batched_bf16(const uint16_t* in, uint16_t* out, int64_t batch,
                                         int64_t rows, int64_t cols, void* stream) {
  return launch<uint16_t>(transpose_bf16_kernel, in, out, batch, rows, cols, 8, stream);
}
