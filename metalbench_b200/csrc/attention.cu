// GQA attention over the paged KV cache.
//
// Reference: mlx/kernels/full/llama_decoder_layer.py:30-37 — q, k, v split
// from qkv, RoPE on q and k, k/v repeated G = H/H_kv times along the head axis
// (query head h reads kv head h // G), softmax(q k^T / sqrt(Dh)) @ v, heads
// re-interleaved to (S, D). The reference hook is non-causal over S keys; the
// decoder configs here add a causal mask and a KV cache (keys at positions
// 0..kv_len-1 of each sequence).
//
// Cache layout (both kernels): k, v = [num_pages][Hkv][PAGE=64][Dh=128] bf16,
// sequence b's position p in page block_table[b*max_pages + p/64], slot p%64.
//
//  * decode: one new token per sequence. Memory-bound split-KV kernel: a CTA
//    owns (sequence, kv head, key split) and ALL G query heads of that kv
//    head (the 16 rows of a warp MMA), so every K/V byte is read once; whole
//    16 KiB pages stream into shared memory through a cp.async ring; partial
//    (max, sum, o) triples are merged by a small combine kernel.
//  * prefill: tcgen05/TMEM kernel in attention_tc.cu when TMA can address the
//    operands (16-byte aligned rows); otherwise FlashAttention-2 style tiles
//    on the warp-level bf16 MMA (mma.sync m16n8k16) below, 64 queries x 64
//    keys per step, online softmax in fp32, causal skip of key tiles above
//    the diagonal.
#include "common.cuh"
#include "kernels.h"

namespace {

constexpr int PAGE = 64;
constexpr int DH = 128;

__device__ __forceinline__ float bf2f(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }
__device__ __forceinline__ float lo_bf(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_bf(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Decode partials: every (CTA, unit) segment of the flattened page range has
// pps (max, sum, o) triples per query head -- one per warp (pps = 4), or one
// merged over the warps (pps = 1) -- at
//   part_ml[((unit*smax + j)*pps + w)*G + g][0..1], part_o[...][0..DH-1],
// j = CTA index - first CTA of the unit. The combine merges the segments of
// its unit: out = sum o * 2^(m - M) / sum l * 2^(m - M).
__global__ void __launch_bounds__(128) attn_combine_kernel(
    const float* __restrict__ part_o, const float* __restrict__ part_ml, int pages, int per,
    int smax, int pps, int G, int Hkv, uint16_t* __restrict__ out, int ldo) {
  mbd::pdl_trigger();
  mbd::pdl_wait();
  extern __shared__ float wsh[];  // one weight per partial
  __shared__ float red[4];
  const int g = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z, d = threadIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t unit = (int64_t)b * Hkv + kvh;
  const int64_t c0 = unit * pages / per, c1 = (unit * pages + pages - 1) / per;
  const int nparts = (int)(c1 - c0 + 1) * pps;
  const int64_t base = unit * smax * pps;
  // all partials' (max, sum) at once, one per thread, then block reductions
  float M = -INFINITY;
  for (int i = threadIdx.x; i < nparts; i += 128) M = fmaxf(M, part_ml[((base + i) * G + g) * 2]);
#pragma unroll
  for (int off = 16; off; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  if (lane == 0) red[warp] = M;
  __syncthreads();
  M = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  __syncthreads();
  float Ls = 0.f;
  for (int i = threadIdx.x; i < nparts; i += 128) {
    const float2 ml = *reinterpret_cast<const float2*>(part_ml + ((base + i) * G + g) * 2);
    const float w = ml.x == -INFINITY ? 0.f : exp2f(ml.x - M);
    wsh[i] = w;
    Ls += ml.y * w;
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) Ls += __shfl_xor_sync(0xffffffffu, Ls, off);
  if (lane == 0) red[warp] = Ls;
  __syncthreads();
  Ls = red[0] + red[1] + red[2] + red[3];
  // o: thread d sums its column over the partials, loads four at a time
  float acc = 0.f;
  int i = 0;
  for (; i + 4 <= nparts; i += 4) {
    float t[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) t[j] = part_o[((base + i + j) * G + g) * DH + d];
#pragma unroll
    for (int j = 0; j < 4; ++j) acc += t[j] * wsh[i + j];
  }
  for (; i < nparts; ++i) acc += part_o[((base + i) * G + g) * DH + d] * wsh[i];
  const float r = Ls > 0.f ? acc / Ls : 0.f;
  __nv_bfloat16 h = __float2bfloat16_rn(r);
  out[(int64_t)b * ldo + (kvh * G + g) * DH + d] = *reinterpret_cast<uint16_t*>(&h);
}

}  // namespace

namespace {

// ---------------------------------------------------------------------------
// prefill
// ---------------------------------------------------------------------------
constexpr int KV_LD = DH + 8;  // padded shared row (272 B): conflict-free fragment loads

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(mbd::smem_u32(smem)),
               "l"(gmem), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Four 8x8 b16 matrices from shared memory; lane l gives the address of row
// l%8 of matrix l/8. Padded 272-byte rows put the 8 rows on distinct banks.
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(mbd::smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(mbd::smem_u32(p)));
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// grid (ceil(S/64), Hq, B), 128 threads: warp w owns query rows 16w..16w+15
// of the tile. Keys 0..kv_len[b]-1 of sequence b are read from the paged
// cache one 64-key page at a time (double-buffered with cp.async; rows past
// kv_len are zero-filled so masked keys contribute exactly 0).
template <bool CAUSAL>
__global__ void __launch_bounds__(128) attn_prefill_kernel(
    const uint16_t* __restrict__ q, int ldq, const uint16_t* __restrict__ kc,
    const uint16_t* __restrict__ vc, const int* __restrict__ block_table, int max_pages,
    const int* __restrict__ start_pos, const int* __restrict__ kv_len, int S, int Hkv, int G,
    float scale_log2, uint16_t* __restrict__ out, int ldo) {
  extern __shared__ __align__(16) uint16_t sm[];
  uint16_t* Ks = sm;                       // [2][64][KV_LD]
  uint16_t* Vs = sm + 2 * PAGE * KV_LD;    // [2][64][KV_LD]
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int p0 = start_pos[b];
  const int L = kv_len[b];
  const int r0 = qt * 64 + warp * 16;  // first query row of this warp (within the sequence)

  // Q fragments for all 8 k-steps of Dh = 128.
  uint32_t qa[8][4];
  {
    const int ra = r0 + gid, rb = r0 + gid + 8;
    const uint16_t* qra = q + ((int64_t)b * S + ra) * ldq + h * DH;
    const uint16_t* qrb = q + ((int64_t)b * S + rb) * ldq + h * DH;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int c = ks * 16 + tig * 2;
      qa[ks][0] = ra < S ? *reinterpret_cast<const uint32_t*>(qra + c) : 0u;
      qa[ks][1] = rb < S ? *reinterpret_cast<const uint32_t*>(qrb + c) : 0u;
      qa[ks][2] = ra < S ? *reinterpret_cast<const uint32_t*>(qra + c + 8) : 0u;
      qa[ks][3] = rb < S ? *reinterpret_cast<const uint32_t*>(qrb + c + 8) : 0u;
    }
  }
  const int qpos_a = p0 + r0 + gid, qpos_b = qpos_a + 8;
  // key tiles to visit
  int n_tiles = (L + PAGE - 1) / PAGE;
  if (CAUSAL) {
    const int last_q = p0 + min(S - 1, qt * 64 + 63);
    n_tiles = min(n_tiles, last_q / PAGE + 1);
  }

  auto load_tile = [&](int kt, int buf) {
    const int pg = block_table[b * max_pages + kt];
    const int64_t base = ((int64_t)pg * Hkv + kvh) * PAGE * DH;
    for (int c = threadIdx.x; c < PAGE * DH / 8; c += 128) {
      const int row = c >> 4, col = (c & 15) * 8;
      const bool ok = kt * PAGE + row < L;
      cp_async16(Ks + (buf * PAGE + row) * KV_LD + col, kc + base + row * DH + col, ok);
      cp_async16(Vs + (buf * PAGE + row) * KV_LD + col, vc + base + row * DH + col, ok);
    }
    cp_async_commit();
  };

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;

  if (n_tiles > 0) load_tile(0, 0);
  for (int kt = 0; kt < n_tiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < n_tiles) {
      load_tile(kt + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint16_t* K = Ks + buf * PAGE * KV_LD;
    const uint16_t* V = Vs + buf * PAGE * KV_LD;

    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
      // matrices (keys nt*8.., dims ks*16 + {0,8,16,24}): b0, b1 of k-steps ks, ks+1
      const uint16_t* kr = K + (nt * 8 + (lane & 7)) * KV_LD + (lane >> 3) * 8;
#pragma unroll
      for (int ks = 0; ks < 8; ks += 2) {
        uint32_t b[4];
        ldsm_x4(b, kr + ks * 16);
        mma_bf16_16816(s[nt], qa[ks], b[0], b[1]);
        mma_bf16_16816(s[nt], qa[ks + 1], b[2], b[3]);
      }
    }
    // mask + scale, row max
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = kt * PAGE + nt * 8 + tig * 2 + e;
        const bool ok_a = j < L && (!CAUSAL || j <= qpos_a);
        const bool ok_b = j < L && (!CAUSAL || j <= qpos_b);
        s[nt][e] = ok_a ? s[nt][e] * scale_log2 : -INFINITY;
        s[nt][2 + e] = ok_b ? s[nt][2 + e] * scale_log2 : -INFINITY;
        mx_a = fmaxf(mx_a, s[nt][e]);
        mx_b = fmaxf(mx_b, s[nt][2 + e]);
      }
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, off));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, off));
    }
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
    const float sa = mn_a == -INFINITY ? 0.f : mn_a;  // fully masked row so far
    const float sb = mn_b == -INFINITY ? 0.f : mn_b;
    const float corr_a = exp2f(m_a - sa), corr_b = exp2f(m_b - sb);
    m_a = mn_a;
    m_b = mn_b;
    float sum_a = 0.f, sum_b = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = exp2f(s[nt][0] - sa);
      s[nt][1] = exp2f(s[nt][1] - sa);
      s[nt][2] = exp2f(s[nt][2] - sb);
      s[nt][3] = exp2f(s[nt][3] - sb);
      sum_a += s[nt][0] + s[nt][1];
      sum_b += s[nt][2] + s[nt][3];
    }
    l_a = l_a * corr_a + sum_a;
    l_b = l_b * corr_b + sum_b;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      o[dt][0] *= corr_a;
      o[dt][1] *= corr_a;
      o[dt][2] *= corr_b;
      o[dt][3] *= corr_b;
    }
    // o += p @ v
#pragma unroll
    for (int k2 = 0; k2 < 4; ++k2) {
      uint32_t pa[4];
      pa[0] = pack2(s[2 * k2][0], s[2 * k2][1]);
      pa[1] = pack2(s[2 * k2][2], s[2 * k2][3]);
      pa[2] = pack2(s[2 * k2 + 1][0], s[2 * k2 + 1][1]);
      pa[3] = pack2(s[2 * k2 + 1][2], s[2 * k2 + 1][3]);
      // transposed matrices (keys k2*16 + {0,8}, dims dt*8 + {0,8}): b0, b1 of dt, dt+1
      const uint16_t* vr =
          V + (k2 * 16 + ((lane >> 3) & 1) * 8 + (lane & 7)) * KV_LD + (lane >> 4) * 8;
#pragma unroll
      for (int dt = 0; dt < 16; dt += 2) {
        uint32_t b[4];
        ldsm_x4_t(b, vr + dt * 8);
        mma_bf16_16816(o[dt], pa, b[0], b[1]);
        mma_bf16_16816(o[dt + 1], pa, b[2], b[3]);
      }
    }
    __syncthreads();  // the buffer is refilled two iterations later
  }
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    l_a += __shfl_xor_sync(0xffffffffu, l_a, off);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, off);
  }
  const float ia = l_a > 0.f ? 1.f / l_a : 0.f, ib = l_b > 0.f ? 1.f / l_b : 0.f;
  const int ra = r0 + gid, rb = ra + 8;
#pragma unroll
  for (int dt = 0; dt < 16; ++dt) {
    const int c = h * DH + dt * 8 + tig * 2;
    if (ra < S)
      *reinterpret_cast<uint32_t*>(out + ((int64_t)b * S + ra) * ldo + c) =
          pack2(o[dt][0] * ia, o[dt][1] * ia);
    if (rb < S)
      *reinterpret_cast<uint32_t*>(out + ((int64_t)b * S + rb) * ldo + c) =
          pack2(o[dt][2] * ib, o[dt][3] * ib);
  }
}

}  // namespace

namespace {

// ---------------------------------------------------------------------------
// decode on the warp MMA: the G query heads of one kv head are the 16 MMA rows
// (rows >= G are zero). The work is the flat list of (unit, page) pairs,
// unit = (sequence, kv head), each unit `pages` long (pages past a sequence's
// kv_len are skipped); CTA c streams pairs c*per .. (c+1)*per-1. With few
// units (tensor parallel) the ranges cross unit boundaries, so every SM gets
// the same number of pages in one resident wave; with many, they are
// unit-aligned splits (decode_plan).
// Pages are staged whole (K and V, 16 KiB each) into a three-deep cp.async
// ring; warp w takes keys 16w..16w+15 of every page with its own
// online-softmax state, which it writes out as a partial whenever the unit
// changes (and at the end); attn_combine_kernel merges the partials.
// ---------------------------------------------------------------------------
constexpr int DEC_STAGES = 3;

__global__ void __launch_bounds__(128) attn_decode_mma_kernel(
    const uint16_t* __restrict__ q, int ldq, const uint16_t* __restrict__ kc,
    const uint16_t* __restrict__ vc, const int* __restrict__ block_table, int max_pages,
    const int* __restrict__ kv_len, int Hkv, int G, int pages, int per, int64_t total, int smax,
    int merged, float scale_log2, float* __restrict__ part_o, float* __restrict__ part_ml) {
  mbd::pdl_trigger();
  mbd::pdl_wait();
  extern __shared__ __align__(16) uint16_t sm[];
  uint16_t* Ks = sm;                                // [STAGES][64][KV_LD]
  uint16_t* Vs = sm + DEC_STAGES * PAGE * KV_LD;    // [STAGES][64][KV_LD]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int64_t begin = (int64_t)blockIdx.x * per;
  const int64_t endp = begin + per < total ? begin + per : total;
  const int n = (int)(endp - begin);

  // Pages are loaded and consumed in order: both sides step a (unit, page)
  // cursor instead of dividing the flat index.
  const int64_t units = total / pages;
  int ld_u = (int)(begin / pages), ld_kt = (int)(begin - (int64_t)ld_u * pages);
  int ld_b = ld_u / Hkv, ld_L = kv_len[ld_b];
  auto load_next = [&](int buf) {
    if (ld_kt * PAGE < ld_L) {  // else nothing of this page is attended
      const int kvh = ld_u - ld_b * Hkv;
      const int pg = block_table[ld_b * max_pages + ld_kt];
      const int64_t base = ((int64_t)pg * Hkv + kvh) * PAGE * DH;
      for (int c = threadIdx.x; c < PAGE * DH / 8; c += 128) {
        const int row = c >> 4, col = (c & 15) * 8;
        const bool ok = ld_kt * PAGE + row < ld_L;
        cp_async16(Ks + (buf * PAGE + row) * KV_LD + col, kc + base + row * DH + col, ok);
        cp_async16(Vs + (buf * PAGE + row) * KV_LD + col, vc + base + row * DH + col, ok);
      }
    }
    if (++ld_kt == pages) {
      ld_kt = 0;
      if (++ld_u < units) {
        ld_b = ld_u / Hkv;
        ld_L = kv_len[ld_b];
      }
    }
  };
  // prologue: STAGES-1 pages in flight (empty groups keep the counting uniform)
#pragma unroll
  for (int i = 0; i < DEC_STAGES - 1; ++i) {
    if (i < n) load_next(i);
    cp_async_commit();
  }
  uint32_t qa[8][4];
  float o[16][4];
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  int cur = -1, cur_b = 0, cur_L = 0;
  int unit = (int)(begin / pages), kt = (int)(begin - (int64_t)unit * pages);  // consumer cursor

  // this warp's (max, sum, o) of unit `cur` -> its partial slot; state reset
  auto flush = [&]() {
    float la = l_a, lb = l_b;
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      la += __shfl_xor_sync(0xffffffffu, la, off);
      lb += __shfl_xor_sync(0xffffffffu, lb, off);
    }
    const int64_t c0 = (int64_t)cur * pages / per;
    const int64_t slot = (((int64_t)cur * smax + (blockIdx.x - c0)) * 4 + warp) * G;
    if (gid < G) {
      float* po = part_o + (slot + gid) * DH;
#pragma unroll
      for (int dt = 0; dt < 16; ++dt)
        *reinterpret_cast<float2*>(po + dt * 8 + tig * 2) = make_float2(o[dt][0], o[dt][1]);
      if (tig == 0) *reinterpret_cast<float2*>(part_ml + (slot + gid) * 2) = make_float2(m_a, la);
    }
    if (gid + 8 < G) {
      float* po = part_o + (slot + gid + 8) * DH;
#pragma unroll
      for (int dt = 0; dt < 16; ++dt)
        *reinterpret_cast<float2*>(po + dt * 8 + tig * 2) = make_float2(o[dt][2], o[dt][3]);
      if (tig == 0)
        *reinterpret_cast<float2*>(part_ml + (slot + gid + 8) * 2) = make_float2(m_b, lb);
    }
  };

  for (int i = 0; i < n; ++i, ++kt) {
    const int buf = i % DEC_STAGES;
    if (i + DEC_STAGES - 1 < n) load_next((i + DEC_STAGES - 1) % DEC_STAGES);
    cp_async_commit();
    if (kt == pages) {
      kt = 0;
      ++unit;
    }
    if (unit != cur) {  // a new (sequence, kv head): flush the old one, load q
      if (cur >= 0) flush();
      cur = unit;
      cur_b = unit / Hkv;
      cur_L = kv_len[cur_b];
      const int kvh = unit - cur_b * Hkv;
      const uint16_t* qr = q + (int64_t)cur_b * ldq + (kvh * G) * DH;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int c = ks * 16 + tig * 2;
        const bool ra = gid < G, rb = gid + 8 < G;
        qa[ks][0] = ra ? *reinterpret_cast<const uint32_t*>(qr + gid * DH + c) : 0u;
        qa[ks][1] = rb ? *reinterpret_cast<const uint32_t*>(qr + (gid + 8) * DH + c) : 0u;
        qa[ks][2] = ra ? *reinterpret_cast<const uint32_t*>(qr + gid * DH + c + 8) : 0u;
        qa[ks][3] = rb ? *reinterpret_cast<const uint32_t*>(qr + (gid + 8) * DH + c + 8) : 0u;
      }
#pragma unroll
      for (int t = 0; t < 16; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
      m_a = m_b = -INFINITY;
      l_a = l_b = 0.f;
    }
    cp_async_wait<DEC_STAGES - 1>();
    __syncthreads();
    const int key0 = kt * PAGE + warp * 16;
    if (key0 < cur_L) {  // warp-uniform: some of this warp's 16 keys are attended
      const uint16_t* K = Ks + (buf * PAGE + warp * 16) * KV_LD;
      const uint16_t* V = Vs + (buf * PAGE + warp * 16) * KV_LD;
      float s[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
        const uint16_t* kr = K + (nt * 8 + (lane & 7)) * KV_LD + (lane >> 3) * 8;
#pragma unroll
        for (int ks = 0; ks < 8; ks += 2) {
          uint32_t bb[4];
          ldsm_x4(bb, kr + ks * 16);
          mma_bf16_16816(s[nt], qa[ks], bb[0], bb[1]);
          mma_bf16_16816(s[nt], qa[ks + 1], bb[2], bb[3]);
        }
      }
      float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const bool ok = key0 + nt * 8 + tig * 2 + e < cur_L;
          s[nt][e] = ok ? s[nt][e] * scale_log2 : -INFINITY;
          s[nt][2 + e] = ok ? s[nt][2 + e] * scale_log2 : -INFINITY;
          mx_a = fmaxf(mx_a, s[nt][e]);
          mx_b = fmaxf(mx_b, s[nt][2 + e]);
        }
#pragma unroll
      for (int off = 1; off <= 2; off <<= 1) {
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, off));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, off));
      }
      const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
      const float sa = mn_a == -INFINITY ? 0.f : mn_a, sb = mn_b == -INFINITY ? 0.f : mn_b;
      const float ca = exp2f(m_a - sa), cb = exp2f(m_b - sb);
      m_a = mn_a;
      m_b = mn_b;
      float sum_a = 0.f, sum_b = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        s[nt][0] = exp2f(s[nt][0] - sa);
        s[nt][1] = exp2f(s[nt][1] - sa);
        s[nt][2] = exp2f(s[nt][2] - sb);
        s[nt][3] = exp2f(s[nt][3] - sb);
        sum_a += s[nt][0] + s[nt][1];
        sum_b += s[nt][2] + s[nt][3];
      }
      l_a = l_a * ca + sum_a;
      l_b = l_b * cb + sum_b;
      uint32_t pa[4];
      pa[0] = pack2(s[0][0], s[0][1]);
      pa[1] = pack2(s[0][2], s[0][3]);
      pa[2] = pack2(s[1][0], s[1][1]);
      pa[3] = pack2(s[1][2], s[1][3]);
      const uint16_t* vr = V + (((lane >> 3) & 1) * 8 + (lane & 7)) * KV_LD + (lane >> 4) * 8;
#pragma unroll
      for (int dt = 0; dt < 16; dt += 2) {
        o[dt][0] *= ca;
        o[dt][1] *= ca;
        o[dt][2] *= cb;
        o[dt][3] *= cb;
        o[dt + 1][0] *= ca;
        o[dt + 1][1] *= ca;
        o[dt + 1][2] *= cb;
        o[dt + 1][3] *= cb;
        uint32_t bb[4];
        ldsm_x4_t(bb, vr + dt * 8);
        mma_bf16_16816(o[dt], pa, bb[0], bb[1]);
        mma_bf16_16816(o[dt + 1], pa, bb[2], bb[3]);
      }
    }
    __syncthreads();  // this buffer is refilled STAGES-1 iterations later
  }
  cp_async_wait<0>();
  if (cur < 0) return;
  if (!merged) {
    flush();
    return;
  }
  // Unit-aligned range: the ring is free now, so the four warps' states are
  // merged in shared memory and one partial per (unit, split) is written.
  __syncthreads();
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    l_a += __shfl_xor_sync(0xffffffffu, l_a, off);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, off);
  }
  float* red = reinterpret_cast<float*>(sm);  // [4][16] m, [4][16] l, [4][16][DH] o
  float* rm = red;
  float* rl = red + 64;
  float* ro = red + 128;
  if (tig == 0) {
    rm[warp * 16 + gid] = m_a;
    rm[warp * 16 + gid + 8] = m_b;
    rl[warp * 16 + gid] = l_a;
    rl[warp * 16 + gid + 8] = l_b;
  }
#pragma unroll
  for (int dt = 0; dt < 16; ++dt) {
    const int d = dt * 8 + tig * 2;
    *reinterpret_cast<float2*>(ro + (warp * 16 + gid) * DH + d) = make_float2(o[dt][0], o[dt][1]);
    *reinterpret_cast<float2*>(ro + (warp * 16 + gid + 8) * DH + d) =
        make_float2(o[dt][2], o[dt][3]);
  }
  __syncthreads();
  const int64_t c0 = (int64_t)cur * pages / per;
  const int64_t slot = ((int64_t)cur * smax + (blockIdx.x - c0)) * G;
  for (int idx = threadIdx.x; idx < G * DH; idx += 128) {
    const int g = idx / DH, d = idx % DH;
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, rm[w * 16 + g]);
    float Ls = 0.f, acc = 0.f;
    for (int w = 0; w < 4; ++w) {
      const float mw = rm[w * 16 + g];
      const float c = mw == -INFINITY ? 0.f : exp2f(mw - M);
      Ls += rl[w * 16 + g] * c;
      acc += ro[(w * 16 + g) * DH + d] * c;
    }
    part_o[(slot + g) * DH + d] = acc;
    if (d == 0) *reinterpret_cast<float2*>(part_ml + (slot + g) * 2) = make_float2(M, Ls);
  }
}

}  // namespace

namespace {
constexpr int DEC_SMEM = 2 * DEC_STAGES * PAGE * KV_LD * 2;

// Decode plan: `pages` per unit (padded to a multiple of `per` when the CTA
// ranges are unit-aligned), `per` pages per CTA over the B*Hkv*pages pairs,
// `smax` = most CTAs one unit can span, grid = CTAs launched.
struct DecodePlan {
  int pages, per, smax, grid, merged;
  int64_t total;
};

int decode_resident_ctas() {
  static int per_sm[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!per_sm[dev]) {
    // the occupancy query sees the dynamic shared memory opt-in, so set it first
    int nb = 0;
    if (mb::ensure_smem_attr(reinterpret_cast<const void*>(attn_decode_mma_kernel), DEC_SMEM) ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, attn_decode_mma_kernel, 128,
                                                      DEC_SMEM) != cudaSuccess || nb < 1)
      nb = 1;
    per_sm[dev] = nb;
  }
  return per_sm[dev] * mb::num_sms();
}

DecodePlan decode_plan(int B, int Hkv, int max_kv_len) {
  DecodePlan p;
  const int pages = (max_kv_len + PAGE - 1) / PAGE;
  const int64_t units = (int64_t)B * Hkv;
  const int64_t slots = decode_resident_ctas();
  if (units >= slots) {
    // Enough (sequence, kv head) units to fill the GPU: unit-aligned splits of
    // at least 4 pages, ~12 CTAs per SM in all. Consecutive CTAs then read the
    // same page range of neighbouring kv heads, which lie next to each other
    // in the cache, and the many short waves hide each CTA's ramp.
    const int64_t want = (12 * (int64_t)mb::num_sms() + units - 1) / units;
    int pps = (int)((pages + want - 1) / want);
    if (pps < 4) pps = 4;
    const int splits = (pages + pps - 1) / pps;
    p.pages = splits * pps;  // padded: no CTA range crosses a unit
    p.per = pps;
    p.merged = 1;
  } else {
    // Few units (tensor parallel: B * Hkv/P): one resident wave, each CTA the
    // same share of the flat page list, crossing unit boundaries.
    p.pages = pages;
    int64_t per = (units * pages + slots - 1) / slots;
    if (per < 2) per = 2;
    p.per = (int)per;
    p.merged = 0;
  }
  p.total = units * p.pages;
  p.grid = (int)((p.total + p.per - 1) / p.per);
  p.smax = (p.pages + p.per - 1) / p.per + 1;
  return p;
}
}  // namespace

extern "C" size_t mb_attention_decode_workspace_bytes(int B, int Hq, int Hkv, int max_kv_len) {
  if (B <= 0 || Hkv <= 0 || Hq <= 0 || max_kv_len <= 0) return 0;
  const DecodePlan p = decode_plan(B, Hkv, max_kv_len);
  const size_t rows = (size_t)B * Hkv * p.smax * (p.merged ? 1 : 4) * (size_t)(Hq / Hkv);
  return rows * DH * 4 + rows * 2 * 4 + 256;
}

extern "C" int mb_attention_decode_bf16(const uint16_t* q, int ldq, const uint16_t* k_cache,
                                        const uint16_t* v_cache, const int* block_table,
                                        int max_pages, const int* kv_len, int max_kv_len, int B,
                                        int Hq, int Hkv, int Dh, uint16_t* out, int ldo,
                                        void* workspace, size_t workspace_bytes, void* stream) {
  MB_REQUIRE(Dh == DH, "attention: head_dim must be 128 (got %d)", Dh);
  MB_REQUIRE(Hkv > 0 && Hq % Hkv == 0, "attention: Hq must be a multiple of Hkv");
  const int G = Hq / Hkv;
  MB_REQUIRE(G <= 16, "attention decode: at most 16 query heads per kv head");
  MB_REQUIRE(max_kv_len > 0 && max_kv_len <= max_pages * PAGE, "attention: bad max_kv_len");
  if (B == 0) return MB_OK;
  MB_REQUIRE(B <= 65535 && Hkv <= 65535, "attention decode: grid too large");
  const size_t need = mb_attention_decode_workspace_bytes(B, Hq, Hkv, max_kv_len);
  MB_REQUIRE(workspace && workspace_bytes >= need,
             "attention decode: workspace of %zu bytes required", need);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = mb::ensure_smem_attr(reinterpret_cast<const void*>(attn_decode_mma_kernel), DEC_SMEM);
  if (rc) return rc;
  const DecodePlan p = decode_plan(B, Hkv, max_kv_len);
  float* part_o = static_cast<float*>(workspace);
  const int pps = p.merged ? 1 : 4;
  float* part_ml = part_o + (size_t)B * Hkv * p.smax * pps * G * DH;
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)DH);
  MB_CUDA(mb::launch_pdl(attn_decode_mma_kernel, dim3(p.grid), dim3(128), DEC_SMEM, s, q, ldq,
                          k_cache, v_cache, block_table, max_pages, kv_len, Hkv, G, p.pages, p.per,
                          p.total, p.smax, p.merged, scale_log2, part_o, part_ml));
  const size_t comb_smem = (size_t)p.smax * pps * sizeof(float);
  MB_REQUIRE(comb_smem <= 48 * 1024, "attention decode: too many partials per unit");
  MB_CUDA(mb::launch_pdl(attn_combine_kernel, dim3(G, Hkv, B), dim3(DH), comb_smem, s,
                          (const float*)part_o, (const float*)part_ml, p.pages, p.per, p.smax,
                          pps, G, Hkv, out, ldo));
  return MB_OK;
}

extern "C" int mb_attention_prefill_bf16(const uint16_t* q, int ldq, const uint16_t* k_cache,
                                         const uint16_t* v_cache, const int* block_table,
                                         int max_pages, const int* start_pos, const int* kv_len,
                                         int B, int S, int Hq, int Hkv, int Dh, int causal,
                                         uint16_t* out, int ldo, void* stream) {
  MB_REQUIRE(Dh == DH, "attention: head_dim must be 128 (got %d)", Dh);
  MB_REQUIRE(Hkv > 0 && Hq % Hkv == 0, "attention: Hq must be a multiple of Hkv");
  MB_REQUIRE(ldq % 2 == 0 && ldo % 2 == 0, "attention: leading dimensions must be even");
  if (B == 0 || S == 0) return MB_OK;
  MB_REQUIRE(Hq <= 65535 && B <= 65535, "attention: grid too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // tcgen05 kernel (attention_tc.cu) whenever TMA can address the operands
  if (mb::attention_prefill_tc_ok(q, ldq, k_cache, v_cache, out, ldo))
    return mb::attention_prefill_tc(q, ldq, k_cache, v_cache, block_table, max_pages, start_pos,
                                    kv_len, B, S, Hq, Hkv, causal, out, ldo, s);
  const int smem = 4 * PAGE * KV_LD * 2;
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)DH);
  dim3 grid((S + 63) / 64, Hq, B);
  int arc = mb::ensure_smem_attr(reinterpret_cast<const void*>(attn_prefill_kernel<true>), smem);
  if (!arc) arc = mb::ensure_smem_attr(reinterpret_cast<const void*>(attn_prefill_kernel<false>), smem);
  if (arc) return arc;
  if (causal)
    attn_prefill_kernel<true><<<grid, 128, smem, s>>>(q, ldq, k_cache, v_cache, block_table,
                                                       max_pages, start_pos, kv_len, S, Hkv,
                                                       Hq / Hkv, scale_log2, out, ldo);
  else
    attn_prefill_kernel<false><<<grid, 128, smem, s>>>(q, ldq, k_cache, v_cache, block_table,
                                                        max_pages, start_pos, kv_len, S, Hkv,
                                                        Hq / Hkv, scale_log2, out, ldo);
  MB_CUDA(cudaGetLastError());
  return MB_OK;
}

