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
//  * decode: one new token per sequence. Memory-bound split-KV kernel on CUDA
//    cores: a CTA owns (sequence, kv head, key split) and ALL G query heads of
//    that kv head, so every K/V byte is read once; partial (max, sum, o)
//    triples are merged by a small combine kernel.
//  * prefill: FlashAttention-2 style tiles on the warp-level bf16 tensor-core
//    MMA (mma.sync m16n8k16), 64 queries x 64 keys per step, online softmax in
//    fp32, causal skip of key tiles above the diagonal.
#include "common.cuh"

namespace {

constexpr int PAGE = 64;
constexpr int DH = 128;

__device__ __forceinline__ float bf2f(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }
__device__ __forceinline__ float lo_bf(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_bf(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// ---------------------------------------------------------------------------
// decode
// ---------------------------------------------------------------------------
// grid (splits, Hkv, B), 128 threads (4 warps). Each warp walks 32 keys at a
// time: lane = key for q.k (the key's 256-byte row read by its lane, q for the
// G heads broadcast from shared memory), then lane = 4 dims for p.v.
template <int G>
__global__ void __launch_bounds__(128) attn_decode_kernel(
    const uint16_t* __restrict__ q, int ldq, const uint16_t* __restrict__ kc,
    const uint16_t* __restrict__ vc, const int* __restrict__ block_table, int max_pages,
    const int* __restrict__ kv_len, int Hkv, int keys_per_split, float scale_log2,
    float* __restrict__ part_o, float* __restrict__ part_ml) {
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int splits = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ __align__(16) float qs[G][DH];
  __shared__ float wm[4][G], wl[4][G];
  __shared__ __align__(16) float wo[4][G][DH];

  for (int i = threadIdx.x; i < G * DH; i += 128) {
    const int g = i / DH, d = i % DH;
    qs[g][d] = bf2f(q[(int64_t)b * ldq + (kvh * G + g) * DH + d]);
  }
  __syncthreads();

  const int L = kv_len[b];
  const int k_begin = split * keys_per_split;
  const int k_end = min(L, k_begin + keys_per_split);
  float m[G], l[G], o[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) o[g][j] = 0.f;
  }
  for (int k0 = k_begin + warp * 32; k0 < k_end; k0 += 128) {
    const int key = k0 + lane;
    const bool valid = key < k_end;
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = 0.f;
    const int kk = valid ? key : k0;
    const int pg = block_table[b * max_pages + kk / PAGE];
    const int64_t row = (((int64_t)pg * Hkv + kvh) * PAGE + kk % PAGE) * DH;
    const uint4* kr = reinterpret_cast<const uint4*>(kc + row);
#pragma unroll 4
    for (int c = 0; c < DH / 8; ++c) {
      const uint4 w = kr[c];
      const float kf[8] = {lo_bf(w.x), hi_bf(w.x), lo_bf(w.y), hi_bf(w.y),
                           lo_bf(w.z), hi_bf(w.z), lo_bf(w.w), hi_bf(w.w)};
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float4 qa = *reinterpret_cast<const float4*>(&qs[g][c * 8]);
        const float4 qb = *reinterpret_cast<const float4*>(&qs[g][c * 8 + 4]);
        s[g] += qa.x * kf[0] + qa.y * kf[1] + qa.z * kf[2] + qa.w * kf[3] + qb.x * kf[4] +
                qb.y * kf[5] + qb.z * kf[6] + qb.w * kf[7];
      }
    }
    // online softmax over this group of 32 keys (log2 domain)
    float p[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float sv = valid ? s[g] * scale_log2 : -INFINITY;
      float mx = sv;
#pragma unroll
      for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mn = fmaxf(m[g], mx);
      const float corr = exp2f(m[g] - mn);  // m = -inf initially -> 0
      p[g] = valid ? exp2f(sv - mn) : 0.f;
      float ps = p[g];
#pragma unroll
      for (int off = 16; off; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l[g] = l[g] * corr + ps;
      m[g] = mn;
#pragma unroll
      for (int j = 0; j < 4; ++j) o[g][j] *= corr;
    }
    // p . v: lane owns dims 4*lane..4*lane+3, loops over the 32 keys
    const int nk = min(32, k_end - k0);
    for (int t = 0; t < nk; ++t) {
      const int key2 = k0 + t;
      const int pg2 = block_table[b * max_pages + key2 / PAGE];
      const int64_t row2 = (((int64_t)pg2 * Hkv + kvh) * PAGE + key2 % PAGE) * DH;
      const uint2 w = *reinterpret_cast<const uint2*>(vc + row2 + 4 * lane);
      const float v0 = lo_bf(w.x), v1 = hi_bf(w.x), v2 = lo_bf(w.y), v3 = hi_bf(w.y);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pt = __shfl_sync(0xffffffffu, p[g], t);
        o[g][0] += pt * v0;
        o[g][1] += pt * v1;
        o[g][2] += pt * v2;
        o[g][3] += pt * v3;
      }
    }
  }
  // merge the 4 warps of the CTA
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      wm[warp][g] = m[g];
      wl[warp][g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
    *reinterpret_cast<float4*>(&wo[warp][g][4 * lane]) =
        make_float4(o[g][0], o[g][1], o[g][2], o[g][3]);
  __syncthreads();
  const int64_t unit = ((int64_t)b * Hkv + kvh) * splits + split;
  for (int i = threadIdx.x; i < G * DH; i += 128) {
    const int g = i / DH, d = i % DH;
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w][g]);
    float Ls = 0.f, acc = 0.f;
    for (int w = 0; w < 4; ++w) {
      const float c = wm[w][g] == -INFINITY ? 0.f : exp2f(wm[w][g] - M);
      Ls += wl[w][g] * c;
      acc += wo[w][g][d] * c;
    }
    part_o[(unit * G + g) * DH + d] = acc;
    if (d == 0) {
      part_ml[(unit * G + g) * 2] = M;
      part_ml[(unit * G + g) * 2 + 1] = Ls;
    }
  }
}

// out[b, (kvh*G+g)*DH + d] = sum_split o * 2^(m - M) / sum_split l * 2^(m - M)
__global__ void attn_combine_kernel(const float* __restrict__ part_o,
                                    const float* __restrict__ part_ml, int splits, int G, int Hkv,
                                    uint16_t* __restrict__ out, int ldo) {
  const int g = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z, d = threadIdx.x;
  const int64_t base = ((int64_t)b * Hkv + kvh) * splits;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, part_ml[((base + s) * G + g) * 2]);
  float Ls = 0.f, acc = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float m = part_ml[((base + s) * G + g) * 2];
    if (m == -INFINITY) continue;
    const float c = exp2f(m - M);
    Ls += part_ml[((base + s) * G + g) * 2 + 1] * c;
    acc += part_o[((base + s) * G + g) * DH + d] * c;
  }
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
      const uint16_t* kr = K + (nt * 8 + gid) * KV_LD + tig * 2;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(kr + ks * 16);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(kr + ks * 16 + 8);
        mma_bf16_16816(s[nt], qa[ks], b0, b1);
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
      const uint16_t* v0 = V + (k2 * 16 + tig * 2) * KV_LD + gid;
#pragma unroll
      for (int dt = 0; dt < 16; ++dt) {
        const uint16_t* vp = v0 + dt * 8;
        const uint32_t b0 = (uint32_t)vp[0] | ((uint32_t)vp[KV_LD] << 16);
        const uint32_t b1 = (uint32_t)vp[8 * KV_LD] | ((uint32_t)vp[9 * KV_LD] << 16);
        mma_bf16_16816(o[dt], pa, b0, b1);
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
int decode_splits(int B, int Hkv, int max_kv_len, int* keys_per_split) {
  // Aim for about 4 CTAs per SM; splits are whole multiples of 128 keys.
  const int units = B * Hkv;
  int want = (4 * mb::num_sms() + units - 1) / units;
  int kps = (max_kv_len + want - 1) / want;
  kps = ((kps + 127) / 128) * 128;
  if (kps < 128) kps = 128;
  *keys_per_split = kps;
  return (max_kv_len + kps - 1) / kps;
}
}  // namespace

extern "C" size_t mb_attention_decode_workspace_bytes(int B, int Hq, int Hkv, int max_kv_len) {
  if (B <= 0 || Hkv <= 0 || max_kv_len <= 0) return 0;
  int kps;
  const int splits = decode_splits(B, Hkv, max_kv_len, &kps);
  const size_t units = (size_t)B * Hq * splits;
  return units * DH * 4 + units * 2 * 4 + 256;
}

extern "C" int mb_attention_decode_bf16(const uint16_t* q, int ldq, const uint16_t* k_cache,
                                        const uint16_t* v_cache, const int* block_table,
                                        int max_pages, const int* kv_len, int max_kv_len, int B,
                                        int Hq, int Hkv, int Dh, uint16_t* out, int ldo,
                                        void* workspace, size_t workspace_bytes, void* stream) {
  MB_REQUIRE(Dh == DH, "attention: head_dim must be 128 (got %d)", Dh);
  MB_REQUIRE(Hkv > 0 && Hq % Hkv == 0, "attention: Hq must be a multiple of Hkv");
  const int G = Hq / Hkv;
  MB_REQUIRE(G == 1 || G == 2 || G == 4 || G == 8, "attention decode: G = Hq/Hkv must be 1, 2, 4 or 8");
  MB_REQUIRE(max_kv_len > 0 && max_kv_len <= max_pages * PAGE, "attention: bad max_kv_len");
  if (B == 0) return MB_OK;
  const size_t need = mb_attention_decode_workspace_bytes(B, Hq, Hkv, max_kv_len);
  MB_REQUIRE(workspace && workspace_bytes >= need,
             "attention decode: workspace of %zu bytes required", need);
  int kps;
  const int splits = decode_splits(B, Hkv, max_kv_len, &kps);
  float* part_o = static_cast<float*>(workspace);
  float* part_ml = part_o + (size_t)B * Hq * splits * DH;
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)DH);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  dim3 grid(splits, Hkv, B);
#define MB_DEC(GG)                                                                               \
  attn_decode_kernel<GG><<<grid, 128, 0, s>>>(q, ldq, k_cache, v_cache, block_table, max_pages, \
                                              kv_len, Hkv, kps, scale_log2, part_o, part_ml)
  switch (G) {
    case 1: MB_DEC(1); break;
    case 2: MB_DEC(2); break;
    case 4: MB_DEC(4); break;
    default: MB_DEC(8); break;
  }
#undef MB_DEC
  MB_CUDA(cudaGetLastError());
  attn_combine_kernel<<<dim3(G, Hkv, B), DH, 0, s>>>(part_o, part_ml, splits, G, Hkv, out, ldo);
  MB_CUDA(cudaGetLastError());
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
  const int smem = 4 * PAGE * KV_LD * 2;
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)DH);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  dim3 grid((S + 63) / 64, Hq, B);
  static bool attr = false;
  if (!attr) {
    MB_CUDA(cudaFuncSetAttribute(attn_prefill_kernel<true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    MB_CUDA(cudaFuncSetAttribute(attn_prefill_kernel<false>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr = true;
  }
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
