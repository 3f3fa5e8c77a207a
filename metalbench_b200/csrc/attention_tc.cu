// Prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Same contract as the mma.sync prefill kernel in attention.cu (reference
// mlx/kernels/full/llama_decoder_layer.py:30-37 and
// mlx/kernels/standard/llama_attention.py:43-48: softmax(q k^T / sqrt(Dh)) v
// per query head, query head h reading kv head h / G, keys from the paged
// cache [pages][Hkv][64][128]), used when the operands allow TMA (16-byte
// aligned q/out rows).
//
// One CTA = 128 queries of one head (MMA M = 128), walking the keys in tiles
// of 128 (two cache pages):
//   warp 0     TMA producer: Q once; K and V of each key tile into separate
//              2-deep rings (each 64-key page is one {64 dims x 64 rows} box
//              per 64-dim half, 128-byte swizzle). A K slot is refilled as
//              soon as its S MMA has completed, a V slot once its P V has.
//              K is the K-major B operand of S = Q K^T; V, stored
//              [key][dim], is the MN-major B operand of O += P V.
//   warp 1     MMA issuer (one lane): S_j = Q K_j^T into TMEM buffer j % 2,
//              then O += P_{j-1} V_{j-1} (O in TMEM), so the tensor core
//              works on tile j while the softmax warps finish tile j-1.
//   warps 2-9  softmax, two threads per query row (TMEM lane), 64 keys each:
//              load the S half-row, mask (keys >= kv_len, and keys after the
//              query's position when causal), row maximum (the two halves
//              swap theirs through shared memory), p = 2^(s*scale - m), row
//              sums in fp32, P as bf16 into a 128-byte-swizzled shared tile
//              (the K-major A operand of P V). The running max is only
//              raised when a row's maximum grows by more than 8 (p stays
//              <= 256), and only then is that row of O rescaled in TMEM,
//              after the previous P V has completed. The MUFU exp2 rate
//              (16 per clock per SM) equals the tensor work of S and P V at
//              M = N = 128; two threads per row hide the per-thread latency.
// TMEM: S0 (128 cols) | S1 (128) | O (128) of a 512-column allocation.
// Every mbarrier wait is bounded (common.cuh) and reports through the device
// status word; the teardown drains the MMA pipe and in-flight copies.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace {

constexpr int TQ = 128;             // queries per CTA
constexpr int TK = 128;             // keys per tile
constexpr int DHT = 128;            // head dim
constexpr int PGK = 64;             // keys per cache page
constexpr int CHUNK = 128 * 128;    // one 64-element-wide, 128-row swizzled chunk (16 KiB)
constexpr int HALF_PAGE = 64 * 128; // one page's rows within a chunk (8 KiB)
constexpr int TILE = 2 * CHUNK;     // one 128 x 128 bf16 operand tile (32 KiB)
constexpr int OFF_K = TILE;                      // after Q: K[2]
constexpr int OFF_V = OFF_K + 2 * TILE;          // V[2]
constexpr int OFF_P = OFF_V + 2 * TILE;          // P[2]
constexpr int OFF_RED = OFF_P + 2 * TILE;        // row-max exchange [2 halves][128]
constexpr int OFF_BAR = OFF_RED + 2 * TQ * 4;
constexpr int NBAR = 19;
constexpr int SMEM_BYTES = 1024 + OFF_BAR + NBAR * 8 + 16;
constexpr int NSOFT = 256;     // softmax threads
constexpr float kRaise = 8.f;  // log2 headroom before the running max is raised

struct AttnTcParams {
  CUtensorMap qmap, kmap, vmap;
  const int* block_table;
  int max_pages;
  const int* start_pos;
  const int* kv_len;
  int S, Hkv, G, causal, n_qt;
  float scale_log2;
  uint16_t* out;
  int ldo;
  // split-KV (non-causal only): CTA split sp handles key tiles
  // [sp*tiles_per_split, +tiles_per_split) and writes its unnormalised O,
  // running max and row sum per row to part_o / part_ml instead of out
  int splits, tiles_per_split, Hq;
  float* part_o;   // [B][Hq][S][splits][128]
  float* part_ml;  // [B][Hq][S][splits][2]
};

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 2^x on the SFU (MUFU.EX2, flush-to-zero; 2^-inf = 0)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// K-major, 128B-swizzled operand of 128 rows x 128 elements stored as two
// 64-element chunks CHUNK bytes apart; k-step kk covers elements 16kk..16kk+15.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk) {
  return mbd::sw128_desc(base + (kk >> 2) * CHUNK + (kk & 3) * 32, 16, 1024);
}

__device__ __forceinline__ void pair_sync(int quad) {  // the two warps of a TMEM quadrant
  asm volatile("bar.sync %0, 64;" ::"r"(1 + quad) : "memory");
}

__global__ void __launch_bounds__(64 + NSOFT, 1)
    attn_prefill_tc_kernel(const __grid_constant__ AttnTcParams p, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* kfull = bars + 1;   // [2]
  uint64_t* kempty = bars + 3;  // [2]
  uint64_t* vfull = bars + 5;   // [2]
  uint64_t* vempty = bars + 7;  // [2]
  uint64_t* sfull = bars + 9;   // [2]
  uint64_t* sfree = bars + 11;  // [2]
  uint64_t* pfull = bars + 13;  // [2]
  uint64_t* pfree = bars + 15;  // [2]
  uint64_t* vfix = bars + 17;
  uint64_t* ofinal = bars + 18;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(base + OFF_RED);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = p.n_qt - 1 - (int)blockIdx.x / p.splits;  // longest causal tiles first
  const int sp = (int)blockIdx.x % p.splits;
  const int h = blockIdx.y, b = blockIdx.z, kvh = h / p.G;
  const int p0 = p.start_pos[b], L = p.kv_len[b];
  const int q_first = qt * TQ;
  int kend = L;
  if (p.causal) kend = min(L, p0 + min(p.S - 1, q_first + TQ - 1) + 1);
  const int tiles_all = kend > 0 ? (kend + TK - 1) / TK : 0;
  const int jbase = sp * p.tiles_per_split;  // first key tile of this CTA
  const int n_tiles = max(0, min(tiles_all, jbase + p.tiles_per_split) - jbase);
  const int valid_pages = (L + PGK - 1) / PGK;

  if (threadIdx.x == 0) {
    mbd::mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbd::mbar_init(&kfull[i], 1);
      mbd::mbar_init(&kempty[i], 1);
      mbd::mbar_init(&vfull[i], 1);
      mbd::mbar_init(&vempty[i], 1);
      mbd::mbar_init(&sfull[i], 1);
      mbd::mbar_init(&sfree[i], NSOFT);
      mbd::mbar_init(&pfull[i], NSOFT);
      mbd::mbar_init(&pfree[i], 1);
    }
    mbd::mbar_init(vfix, 1);
    mbd::mbar_init(ofinal, 1);
    *abort_flag = 0;
    mbd::fence_mbar_init();
  }
  if (warp == 1) mbd::tmem_alloc(tmem_slot, 512);
  __syncthreads();
  mbd::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS0 = tmem, tO = tmem + 256;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    // per ring: bit st = slot st received a load, bit 2+st = that load's parity
    uint32_t used_k = 0, used_v = 0;
    if (lane == 0) {
      mbd::prefetch_tmap(&p.qmap);
      mbd::prefetch_tmap(&p.kmap);
      mbd::prefetch_tmap(&p.vmap);
      mbd::mbar_expect_tx(q_full, TILE);
      for (int c = 0; c < 2; ++c)
        mbd::tma_load_2d(base + c * CHUNK, &p.qmap, q_full, h * DHT + c * 64, b * p.S + q_first);
    }
    __syncwarp();
    // one key tile (up to two pages) of the K or V cache into slot `dst`
    auto load_tile = [&](int j, const CUtensorMap* map, uint8_t* dst, uint64_t* bar) {
      const int pg0 = 2 * (jbase + j);
      const int npg = min(2, valid_pages - pg0);
      mbd::mbar_expect_tx(bar, (uint32_t)npg * 2 * HALF_PAGE);
      for (int pi = 0; pi < npg; ++pi) {
        const int phys = p.block_table[(int64_t)b * p.max_pages + pg0 + pi];
        const int row = (phys * p.Hkv + kvh) * PGK;
        for (int c = 0; c < 2; ++c)
          mbd::tma_load_2d(dst + c * CHUNK + pi * HALF_PAGE, map, bar, c * 64, row);
      }
    };
    // K runs one tile ahead of V: K_{j+1} is requested before V_j, since a K
    // slot frees up (S done) about a tile before a V slot (P V done) and a
    // load takes about a tile to land.
    bool ok = true;
    if (n_tiles > 0) {
      if (lane == 0) load_tile(0, &p.kmap, base + OFF_K, &kfull[0]);
      __syncwarp();
      used_k = 1u;
    }
    for (int j = 0; j < n_tiles && ok; ++j) {
      const int st = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      if (j + 1 < n_tiles) {
        const int kst = (j + 1) & 1;
        ok = __all_sync(0xffffffffu, mbd::mbar_wait(&kempty[kst], (((j + 1) >> 1) & 1) ^ 1,
                                                    status, MB_DEV_TIMEOUT_TMA, abort_flag));
        if (!ok) break;
        if (lane == 0) load_tile(j + 1, &p.kmap, base + OFF_K + kst * TILE, &kfull[kst]);
        __syncwarp();
        used_k = (used_k & ~(5u << kst)) | (1u << kst) | ((((j + 1) >> 1) & 1) << (2 + kst));
      }
      ok = __all_sync(0xffffffffu, mbd::mbar_wait(&vempty[st], ph ^ 1, status,
                                                  MB_DEV_TIMEOUT_TMA, abort_flag));
      if (!ok) break;
      if (lane == 0) load_tile(j, &p.vmap, base + OFF_V + st * TILE, &vfull[st]);
      __syncwarp();
      used_v = (used_v & ~(5u << st)) | (1u << st) | (ph << (2 + st));
    }
    // V rows past kv_len in the last tile (unloaded pages, or the rest of a
    // partial page) must be finite: P is 0 there, but 0 * NaN is not.
    if (ok && n_tiles > 0) {
      const int j = n_tiles - 1, st = j & 1;
      const int rows_valid = min(TK, L - TK * (jbase + j));
      if (rows_valid < TK) {
        ok = __all_sync(0xffffffffu, mbd::mbar_wait(&vfull[st], (j >> 1) & 1, status,
                                                    MB_DEV_TIMEOUT_TMA, abort_flag));
        if (ok) {
          uint8_t* sv = base + OFF_V + st * TILE;
          const int per_chunk = (TK - rows_valid) * 8;  // 16-byte units
          for (int i = lane; i < 2 * per_chunk; i += 32) {
            const int c = i / per_chunk, rem = i % per_chunk;
            const int r = rows_valid + rem / 8, u = rem % 8;
            *reinterpret_cast<uint4*>(sv + c * CHUNK + r * 128 + u * 16) = make_uint4(0, 0, 0, 0);
          }
          mbd::fence_proxy_async();
        }
        __syncwarp();
      }
      if (ok && lane == 0) mbd::mbar_arrive(vfix);
    }
    // no copy may still be landing in shared memory when the CTA exits
    if (lane == 0) {
      mbd::mbar_wait(q_full, 0, status, MB_DEV_TIMEOUT_TMA);
      for (int st = 0; st < 2; ++st)
      {
        if (used_k & (1u << st))
          mbd::mbar_wait(&kfull[st], (used_k >> (2 + st)) & 1, status, MB_DEV_TIMEOUT_TMA);
        if (used_v & (1u << st))
          mbd::mbar_wait(&vfull[st], (used_v >> (2 + st)) & 1, status, MB_DEV_TIMEOUT_TMA);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc_s = mbd::make_idesc(1u, TQ, TK, 0, 0);
    constexpr uint32_t idesc_pv = mbd::make_idesc(1u, TQ, DHT, 0, 1);
    const uint32_t sq = mbd::smem_u32(base);
    bool ok = __all_sync(0xffffffffu,
                         mbd::mbar_wait(q_full, 0, status, MB_DEV_TIMEOUT_MMA, abort_flag));
    for (int j = 0; ok && j <= n_tiles; ++j) {
      if (j < n_tiles) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        ok = __all_sync(0xffffffffu, mbd::mbar_wait(&kfull[st], ph, status, MB_DEV_TIMEOUT_MMA,
                                                    abort_flag) &&
                                         mbd::mbar_wait(&sfree[st], ph ^ 1, status,
                                                        MB_DEV_TIMEOUT_MMA, abort_flag));
        if (!ok) break;
        mbd::tc_fence_after();
        if (lane == 0) {
          const uint32_t sk = mbd::smem_u32(base + OFF_K + st * TILE);
#pragma unroll
          for (int kk = 0; kk < DHT / 16; ++kk)
            mbd::mma_f16(tS0 + st * TK, kmajor_desc(sq, kk), kmajor_desc(sk, kk), idesc_s,
                         kk > 0 ? 1u : 0u);
          mbd::mma_commit(&sfull[st]);
          mbd::mma_commit(&kempty[st]);
        }
        __syncwarp();
      }
      if (j >= 1) {
        const int pj = j - 1, pst = pj & 1;
        const uint32_t pph = (pj >> 1) & 1;
        bool got = mbd::mbar_wait(&pfull[pst], pph, status, MB_DEV_TIMEOUT_MMA, abort_flag) &&
                   mbd::mbar_wait(&vfull[pst], pph, status, MB_DEV_TIMEOUT_MMA, abort_flag);
        if (got && pj == n_tiles - 1)
          got = mbd::mbar_wait(vfix, 0, status, MB_DEV_TIMEOUT_MMA, abort_flag);
        ok = __all_sync(0xffffffffu, got);
        if (!ok) break;
        mbd::tc_fence_after();
        if (lane == 0) {
          const uint32_t sp = mbd::smem_u32(base + OFF_P + pst * TILE);
          const uint32_t sv = mbd::smem_u32(base + OFF_V + pst * TILE);
#pragma unroll
          for (int kk = 0; kk < TK / 16; ++kk)
            mbd::mma_f16(tO, kmajor_desc(sp, kk), mbd::sw128_desc(sv + kk * 2048, CHUNK, 1024),
                         idesc_pv, (pj > 0 || kk > 0) ? 1u : 0u);
          mbd::mma_commit(&pfree[pst]);
          mbd::mma_commit(&vempty[pst]);
        }
        __syncwarp();
      }
    }
    // ofinal: every MMA of this CTA has completed (also the drain before dealloc)
    if (lane == 0) mbd::mma_commit(ofinal);
    __syncwarp();
    mbd::mbar_wait(ofinal, 0, status, MB_DEV_TIMEOUT_MMA);
  } else {
    // ---------------- softmax + output (warps 2-9) ----------------
    const int quad = warp & 3;          // TMEM lane quadrant
    const int half = (warp - 2) >> 2;   // keys / O columns [64*half, 64*half + 64)
    const int r = quad * 32 + lane;     // query row of the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int row = q_first + r;
    const int qpos = p0 + row;
    const int c0 = half * 64;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    // Every iteration runs both pair barriers, also after a failed (timed
    // out) wait, so the two warps of a quadrant never wait for each other in
    // vain: a failure only skips the work.
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      if (ok)
        ok = __all_sync(0xffffffffu,
                        mbd::mbar_wait(&sfull[st], ph, status, MB_DEV_TIMEOUT_EPI, abort_flag));
      uint32_t s[4][16];
      if (ok) {
        mbd::tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) mbd::tmem_ld16(tS0 + st * TK + lane_off + c0 + c * 16, s[c]);
        mbd::tmem_ld_wait();
        mbd::tc_fence_before();
        mbd::mbar_arrive(&sfree[st]);
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 16; ++e) s[c][e] = 0u;
      }
      // mask in place; maximum of this half-row in 8 independent chains
      const int kbase = (jbase + j) * TK + c0;
      int kmax = L - 1;  // last key this row may see
      if (p.causal) kmax = min(kmax, qpos);
      const bool full = kbase + 63 <= kmax;
      float mx[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) mx[e] = -INFINITY;
      if (full) {  // the common case: no per-key compare at all
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 16; ++e) mx[e & 7] = fmaxf(mx[e & 7], __uint_as_float(s[c][e]));
      } else {
        const int lim = kmax - kbase;  // keys [0, lim] of this half-row are visible
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            if (c * 16 + e > lim) s[c][e] = __float_as_uint(-INFINITY);
            mx[e & 7] = fmaxf(mx[e & 7], __uint_as_float(s[c][e]));
          }
      }
      red[half * TQ + r] = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                 fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      pair_sync(quad);
      const float mt = fmaxf(red[r], red[TQ + r]) * p.scale_log2;
      pair_sync(quad);  // both read before either writes the next tile's
      float alpha = 1.f;
      bool rescale = false;
      if (mt > m + kRaise) {
        if (m != -INFINITY) {
          alpha = exp2f(m - mt);
          rescale = true;
        }
        m = mt;
      }
      const float mu = m == -INFINITY ? 0.f : m;
      // O columns that must follow the raised maximum: after P_{j-1} V_{j-1}
      if (ok && __any_sync(0xffffffffu, rescale)) {
        const int pj = j - 1;
        ok = __all_sync(0xffffffffu, mbd::mbar_wait(&pfree[pj & 1], (pj >> 1) & 1, status,
                                                    MB_DEV_TIMEOUT_EPI, abort_flag));
        if (ok) {
          mbd::tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t o[16];
            mbd::tmem_ld16(tO + lane_off + c0 + c * 16, o);
            mbd::tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st16(tO + lane_off + c0 + c * 16, o);
          }
          tmem_st_wait();
        }
      }
      // P tile st is free once P_{j-2} V_{j-2} has completed
      if (ok)
        ok = __all_sync(0xffffffffu, mbd::mbar_wait(&pfree[st], ph ^ 1, status,
                                                    MB_DEV_TIMEOUT_EPI, abort_flag));
      if (!ok) continue;
      uint8_t* prow = base + OFF_P + st * TILE + half * CHUNK + r * 128;
      const float scl = p.scale_log2;
      float sm[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) sm[e] = 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) {  // 8 keys = one 16-byte unit
        float e8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          e8[e] = ex2(fmaf(__uint_as_float(s[u >> 1][(u & 1) * 8 + e]), scl, -mu));
          sm[e] += e8[e];
        }
        const uint4 w = make_uint4(pack_bf16x2(e8[0], e8[1]), pack_bf16x2(e8[2], e8[3]),
                                   pack_bf16x2(e8[4], e8[5]), pack_bf16x2(e8[6], e8[7]));
        *reinterpret_cast<uint4*>(prow + ((u ^ (r & 7)) << 4)) = w;
      }
      l = l * alpha + (((sm[0] + sm[1]) + (sm[2] + sm[3])) + ((sm[4] + sm[5]) + (sm[6] + sm[7])));
      mbd::fence_proxy_async();
      mbd::tc_fence_before();
      mbd::mbar_arrive(&pfull[st]);
    }
    // all P V done: O / l -> bf16 half-row of the output
    const bool fin = ok && __all_sync(0xffffffffu, mbd::mbar_wait(ofinal, 0, status,
                                                                  MB_DEV_TIMEOUT_EPI, abort_flag));
    // row sum = both halves' sums (the exchange buffer is free: both threads
    // passed the second pair barrier of their last tile)
    red[half * TQ + r] = l;
    pair_sync(quad);
    const float lt = red[r] + red[TQ + r];
    if (fin && p.splits > 1) {
      // partial of this key split: unnormalised O, max (log2 units), row sum
      mbd::tc_fence_after();
      const int64_t prow = (((int64_t)b * p.Hq + h) * p.S + row) * p.splits + sp;
      float4* dst = reinterpret_cast<float4*>(p.part_o + prow * DHT + c0);
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[16];
        mbd::tmem_ld16(tO + lane_off + c0 + c * 16, o);
        mbd::tmem_ld_wait();
        if (row < p.S)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            dst[4 * c + e] = make_float4(__uint_as_float(o[4 * e]), __uint_as_float(o[4 * e + 1]),
                                         __uint_as_float(o[4 * e + 2]),
                                         __uint_as_float(o[4 * e + 3]));
      }
      if (row < p.S && half == 0) {
        p.part_ml[prow * 2] = m;
        p.part_ml[prow * 2 + 1] = lt;
      }
    } else if (fin) {
      mbd::tc_fence_after();
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      const uint32_t keep = lt > 0.f ? 0xFFFFFFFFu : 0u;  // no visible key: O was never written
      uint4* dst =
          reinterpret_cast<uint4*>(p.out + ((int64_t)b * p.S + row) * p.ldo + h * DHT + c0);
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[16];
        mbd::tmem_ld16(tO + lane_off + c0 + c * 16, o);
        mbd::tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) o[e] &= keep;
        if (row < p.S) {
          uint4 w0, w1;
          w0.x = pack_bf16x2(__uint_as_float(o[0]) * inv, __uint_as_float(o[1]) * inv);
          w0.y = pack_bf16x2(__uint_as_float(o[2]) * inv, __uint_as_float(o[3]) * inv);
          w0.z = pack_bf16x2(__uint_as_float(o[4]) * inv, __uint_as_float(o[5]) * inv);
          w0.w = pack_bf16x2(__uint_as_float(o[6]) * inv, __uint_as_float(o[7]) * inv);
          w1.x = pack_bf16x2(__uint_as_float(o[8]) * inv, __uint_as_float(o[9]) * inv);
          w1.y = pack_bf16x2(__uint_as_float(o[10]) * inv, __uint_as_float(o[11]) * inv);
          w1.z = pack_bf16x2(__uint_as_float(o[12]) * inv, __uint_as_float(o[13]) * inv);
          w1.w = pack_bf16x2(__uint_as_float(o[14]) * inv, __uint_as_float(o[15]) * inv);
          dst[2 * c] = w0;
          dst[2 * c + 1] = w1;
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    mbd::tc_fence_after();
    mbd::tmem_dealloc(tmem, 512);
  }
}

// out row = sum_s O_s 2^(m_s - M) / sum_s l_s 2^(m_s - M), M = max_s m_s;
// one 128-thread block per (sequence, head, query row), thread = dim
__global__ void __launch_bounds__(128) attn_split_combine_kernel(
    const float* __restrict__ part_o, const float* __restrict__ part_ml, int S, int Hq,
    int splits, uint16_t* __restrict__ out, int ldo) {
  const int64_t rid = blockIdx.x;  // (b * Hq + h) * S + row
  const int row = (int)(rid % S);
  const int h = (int)((rid / S) % Hq);
  const int64_t b = rid / ((int64_t)S * Hq);
  const float* ml = part_ml + rid * splits * 2;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, ml[2 * s]);
  float acc = 0.f, lsum = 0.f;
  for (int s = 0; s < splits; ++s) {
    if (ml[2 * s] == -INFINITY) continue;  // a split with no visible key: O never written
    const float w = exp2f(ml[2 * s] - M);
    lsum += w * ml[2 * s + 1];
    acc += w * part_o[(rid * splits + s) * DHT + threadIdx.x];
  }
  const float v = lsum > 0.f ? acc / lsum : 0.f;
  __nv_bfloat16 hv = __float2bfloat16_rn(v);
  out[(b * S + row) * (int64_t)ldo + h * DHT + threadIdx.x] = *reinterpret_cast<uint16_t*>(&hv);
}

}  // namespace

namespace mb {

int attention_split_plan(int64_t B, int64_t S, int64_t Hq, int64_t kv_len) {
  const int64_t ctas = B * Hq * ((S + TQ - 1) / TQ);
  const int64_t tiles = (kv_len + TK - 1) / TK;
  int64_t splits = num_sms() / std::max<int64_t>(ctas, 1);
  splits = std::min<int64_t>(splits, tiles / 2);
  return (int)std::max<int64_t>(splits, 1);
}

// false (and nothing launched) when the operands do not fit the TMA path
bool attention_prefill_tc_ok(const uint16_t* q, int ldq, const uint16_t* k_cache,
                             const uint16_t* v_cache, uint16_t* out, int ldo) {
  auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  return ldq % 8 == 0 && ldo % 8 == 0 && al16(q) && al16(out) && al16(k_cache) && al16(v_cache) &&
         getenv("MB_ATTN_NO_TC") == nullptr;
}

int attention_prefill_tc(const uint16_t* q, int ldq, const uint16_t* k_cache,
                         const uint16_t* v_cache, const int* block_table, int max_pages,
                         const int* start_pos, const int* kv_len, int B, int S, int Hq, int Hkv,
                         int causal, uint16_t* out, int ldo, cudaStream_t stream, int splits,
                         int max_kv_len, float* part_o, float* part_ml) {
  MB_REQUIRE(splits == 1 || (!causal && part_o && part_ml && max_kv_len > 0),
             "attention: split-KV needs a non-causal call, max_kv_len and partial buffers");
  AttnTcParams p;
  const auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const auto sw = CU_TENSOR_MAP_SWIZZLE_128B;
  int rc = make_tmap_2d(&p.qmap, q, bf, 2, (uint64_t)ldq, (uint64_t)B * S, (uint64_t)ldq * 2, 64,
                        TQ, sw);
  // the cache's page count is not part of the interface: rows are addressed
  // only through the block table, so the row extent is left open
  const uint64_t cache_rows = uint64_t(1) << 31;
  if (!rc) rc = make_tmap_2d(&p.kmap, k_cache, bf, 2, DHT, cache_rows, DHT * 2, 64, PGK, sw);
  if (!rc) rc = make_tmap_2d(&p.vmap, v_cache, bf, 2, DHT, cache_rows, DHT * 2, 64, PGK, sw);
  if (rc) return rc;
  p.block_table = block_table;
  p.max_pages = max_pages;
  p.start_pos = start_pos;
  p.kv_len = kv_len;
  p.S = S;
  p.Hkv = Hkv;
  p.G = Hq / Hkv;
  p.causal = causal;
  p.n_qt = (S + TQ - 1) / TQ;
  p.scale_log2 = 1.4426950408889634f / sqrtf((float)DHT);
  p.out = out;
  p.ldo = ldo;
  p.splits = splits;
  p.Hq = Hq;
  p.part_o = part_o;
  p.part_ml = part_ml;
  p.tiles_per_split = splits == 1 ? (1 << 30)
                                  : ((max_kv_len + TK - 1) / TK + splits - 1) / splits;
  {
    const int arc =
        mb::ensure_smem_attr(reinterpret_cast<const void*>(attn_prefill_tc_kernel), SMEM_BYTES);
    if (arc) return arc;
  }
  dim3 grid((unsigned)(p.n_qt * splits), (unsigned)Hq, (unsigned)B);
  attn_prefill_tc_kernel<<<grid, 64 + NSOFT, SMEM_BYTES, stream>>>(p, device_status_ptr());
  MB_CUDA(cudaGetLastError());
  if (splits > 1) {
    attn_split_combine_kernel<<<(unsigned)((int64_t)B * Hq * S), 128, 0, stream>>>(
        part_o, part_ml, S, Hq, splits, out, ldo);
    MB_CUDA(cudaGetLastError());
  }
  return MB_OK;
}

}  // namespace mb
