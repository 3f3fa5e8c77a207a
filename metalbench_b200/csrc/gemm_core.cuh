// Persistent, warp-specialised tcgen05 GEMM core for sm_100a.
//
//   D[M, N] = sum_k A[m, k] * B[n, k]       (A: M x K, K contiguous)
//   B is either K-major ([N, K], K contiguous) or MN-major ([K, N], N contiguous).
//
// One CTA per SM walks a static list of output tiles (BM = 128 rows x BN
// columns, optionally split along K). Roles inside the CTA:
//   warp 0      TMA producer: fills a STAGES-deep ring of 128-byte-swizzled
//               A/B tiles (64 bf16 or 32 fp32 of K per stage).
//   warp 1      MMA issuer: one elected thread issues tcgen05.mma into one of
//               two TMEM accumulators (128 lanes x BN fp32 columns each) and
//               frees ring slots with tcgen05.commit.
//   warp 2      allocates / frees TMEM.
//   warps 4-7   epilogue: tcgen05.ld the finished accumulator (warp w owns
//               TMEM lanes 32*(w%4)..+31 = tile rows), apply the fused
//               epilogue functor, store; then hand the accumulator back.
// TF32x3 mode streams four K-major fp32 operands per stage (A_hi, B_hi, A_lo,
// B_lo, produced by a split prepass: hi = low 13 mantissa bits cleared, lo =
// the exact remainder) and issues lo*hi + hi*lo + hi*hi per k-step.
// With two accumulators the epilogue of tile i overlaps the main loop of
// tile i+1. Every mbarrier wait is bounded (common.cuh) and reports through
// the device status word instead of hanging.
#pragma once
#include <type_traits>

#include "common.cuh"

namespace gemm {

constexpr int BM = 128;
constexpr int KBYTES = 128;  // K extent of one stage in bytes (one swizzle row)

enum class Mode { BF16 = 0, TF32X3 = 1 };

__host__ __device__ constexpr int elem_bytes(Mode m) { return m == Mode::BF16 ? 2 : 4; }

// Shared-memory plan: [resident operand (optional)][STAGES x stage][barriers].
template <class Producer, int BN, int STAGES>
struct Smem {
  static constexpr int RES_BYTES = (Producer::RESIDENT_BYTES + 1023) / 1024 * 1024;
  static constexpr int STAGE_BYTES = Producer::STAGE_BYTES;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  // barriers: full, empty per stage; tfull, tempty x2; resident;
  // then tmem slot, abort flag, drain barrier
  static constexpr int BAR_BYTES = 8 * (2 * STAGES + 5) + 16;
  // work list (int4 per unit, Sched::MAX_LISTED of them), 16-byte aligned
  static constexpr int WORK_OFF = (RES_BYTES + RING_BYTES + BAR_BYTES + 15) / 16 * 16;
  static constexpr int WORK_BYTES = 16 * 64;
  static constexpr int TOTAL = 1024 /*alignment slack*/ + WORK_OFF + WORK_BYTES;
  static constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
};

// Integer a / d for 0 <= a, d >= 1 without the ~20-instruction integer
// division sequence: a float product with 1/d, then one correction step (the
// estimate is off by at most one while a < 2^24; larger a divides exactly).
// The schedule and epilogue index maths run on single threads whose latency
// sits between consecutive tiles, so this matters for short tiles.
struct FastDiv {
  int d = 1;
  float r = 1.f;
  __host__ __device__ void set(int dd) {
    d = dd;
    r = 1.f / (float)dd;
  }
  __device__ __forceinline__ int div(int a) const {
    if (a >= (1 << 24)) return a / d;
    int q = (int)((float)a * r);
    const int rem = a - q * d;
    if (rem < 0) --q;
    else if (rem >= d) ++q;
    return q;
  }
  __device__ __forceinline__ int mod(int a) const { return a - div(a) * d; }
};

// Static tile list, rasterised in groups of GROUP_M tile-rows so that CTAs
// running at the same time share A panels and B panels in L2.
struct Sched {
  int tiles_m, tiles_n, ksplit, kblocks, kb_per_split;
  static constexpr int GROUP_M = 16;
  // reciprocals for get()/next(), filled on the device by init_fast()
  FastDiv fd_ksplit, fd_group, fd_gm, fd_glast, fd_kblocks, fd_skper;
  __device__ void init_fast() {
    fd_ksplit.set(ksplit);
    fd_group.set(GROUP_M * tiles_n);
    fd_gm.set(GROUP_M);
    fd_glast.set(tiles_m - (tiles_m - 1) / GROUP_M * GROUP_M);
    fd_kblocks.set(kblocks);
    fd_skper.set(sk_per > 0 ? sk_per : 1);
  }
  __host__ __device__ int total() const { return tiles_m * tiles_n * ksplit; }
  __device__ void get(int t, int& tm, int& tn, int& ks) const {
    const int tq = fd_ksplit.div(t);
    ks = t - tq * ksplit;
    const int g = fd_group.div(tq);
    const int first = g * GROUP_M;
    const FastDiv& gs = tiles_m - first < GROUP_M ? fd_glast : fd_gm;
    const int r = tq - g * fd_group.d;
    tn = gs.div(r);
    tm = first + r - tn * gs.d;
  }
  __device__ void krange(int ks, int& kb0, int& kb1) const {
    kb0 = ks * kb_per_split;
    kb1 = min(kblocks, kb0 + kb_per_split);
  }

  // Stream-K mode: the (tile, k-block) sequence tile-major is cut into equal
  // contiguous ranges of sk_per k-blocks, one per CTA, so every SM gets the
  // same amount of work whatever the tile count. A tile cut by range borders
  // is computed as several "segments"; segment s of tile t is produced by CTA
  // floor(t*kblocks/sk_per) + s and the caller sums the segment partials.
  int streamk = 0;
  int sk_per = 0;

  // Work unit u of this CTA: tile (tm, tn), split/segment index seg and
  // k-blocks [kb0, kb1); false past the last unit. Static mode: tiles
  // blockIdx.x + u*gridDim.x. Stream-K: the tiles that this CTA's k-block
  // range [blockIdx.x*sk_per, +sk_per) touches, in order. The kernel lists the
  // first MAX_LISTED units in shared memory once, in parallel (warp 3, while
  // TMEM is allocated), because computing one costs a single thread about 600
  // cycles, which every role would otherwise pay between consecutive tiles.
  static constexpr int MAX_LISTED = 64;
  __device__ bool unit(int u, int& tm, int& tn, int& seg, int& kb0, int& kb1) const {
    if (streamk) {
      const int p0 = blockIdx.x * sk_per;
      const int p1 = min(p0 + sk_per, tiles_m * tiles_n * kblocks);
      if (p0 >= p1) return false;
      const int tile = fd_kblocks.div(p0) + u;
      const int t0 = tile * kblocks;
      if (t0 >= p1) return false;
      kb0 = max(p0 - t0, 0);
      kb1 = min(p1 - t0, kblocks);
      int dummy;
      get(tile, tm, tn, dummy);
      seg = blockIdx.x - fd_skper.div(t0);
      return true;
    }
    const int t = blockIdx.x + u * gridDim.x;
    if (t >= total()) return false;
    get(t, tm, tn, seg);
    krange(seg, kb0, kb1);
    return true;
  }

};

// 32 consecutive fp32 accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32_raw(uint32_t taddr, float (&v)[32]) {
  uint32_t r[16], t[16];
  mbd::tmem_ld16(taddr, r);
  mbd::tmem_ld16(taddr + 16, t);
  mbd::tmem_ld_wait();
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    v[j] = __uint_as_float(r[j]);
    v[16 + j] = __uint_as_float(t[j]);
  }
}

// Epilogue context handed to the functor for one tile: the TMEM address of
// this thread's row (lane) at column 0 of the accumulator, the global row,
// the first global column, the split index and whether the row is in range.
struct EpiCtx {
  uint32_t taddr;
  int row;
  int n0;
  int ks;
  bool row_ok;
  uint64_t* tempty;  // accumulator-free barrier (for epilogues that release early)
};

// An epilogue functor with `static constexpr bool kEarlyRelease = true` hands
// the accumulator back itself, as soon as its last tcgen05.ld has completed
// (release_acc below) and before its global stores, so the next tile's MMAs
// are not held up by them; the kernel then does not arrive for it.
template <class E, class = void>
struct EarlyRelease : std::false_type {};
template <class E>
struct EarlyRelease<E, std::void_t<decltype(E::kEarlyRelease)>>
    : std::integral_constant<bool, E::kEarlyRelease> {};

__device__ __forceinline__ void release_acc(const EpiCtx& c) {
  mbd::tc_fence_before();
  mbd::mbar_arrive(c.tempty);
}


// ---------------------------------------------------------------------------
// TMA producer for plain GEMM operands (2-D tensor maps, 128-byte swizzle).
//   A map: inner K, outer M, box {128 B of K, 128 rows}.
//   B K-major map: inner K, outer N, box {128 B of K, BN rows}.
//   B MN-major map: inner N, outer K, box {128 B of N, K rows of one stage};
//   BN / (128 B of N) boxes side by side (LBO apart) make one B stage.
// ---------------------------------------------------------------------------
template <Mode MODE, int BN, bool B_MN>
struct GemmProducer {
  CUtensorMap a, b, alo, blo;  // alo / blo: TF32x3 remainders (K-major)
  // Rows of A one stage actually loads (the A box height): BM, or the row count
  // rounded up to 16 when M < BM (decode). Rows past it keep stale shared data
  // that only reaches accumulator rows >= M, which no epilogue stores.
  uint32_t a_rows = BM;
  __device__ uint32_t stage_tx_bytes() const { return PARTS * (a_rows + BN) * KBYTES; }
  // Optional pre-tiled B (bf16, K-major, see tile_weights in gemm_launch.cuh):
  // tile (tn, kb) is BN*128 contiguous bytes already in the 128-byte-swizzled
  // shared-memory image, fetched with one bulk copy instead of a TMA box.
  const uint8_t* b_tiled = nullptr;
  int b_kblocks = 0;
  // Batched K-major B (TF32x3 batch_mm): tile row tm belongs to batch
  // tm / a_tiles_per_batch, whose B rows start at batch * b_rows_per_batch.
  int a_tiles_per_batch = 0;
  int b_rows_per_batch = 0;
  __device__ int b_row(int tm, int tn) const {
    return (a_tiles_per_batch ? tm / a_tiles_per_batch * b_rows_per_batch : 0) + tn * BN;
  }
  static constexpr int KE = KBYTES / elem_bytes(MODE);  // K elements per stage
  static constexpr int PARTS = MODE == Mode::TF32X3 ? 2 : 1;
  static constexpr uint32_t BYTES = PARTS * (BM + BN) * KBYTES;
  static constexpr int STAGE_BYTES = PARTS * (BM + BN) * KBYTES;
  static constexpr int RESIDENT_BYTES = 0;
  __device__ uint32_t resident_tx_bytes() const { return 0; }
  static constexpr int B_BOX_BYTES = KE * KBYTES;       // one MN-major box
  static_assert(MODE == Mode::BF16 || !B_MN, "TF32x3 operands are K-major");
  __device__ void prefetch() const {
    mbd::prefetch_tmap(&a);
    mbd::prefetch_tmap(&b);
    if constexpr (MODE == Mode::TF32X3) {
      mbd::prefetch_tmap(&alo);
      mbd::prefetch_tmap(&blo);
    }
  }
  // Stage layout: [A hi][B hi]([A lo][B lo]).
  __device__ void load(uint8_t* st, uint64_t* bar, int tm, int tn, int kb) const {
    uint8_t* sA = st;
    uint8_t* sB = st + BM * KBYTES;
    mbd::tma_load_2d(sA, &a, bar, kb * KE, tm * BM);
    if constexpr (!B_MN) {
      if (b_tiled)
        mbd::bulk_load(sB, b_tiled + ((size_t)tn * b_kblocks + kb) * (BN * KBYTES), BN * KBYTES,
                       bar);
      else
        mbd::tma_load_2d(sB, &b, bar, kb * KE, b_row(tm, tn));
    } else {
#pragma unroll
      for (int j = 0; j < BN / KE; ++j)
        mbd::tma_load_2d(sB + j * B_BOX_BYTES, &b, bar, tn * BN + j * KE, kb * KE);
    }
    if constexpr (MODE == Mode::TF32X3) {
      mbd::tma_load_2d(sB + BN * KBYTES, &alo, bar, kb * KE, tm * BM);
      mbd::tma_load_2d(sB + BN * KBYTES + BM * KBYTES, &blo, bar, kb * KE, b_row(tm, tn));
    }
  }
  // Shared-memory descriptors for MMA k-step kk of a stage.
  static constexpr int KSTEPS = 4;  // 16 bf16 or 8 tf32 per MMA = 32 bytes of K
  __device__ static uint64_t a_desc(uint32_t sA, int kk) {
    return mbd::sw128_desc(sA + kk * 32, 16, 1024);
  }
  __device__ static uint64_t b_desc(uint32_t sB, int kk) {
    if constexpr (!B_MN) return mbd::sw128_desc(sB + kk * 32, 16, 1024);
    // MN-major: one k-step is 16 bf16 = two 8-row groups, or 8 tf32 = one.
    constexpr int step = MODE == Mode::BF16 ? 2048 : 1024;
    return mbd::sw128_desc(sB + kk * step, B_BOX_BYTES, 1024);
  }
  __device__ void load_resident(uint8_t*, uint64_t*) const {}
  // All MMAs of one stage (k-block kb of output tile row tm) into accumulator
  // d; `first` starts a fresh sum.
  __device__ void issue(uint32_t d, uint32_t st, uint32_t /*res*/, int /*tm*/, int /*kb*/,
                        bool first) const {
    constexpr uint32_t fmt = MODE == Mode::BF16 ? 1u : 2u;
    constexpr uint32_t idesc = mbd::make_idesc(fmt, BM, BN, 0, B_MN ? 1u : 0u);
    const uint32_t a0 = st, b0 = st + BM * KBYTES;
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
      const uint32_t acc = (!first || kk > 0) ? 1u : 0u;
      const uint64_t ad = a_desc(a0, kk), bd = b_desc(b0, kk);
      if constexpr (MODE == Mode::BF16) {
        mbd::mma_f16(d, ad, bd, idesc, acc);
      } else {
        // stage layout [A hi][B hi][A lo][B lo]
        const uint32_t alo = b0 + BN * KBYTES, blo = alo + BM * KBYTES;
        mbd::mma_tf32(d, a_desc(alo, kk), bd, idesc, acc);  // lo * hi
        mbd::mma_tf32(d, ad, b_desc(blo, kk), idesc, 1u);   // hi * lo
        mbd::mma_tf32(d, ad, bd, idesc, 1u);                // hi * hi
      }
    }
  }
};

// Decode-size producer (bf16, both operands K-major): A, the activations, has
// at most AROWS rows, so a stage holds an AROWS-row A box followed by the
// BN-row weight box, and the ring can be deeper than with 128-row A tiles.
// The MMA still reads 128 A rows; rows AROWS..127 alias the start of the B box
// and only reach accumulator rows >= M, which no epilogue stores.
template <int BN, int AROWS>
struct DecodeProducer {
  CUtensorMap a, b;
  static constexpr int KE = 64;
  static constexpr int STAGE_BYTES = (AROWS + BN) * KBYTES;
  static constexpr int RESIDENT_BYTES = 0;
  static_assert((AROWS * KBYTES) % 1024 == 0, "B box must stay swizzle-atom aligned");
  uint32_t a_rows;  // <= AROWS, multiple of 16
  const uint8_t* b_tiled = nullptr;  // pre-tiled B (as GemmProducer::b_tiled)
  int b_kblocks = 0;
  __device__ uint32_t stage_tx_bytes() const { return (a_rows + BN) * KBYTES; }
  __device__ uint32_t resident_tx_bytes() const { return 0; }
  __device__ void prefetch() const {
    mbd::prefetch_tmap(&a);
    mbd::prefetch_tmap(&b);
  }
  __device__ void load_resident(uint8_t*, uint64_t*) const {}
  // B is the layer's packed weight, which no kernel of the stream writes: the
  // kernel requests the B boxes of its first ring stages before it waits for
  // the previous kernel (programmatic dependent launch), so the weight stream
  // overlaps that kernel's tail; A, the activations, follows after the wait.
  static constexpr bool PRELOAD_B = true;
  __device__ void load_a(uint8_t* st, uint64_t* bar, int tm, int, int kb) const {
    mbd::tma_load_2d(st, &a, bar, kb * KE, tm * BM);
  }
  __device__ void load_b(uint8_t* st, uint64_t* bar, int, int tn, int kb) const {
    if (b_tiled)
      mbd::bulk_load(st + AROWS * KBYTES, b_tiled + ((size_t)tn * b_kblocks + kb) * (BN * KBYTES),
                     BN * KBYTES, bar);
    else
      mbd::tma_load_2d(st + AROWS * KBYTES, &b, bar, kb * KE, tn * BN);
  }
  __device__ void load(uint8_t* st, uint64_t* bar, int tm, int tn, int kb) const {
    mbd::tma_load_2d(st, &a, bar, kb * KE, tm * BM);
    if (b_tiled)
      mbd::bulk_load(st + AROWS * KBYTES, b_tiled + ((size_t)tn * b_kblocks + kb) * (BN * KBYTES),
                     BN * KBYTES, bar);
    else
      mbd::tma_load_2d(st + AROWS * KBYTES, &b, bar, kb * KE, tn * BN);
  }
  __device__ void issue(uint32_t d, uint32_t st, uint32_t, int, int, bool first) const {
    constexpr uint32_t idesc = mbd::make_idesc(1u, BM, BN, 0, 0);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
      mbd::mma_f16(d, mbd::sw128_desc(st + kk * 32, 16, 1024),
                   mbd::sw128_desc(st + AROWS * KBYTES + kk * 32, 16, 1024), idesc,
                   (!first || kk > 0) ? 1u : 0u);
  }
};

// preload_b<P>::value: P::PRELOAD_B when the producer declares it.
template <class P, class = void>
struct preload_b : std::false_type {};
template <class P>
struct preload_b<P, std::void_t<decltype(P::PRELOAD_B)>> : std::bool_constant<P::PRELOAD_B> {};

// PROMOTE > 0: the accumulation is cut into chunks of PROMOTE k-blocks. Each
// chunk is summed by the tensor core into a fresh TMEM accumulator and the
// epilogue warps add the chunks in fp32 registers (round-to-nearest CUDA-core
// adds), then call epi.store_acc(ctx, acc). The tensor core's own fp32
// accumulation aligns the addends to the running sum and drops the bits below
// it, so its error grows with the magnitude of the sum; restarting it every
// chunk keeps that error at the level of a PROMOTE-block sum.
template <int BN, int STAGES, class Producer, class Epi, int PROMOTE = 0>
__global__ void __launch_bounds__(256, 1)
    gemm_kernel(const __grid_constant__ Producer prod, const __grid_constant__ Epi epi,
                const Sched sched_in, uint32_t* status) {
  using S = Smem<Producer, BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* res = base;  // resident operand (Producer::RESIDENT_BYTES)
  uint8_t* ring = base + S::RES_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + S::RING_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* res_full = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(res_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* drain = reinterpret_cast<uint64_t*>(tmem_slot + 2);
  int4* work = reinterpret_cast<int4*>(base + S::WORK_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  Sched sched = sched_in;
  sched.init_fast();
  auto sA = [&](int s) { return ring + s * S::STAGE_BYTES; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbd::mbar_init(&full[s], 1);
      mbd::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbd::mbar_init(&tfull[b], 1);
      mbd::mbar_init(&tempty[b], 128);
    }
    mbd::mbar_init(drain, 1);
    mbd::mbar_init(res_full, 1);
    *abort_flag = 0;
    mbd::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) prod.prefetch();
  if (warp == 2) mbd::tmem_alloc(tmem_slot, S::TMEM_COLS);
  if (warp == 3) {
    for (int u = lane; u < Sched::MAX_LISTED; u += 32) {
      int tm, tn, sg, k0, k1;
      work[u] = sched.unit(u, tm, tn, sg, k0, k1) ? make_int4(tm, tn, sg, k0 | (k1 << 16))
                                                  : make_int4(-1, 0, 0, 0);
    }
  }
  // unit u of this CTA: from the list, or computed past its end
  auto unit = [&](int u, int& tm, int& tn, int& sg, int& k0, int& k1) -> bool {
    if (u < Sched::MAX_LISTED) {
      const int4 w = work[u];
      if (w.x < 0) return false;
      tm = w.x;
      tn = w.y;
      sg = w.z;
      k0 = w.w & 0xFFFF;
      k1 = w.w >> 16;
      return true;
    }
    return sched.unit(u, tm, tn, sg, k0, k1);
  };
  __syncthreads();
  mbd::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // set-up above overlaps the previous kernel when launched with PDL
  mbd::pdl_trigger();
  int npre = 0;  // leading ring stages whose B box was requested before the wait
  if constexpr (preload_b<Producer>::value) {
    if (warp == 0) {
      if (lane == 0) {
        int tm, tn, ks, kb0, kb1;
        for (int u = 0; npre < STAGES && unit(u, tm, tn, ks, kb0, kb1); ++u)
          for (int kb = kb0; kb < kb1 && npre < STAGES; ++kb, ++npre) {
            mbd::mbar_expect_tx(&full[npre], prod.stage_tx_bytes());
            prod.load_b(sA(npre), &full[npre], tm, tn, kb);
          }
      }
      npre = __shfl_sync(0xffffffffu, npre, 0);
    }
  }
  mbd::pdl_wait();

  // The producer and MMA warps run their loops with all 32 lanes (waits on
  // every lane, agreed by a warp vote) and only lane 0 issues the TMA copies,
  // MMAs and commits: a warp whose lanes 1-31 sat at the final barrier while
  // lane 0 looped measurably slowed lane 0 down (hundreds of cycles per tile).
  if (warp == 0) {
    // ---------------- TMA producer ----------------
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued = 0;  // bit s: parity of the last load issued into stage s
    uint32_t used = 0;    // bit s: stage s received at least one load
    bool ok = true;
    if constexpr (Producer::RESIDENT_BYTES > 0) {
      if (lane == 0) {
        mbd::mbar_expect_tx(res_full, prod.resident_tx_bytes());
        prod.load_resident(res, res_full);
      }
      __syncwarp();
    }
    int tm, tn, ks, kb0, kb1;
    int cnt = 0;
    for (int u = 0; ok && unit(u, tm, tn, ks, kb0, kb1); ++u) {
      for (int kb = kb0; kb < kb1; ++kb, ++cnt) {
        if (cnt < npre) {  // first use of this stage; its B box is on the way
          if constexpr (preload_b<Producer>::value) {
            if (lane == 0) prod.load_a(sA(stage), &full[stage], tm, tn, kb);
          }
        } else {
          const bool got =
              mbd::mbar_wait(&empty[stage], phase ^ 1, status, MB_DEV_TIMEOUT_TMA, abort_flag);
          if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            break;
          }
          if (lane == 0) {
            mbd::mbar_expect_tx(&full[stage], prod.stage_tx_bytes());
            prod.load(sA(stage), &full[stage], tm, tn, kb);
          }
        }
        __syncwarp();
        issued = (issued & ~(1u << stage)) | (phase << stage);
        used |= 1u << stage;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    // Never leave a bulk copy in flight into shared memory we are about to
    // release: wait (bounded) for the last load of every stage.
    for (int s = 0; s < STAGES; ++s)
      if (used & (1u << s)) mbd::mbar_wait(&full[s], (issued >> s) & 1, status, MB_DEV_TIMEOUT_TMA);
    if constexpr (Producer::RESIDENT_BYTES > 0) mbd::mbar_wait(res_full, 0, status, MB_DEV_TIMEOUT_TMA);
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    if constexpr (Producer::RESIDENT_BYTES > 0)
      ok = __all_sync(0xffffffffu, mbd::mbar_wait(res_full, 0, status, MB_DEV_TIMEOUT_MMA, abort_flag));
    const uint32_t res_u32 = mbd::smem_u32(res);
    int i = 0;
    int tm, tn, ks, kb0, kb1;
    for (int u = 0; ok && unit(u, tm, tn, ks, kb0, kb1); ++u) {
      const int nch = PROMOTE > 0 ? (kb1 - kb0 + PROMOTE - 1) / PROMOTE : 1;
      for (int ch = 0; ok && ch < nch; ++ch, ++i) {
        const int ka = PROMOTE > 0 ? kb0 + ch * PROMOTE : kb0;
        const int kz = PROMOTE > 0 ? min(kb1, ka + PROMOTE) : kb1;
        const int buf = i & 1;
        const uint32_t tph = (i >> 1) & 1;
        const bool got =
            mbd::mbar_wait(&tempty[buf], tph ^ 1, status, MB_DEV_TIMEOUT_MMA, abort_flag);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        mbd::tc_fence_after();
        const uint32_t d = tmem + buf * BN;
        for (int kb = ka; kb < kz; ++kb) {
          const bool landed =
              mbd::mbar_wait(&full[stage], phase, status, MB_DEV_TIMEOUT_MMA, abort_flag);
          if (!__all_sync(0xffffffffu, landed)) {
            ok = false;
            break;
          }
          mbd::tc_fence_after();
          if (lane == 0) {
            prod.issue(d, mbd::smem_u32(sA(stage)), res_u32, tm, kb, kb == ka);
            mbd::mma_commit(&empty[stage]);
          }
          __syncwarp();
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok && lane == 0) mbd::mma_commit(&tfull[buf]);
        __syncwarp();
      }
    }
    // All MMAs issued by lane 0 are complete before TMEM is freed.
    if (lane == 0) mbd::mma_commit(drain);
    __syncwarp();
    mbd::mbar_wait(drain, 0, status, MB_DEV_TIMEOUT_MMA);
  } else if (warp >= 4 && warp < 8) {
    // ---------------- epilogue ----------------
    const int q = warp & 3;
    int i = 0;
    int tm, tn, ks, kb0, kb1;
    bool ok = true;
    for (int u = 0; ok && unit(u, tm, tn, ks, kb0, kb1); ++u) {
      EpiCtx c;
      c.row = tm * BM + q * 32 + lane;
      c.n0 = tn * BN;
      c.ks = ks;
      c.row_ok = c.row < epi.M;
      if constexpr (PROMOTE > 0) {
        float acc[BN];
#pragma unroll
        for (int j = 0; j < BN; ++j) acc[j] = 0.f;
        const int nch = (kb1 - kb0 + PROMOTE - 1) / PROMOTE;
        for (int ch = 0; ch < nch; ++ch, ++i) {
          const int buf = i & 1;
          const uint32_t tph = (i >> 1) & 1;
          const bool got = mbd::mbar_wait(&tfull[buf], tph, status, MB_DEV_TIMEOUT_EPI, abort_flag);
          if (!mbd::vote_all(got, 2, 128)) {
            ok = false;
            break;
          }
          mbd::tc_fence_after();
          const uint32_t ta = tmem + buf * BN + ((uint32_t)(q * 32) << 16);
#pragma unroll
          for (int c0 = 0; c0 < BN; c0 += 32) {
            float v[32];
            tmem_ld32_raw(ta + c0, v);
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[c0 + j] += v[j];
          }
          mbd::tc_fence_before();
          mbd::mbar_arrive(&tempty[buf]);
        }
        if (!ok) break;
        epi.store_acc(c, acc);
      } else {
        const int buf = i & 1;
        const uint32_t tph = (i >> 1) & 1;
        const bool got = mbd::mbar_wait(&tfull[buf], tph, status, MB_DEV_TIMEOUT_EPI, abort_flag);
        // the four epilogue warps continue or stop together, so an epilogue may
        // use a named barrier among them
        if (!mbd::vote_all(got, 2, 128)) break;
        mbd::tc_fence_after();
        c.taddr = tmem + buf * BN + ((uint32_t)(q * 32) << 16);
        c.tempty = &tempty[buf];
        epi(c);
        if constexpr (!EarlyRelease<Epi>::value) {
          mbd::tc_fence_before();
          mbd::mbar_arrive(&tempty[buf]);
        }
        ++i;
      }
    }
  }
  __syncthreads();
  if (warp == 2) {
    mbd::tc_fence_after();
    mbd::tmem_dealloc(tmem, S::TMEM_COLS);
  }
}

}  // namespace gemm
