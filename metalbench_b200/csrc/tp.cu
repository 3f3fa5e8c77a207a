// Tensor-parallel communicator: one process per GPU, NCCL over NVLink /
// NVSwitch. The reference has no distributed code; this backs the row-sharded
// o-proj and down-proj of the decoder (one bf16 sum all-reduce each).
//
// Set-up is bounded: rank 0 writes the NCCL unique id to `nccl_id_path`
// (write to a temporary name, then rename, so readers never see a partial
// file); the other ranks poll for it until `timeout_ms`. The communicator is
// created non-blocking and polled with ncclCommGetAsyncError until ready or
// the deadline, after which it is aborted and MB_ERR_TIMEOUT is returned.
#include <stdio.h>
#include <string.h>
#include <unistd.h>

#include <chrono>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"
#include "kernels.h"

#ifdef MB_HAVE_NCCL
#include <nccl.h>
#endif

namespace mb {

#ifdef MB_HAVE_NCCL
static ncclComm_t g_comm = nullptr;
static int g_world = 1;

static int nccl_fail(ncclResult_t r, const char* what) {
  set_error("NCCL error in %s: %s", what, ncclGetErrorString(r));
  return MB_ERR_NCCL;
}

static int wait_ready(int timeout_ms, const char* what) {
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = ncclCommGetAsyncError(g_comm, &st);
    if (r != ncclSuccess) return nccl_fail(r, what);
    if (st == ncclSuccess) return MB_OK;
    if (st != ncclInProgress) return nccl_fail(st, what);
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                        std::chrono::steady_clock::now() - t0)
                        .count();
    if (ms > timeout_ms) {
      ncclCommAbort(g_comm);
      g_comm = nullptr;
      set_error("%s timed out after %d ms", what, timeout_ms);
      return MB_ERR_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
}
#endif

#ifdef MB_HAVE_NCCL
static int p2p_setup(int rank, int world);
#endif
static void p2p_teardown();

int tp_init(int rank, int world, const char* nccl_id_path, int timeout_ms) {
#ifdef MB_HAVE_NCCL
  if (timeout_ms <= 0) timeout_ms = 60000;
  if (!nccl_id_path || !*nccl_id_path) {
    set_error("mb_init: world > 1 needs an nccl_id_path");
    return MB_ERR_BAD_ARG;
  }
  if (rank < 0 || rank >= world) {
    set_error("mb_init: rank %d out of range for world %d", rank, world);
    return MB_ERR_BAD_ARG;
  }
  ncclUniqueId id;
  if (rank == 0) {
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    const std::string tmp = std::string(nccl_id_path) + ".tmp";
    FILE* f = fopen(tmp.c_str(), "wb");
    if (!f || fwrite(&id, sizeof(id), 1, f) != 1) {
      if (f) fclose(f);
      set_error("mb_init: cannot write %s", tmp.c_str());
      return MB_ERR_BAD_ARG;
    }
    fclose(f);
    if (rename(tmp.c_str(), nccl_id_path) != 0) {
      set_error("mb_init: cannot rename to %s", nccl_id_path);
      return MB_ERR_BAD_ARG;
    }
  } else {
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
      FILE* f = fopen(nccl_id_path, "rb");
      if (f) {
        const size_t n = fread(&id, sizeof(id), 1, f);
        fclose(f);
        if (n == 1) break;
      }
      const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                          std::chrono::steady_clock::now() - t0)
                          .count();
      if (ms > timeout_ms) {
        set_error("mb_init: rank %d saw no NCCL id at %s within %d ms", rank, nccl_id_path,
                  timeout_ms);
        return MB_ERR_TIMEOUT;
      }
      std::this_thread::sleep_for(std::chrono::milliseconds(5));
    }
  }
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = ncclCommInitRankConfig(&g_comm, world, id, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "ncclCommInitRankConfig");
  int rc = wait_ready(timeout_ms, "NCCL communicator set-up");
  if (rc) return rc;
  g_world = world;
  if (getenv("MB_TP_NCCL") == nullptr) {  // map the peers for the fused peer reduction
    rc = p2p_setup(rank, world);
    if (rc) return rc;
  }
  return MB_OK;
#else
  (void)rank; (void)world; (void)nccl_id_path; (void)timeout_ms;
  set_error("mb_init: built without NCCL");
  return MB_ERR_NCCL;
#endif
}

void tp_shutdown() {
  p2p_teardown();
#ifdef MB_HAVE_NCCL
  if (g_comm) {
    ncclCommDestroy(g_comm);
    g_comm = nullptr;
  }
  g_world = 1;
#endif
}

int tp_allreduce_bf16(void* buf, size_t count, cudaStream_t stream) {
#ifdef MB_HAVE_NCCL
  if (!g_comm) {
    set_error("tensor-parallel all-reduce without a communicator (mb_init with world > 1)");
    return MB_ERR_NOT_INIT;
  }
  ncclResult_t r = ncclAllReduce(buf, buf, count, ncclBfloat16, ncclSum, g_comm, stream);
  if (r == ncclInProgress) return wait_ready(60000, "ncclAllReduce enqueue");
  if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce");
  return MB_OK;
#else
  (void)buf; (void)count; (void)stream;
  set_error("built without NCCL");
  return MB_ERR_NCCL;
#endif
}

// ---------------------------------------------------------------------------
// All-reduce over NVLink peer memory (one process per GPU, CUDA IPC).
//
// Every rank owns one region in its HBM, mapped by every peer at set-up
// (handles exchanged with one NCCL all-gather):
//   staging[2][MAXE] bf16   my partial, double-buffered by epoch parity
//   result [2][MAXE] bf16   two-shot: the reduced chunks pushed by their owners
//   flags  [64] u32         flags[r] = last epoch rank r published (peers write)
//   flags2 [64] u32         flags2[r] = last epoch rank r pushed its chunk
// plus private counters (epoch, CTA arrival counts). The epoch lives on the
// device, so a CUDA graph of a whole decode step replays correctly.
//
//   publish  : copy my partial into staging[e%2]; the last CTA fences at system
//              scope and stores e+1 into flags[my rank] of every peer (release),
//              then bumps my epoch.
//   one-shot : wait until every flags[r] >= e+1 (acquire), sum the W staging
//              slots over NVLink into the output (W-1 remote reads of n).
//   two-shot : wait likewise; sum only my chunk n/W, push it into result[e%2]
//              of every rank (remote stores), last CTA signals flags2; then
//              wait for every flags2[r] and copy my result slot to the output
//              (2(W-1)/W of n crosses NVLink per rank instead of (W-1) n).
// Two slots suffice: a rank republishes a slot only after every peer has
// published the next epoch, i.e. after every peer finished reading the slot.
// Every wait is bounded (5 s of %globaltimer) and reports through the device
// status word.
// ---------------------------------------------------------------------------
static constexpr size_t kP2PMaxElems = size_t(4) << 20;  // 8 MiB of bf16 per slot
static constexpr size_t kP2PRegion =
    4 * kP2PMaxElems * sizeof(uint16_t) + 2 * 64 * sizeof(uint32_t) + 256 +
    2 * kP2PMaxElems * sizeof(float);

struct Region {  // offsets inside one rank's region
  static __host__ __device__ uint16_t* staging(void* base, uint32_t slot) {
    return static_cast<uint16_t*>(base) + (size_t)slot * kP2PMaxElems;
  }
  static __host__ __device__ uint16_t* result(void* base, uint32_t slot) {
    return static_cast<uint16_t*>(base) + (size_t)(2 + slot) * kP2PMaxElems;
  }
  static __host__ __device__ uint32_t* flags(void* base) {
    return reinterpret_cast<uint32_t*>(static_cast<uint16_t*>(base) + 4 * kP2PMaxElems);
  }
  static __host__ __device__ uint32_t* flags2(void* base) { return flags(base) + 64; }
  // fp32 partials of the fused reduce + residual step, [2][kP2PMaxElems]
  static __host__ __device__ float* staging32(void* base, uint32_t slot) {
    uint8_t* p = reinterpret_cast<uint8_t*>(flags2(base) + 64);
    p = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 255) & ~uintptr_t(255));
    return reinterpret_cast<float*>(p) + (size_t)slot * kP2PMaxElems;
  }
};

struct P2P {
  bool ready = false;
  int rank = 0, world = 1;
  void* region = nullptr;     // local
  uint32_t* ctr = nullptr;    // local: [0] epoch, [1] publish arrivals, [2] push arrivals
  void* peer[8] = {};         // peer regions (peer[rank] = region)
};
static P2P g_p2p;

struct PeerPtrs {
  void* r[8];
};

__device__ __forceinline__ void store_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void store_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Threads 0..world-1 of the CTA wait for flags[r] >= e; then a CTA barrier.
__device__ __forceinline__ void wait_flags(const uint32_t* flags, uint32_t e, int world,
                                           uint32_t* status) {
  if (threadIdx.x < (unsigned)world) {
    const uint64_t t0 = mbd::globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
      if ((int32_t)(load_acquire_sys(flags + threadIdx.x) - e) >= 0) break;
      if ((it & 63u) == 0 && mbd::globaltimer_ns() - t0 > 5000000000ull) {
        atomicOr(status, MB_DEV_TIMEOUT_EPI);
        break;
      }
    }
  }
  __syncthreads();
}

__device__ __forceinline__ void acc8(float (&a)[8], uint4 w) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    a[2 * m] += __uint_as_float(ws[m] << 16);
    a[2 * m + 1] += __uint_as_float(ws[m] & 0xFFFF0000u);
  }
}
__device__ __forceinline__ uint4 pack8(const float (&a)[8]) {
  uint4 o;
  uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a[2 * m], a[2 * m + 1]);
    op[m] = *reinterpret_cast<uint32_t*>(&h);
  }
  return o;
}

// n is a multiple of 8 * world (checked by the host).
__global__ void p2p_publish_kernel(const uint16_t* __restrict__ src, size_t n, PeerPtrs peers,
                                   uint32_t* ctr, int rank, int world) {
  const uint32_t e = *reinterpret_cast<volatile uint32_t*>(&ctr[0]);
  uint16_t* dst = Region::staging(peers.r[rank], e & 1);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n / 8;
       i += (size_t)gridDim.x * blockDim.x)
    reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (atomicAdd(&ctr[1], 1u) + 1 == gridDim.x) {  // the last CTA of this rank
      __threadfence_system();
      for (int r = 0; r < world; ++r) store_release_sys(Region::flags(peers.r[r]) + rank, e + 1);
      ctr[1] = 0;
      ctr[0] = e + 1;
    }
  }
}

__global__ void p2p_oneshot_kernel(uint16_t* __restrict__ out, size_t n, PeerPtrs peers,
                                   const uint32_t* ctr, int rank, int world, uint32_t* status) {
  const uint32_t e = *reinterpret_cast<const volatile uint32_t*>(&ctr[0]);  // already bumped
  wait_flags(Region::flags(peers.r[rank]), e, world, status);
  const uint32_t slot = (e - 1) & 1;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n / 8;
       i += (size_t)gridDim.x * blockDim.x) {
    float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int r = 0; r < world; ++r)
      acc8(a, reinterpret_cast<const uint4*>(Region::staging(peers.r[r], slot))[i]);
    reinterpret_cast<uint4*>(out)[i] = pack8(a);
  }
}

__global__ void p2p_reduce_push_kernel(size_t n, PeerPtrs peers, uint32_t* ctr, int rank,
                                       int world, uint32_t* status) {
  const uint32_t e = *reinterpret_cast<const volatile uint32_t*>(&ctr[0]);
  wait_flags(Region::flags(peers.r[rank]), e, world, status);
  const uint32_t slot = (e - 1) & 1;
  const size_t chunk8 = n / 8 / world, c0 = (size_t)rank * chunk8;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < chunk8;
       i += (size_t)gridDim.x * blockDim.x) {
    float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int r = 0; r < world; ++r)
      acc8(a, reinterpret_cast<const uint4*>(Region::staging(peers.r[r], slot))[c0 + i]);
    const uint4 o = pack8(a);
    for (int r = 0; r < world; ++r)
      reinterpret_cast<uint4*>(Region::result(peers.r[r], slot))[c0 + i] = o;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (atomicAdd(&ctr[2], 1u) + 1 == gridDim.x) {
      __threadfence_system();
      for (int r = 0; r < world; ++r) store_release_sys(Region::flags2(peers.r[r]) + rank, e);
      ctr[2] = 0;
    }
  }
}

__global__ void p2p_collect_kernel(uint16_t* __restrict__ out, size_t n, PeerPtrs peers,
                                   const uint32_t* ctr, int rank, int world, uint32_t* status) {
  const uint32_t e = *reinterpret_cast<const volatile uint32_t*>(&ctr[0]);
  wait_flags(Region::flags2(peers.r[rank]), e, world, status);
  const uint4* res = reinterpret_cast<const uint4*>(Region::result(peers.r[rank], (e - 1) & 1));
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n / 8;
       i += (size_t)gridDim.x * blockDim.x)
    reinterpret_cast<uint4*>(out)[i] = res[i];
}

// Fused tensor-parallel reduce + residual (the decoder's o-proj and down-proj
// step), two phases over NVLink peer memory. Each rank's fp32 partial product
// [T, D] sits in its staging32 slot 0 (the decoder's epilogue writes it there
// directly). Rows are owned in contiguous blocks of ceil(T / W).
//   reduce   : CTA 0 signals flags[my rank] = e on every peer, every CTA
//              waits for all flags >= e, then sums the W partials of MY rows
//              in rank order (0..W-1, fp32), adds the fp32 (or bf16) residual
//              and stores the row into my staging32 slot 1 (the result area).
//              The last CTA signals flags2[my rank] = e on every peer.
//   gather   : one CTA per row waits for flags2[owner] >= e, reads the
//              owner's result row (local for my own rows), writes the fp32
//              stream, its bf16 copy and optionally rstd = rsqrt(mean(out^2) +
//              eps). The last CTA bumps the epoch.
// NVLink bytes per rank: (W-1)/W of the partial in, (W-1)/W of the result in,
// against (W-1) whole partials for a one-shot sum. Each row is summed by one
// rank and copied by the others, so every rank holds bitwise the same stream.
// One slot of each kind suffices: a rank rewrites its partial (next call)
// only after its gather saw every owner's flags2, i.e. after every peer read
// it; it rewrites its result rows only after every peer signalled the next
// call's reduce, i.e. after every peer's gather finished.
__global__ void p2p_rs_kernel(PeerPtrs peers, uint32_t* ctr, int rank, int world, int64_t T, int D,
                              const float* __restrict__ res32, const uint16_t* __restrict__ res16,
                              uint32_t* status) {
  // Launched with programmatic dependent launch: let the next kernels start
  // their set-up (the next GEMM also requests its first weight boxes), then
  // wait for the kernel that wrote the partial before touching anything.
  mbd::pdl_trigger();
  mbd::pdl_wait();
  const uint32_t e = *reinterpret_cast<volatile uint32_t*>(&ctr[0]) + 1;
  // The partial was written by an earlier kernel on this stream, so it is
  // complete in this GPU's memory (which serves the peers' reads) before this
  // grid starts: a relaxed store is enough to announce it. CTA 0 signals for
  // the grid; nothing that runs before it on this GPU waits on this grid, so
  // it always gets an SM even if its siblings are spinning already.
  if (blockIdx.x == 0 && threadIdx.x < (unsigned)world)
    store_relaxed_sys(Region::flags(peers.r[threadIdx.x]) + rank, e);
  wait_flags(Region::flags(peers.r[rank]), e, world, status);
  const int64_t per = (T + world - 1) / world;
  const int64_t r0 = (int64_t)rank * per;
  const int64_t r1 = r0 + per < T ? r0 + per : T;
  const int64_t base = r0 * D / 4, n4 = r1 > r0 ? (r1 - r0) * D / 4 : 0;
  float4* out = reinterpret_cast<float4*>(Region::staging32(peers.r[rank], 1));
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = base + i;
    float4 t[8];
#pragma unroll
    for (int r = 0; r < 8; ++r)
      if (r < world) t[r] = reinterpret_cast<const float4*>(Region::staging32(peers.r[r], 0))[j];
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < 8; ++r)
      if (r < world) {
        a.x += t[r].x;
        a.y += t[r].y;
        a.z += t[r].z;
        a.w += t[r].w;
      }
    if (res32) {
      const float4 u = reinterpret_cast<const float4*>(res32)[j];
      a.x += u.x;
      a.y += u.y;
      a.z += u.z;
      a.w += u.w;
    } else {
      const uint2 u = reinterpret_cast<const uint2*>(res16)[j];
      a.x += __uint_as_float(u.x << 16);
      a.y += __uint_as_float(u.x & 0xFFFF0000u);
      a.z += __uint_as_float(u.y << 16);
      a.w += __uint_as_float(u.y & 0xFFFF0000u);
    }
    out[j] = a;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // GPU-scope fence per CTA; the last CTA's system-scope release is
    // cumulative over the writes it observed through the arrival counter.
    __threadfence();
    if (atomicAdd(&ctr[1], 1u) + 1 == gridDim.x) {  // the last CTA of this rank
      __threadfence_system();
      for (int r = 0; r < world; ++r) store_release_sys(Region::flags2(peers.r[r]) + rank, e);
      ctr[1] = 0;
    }
  }
}

__global__ void p2p_ag_kernel(PeerPtrs peers, uint32_t* ctr, int rank, int world, int64_t T, int D,
                              float* __restrict__ out32, uint16_t* __restrict__ out16,
                              float* __restrict__ rstd_out, float eps, uint32_t* status) {
  mbd::pdl_trigger();
  mbd::pdl_wait();
  const uint32_t e = *reinterpret_cast<volatile uint32_t*>(&ctr[0]) + 1;
  const int64_t row = blockIdx.x;
  const int64_t per = (T + world - 1) / world;
  const int owner = (int)(row / per);
  if (threadIdx.x == 0) {
    const uint32_t* f = Region::flags2(peers.r[rank]) + owner;
    const uint64_t t0 = mbd::globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
      if ((int32_t)(load_acquire_sys(f) - e) >= 0) break;
      if ((it & 63u) == 0 && mbd::globaltimer_ns() - t0 > 5000000000ull) {
        atomicOr(status, MB_DEV_TIMEOUT_EPI);
        break;
      }
    }
  }
  __syncthreads();
  const float* src = Region::staging32(peers.r[owner], 1);
  float ss = 0.f;
  for (int c = threadIdx.x * 4; c < D; c += blockDim.x * 4) {
    const int64_t off = row * D + c;
    const float4 a = *reinterpret_cast<const float4*>(src + off);
    if (out32) *reinterpret_cast<float4*>(out32 + off) = a;
    __nv_bfloat162 h0 = __floats2bfloat162_rn(a.x, a.y), h1 = __floats2bfloat162_rn(a.z, a.w);
    *reinterpret_cast<uint2*>(out16 + off) =
        make_uint2(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1));
    ss += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
  }
  if (rstd_out) {
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
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
  if (threadIdx.x == 0 && atomicAdd(&ctr[2], 1u) + 1 == gridDim.x) {  // the last CTA
    ctr[2] = 0;
    ctr[0] = e;
  }
}

#ifdef MB_HAVE_NCCL
static int p2p_setup(int rank, int world) {
  if (world > 8) {
    set_error("peer all-reduce supports up to 8 ranks");
    return MB_ERR_BAD_ARG;
  }
  P2P& p = g_p2p;
  p.rank = rank;
  p.world = world;
  MB_CUDA(cudaMalloc(&p.region, kP2PRegion));
  MB_CUDA(cudaMemset(p.region, 0, kP2PRegion));
  MB_CUDA(cudaMalloc(&p.ctr, 4 * sizeof(uint32_t)));
  MB_CUDA(cudaMemset(p.ctr, 0, 4 * sizeof(uint32_t)));
  cudaIpcMemHandle_t mine;
  MB_CUDA(cudaIpcGetMemHandle(&mine, p.region));
  void* dmine = nullptr;
  void* dall = nullptr;
  MB_CUDA(cudaMalloc(&dmine, sizeof(mine)));
  MB_CUDA(cudaMalloc(&dall, sizeof(mine) * world));
  MB_CUDA(cudaMemcpy(dmine, &mine, sizeof(mine), cudaMemcpyHostToDevice));
  ncclResult_t r = ncclAllGather(dmine, dall, sizeof(mine), ncclUint8, g_comm, 0);
  if (r == ncclInProgress) {
    int rc = wait_ready(60000, "IPC handle all-gather");
    if (rc) return rc;
  } else if (r != ncclSuccess) {
    return nccl_fail(r, "ncclAllGather(ipc handles)");
  }
  MB_CUDA(cudaDeviceSynchronize());
  std::vector<cudaIpcMemHandle_t> all(world);
  MB_CUDA(cudaMemcpy(all.data(), dall, sizeof(mine) * world, cudaMemcpyDeviceToHost));
  cudaFree(dmine);
  cudaFree(dall);
  for (int q = 0; q < world; ++q) {
    if (q == rank) {
      p.peer[q] = p.region;
      continue;
    }
    MB_CUDA(cudaIpcOpenMemHandle(&p.peer[q], all[q], cudaIpcMemLazyEnablePeerAccess));
  }
  p.ready = true;
  return MB_OK;
}
#endif

static void p2p_teardown() {
  P2P& p = g_p2p;
  if (!p.ready) return;
  for (int q = 0; q < p.world; ++q)
    if (q != p.rank && p.peer[q]) cudaIpcCloseMemHandle(p.peer[q]);
  cudaFree(p.region);
  cudaFree(p.ctr);
  p = P2P();
}

// bf16 all-reduce (used when the fused fp32 peer reduction does not apply,
// e.g. prefill messages larger than a slot). NCCL by default; MB_TP_P2P=
// 1shot|2shot selects the bf16 peer kernels for messages that fit a slot.
int tp_allreduce_sum(void* buf, size_t count, cudaStream_t stream) {
  static const char* mode = getenv("MB_TP_P2P");
  static const bool use_p2p = mode && (!strcmp(mode, "1shot") || !strcmp(mode, "2shot"));
  static const bool force_nccl = !use_p2p || getenv("MB_TP_NCCL") != nullptr;
  static const bool oneshot = use_p2p && !strcmp(mode, "1shot");
  if (!g_p2p.ready || force_nccl || count > kP2PMaxElems || count % (8 * g_p2p.world) != 0 ||
      reinterpret_cast<uintptr_t>(buf) % 16 != 0)
    return tp_allreduce_bf16(buf, count, stream);
  PeerPtrs pp;
  for (int q = 0; q < 8; ++q) pp.r[q] = g_p2p.peer[q];
  const int W = g_p2p.world, R = g_p2p.rank;
  auto grid = [](size_t vec) {
    int b = (int)((vec + 255) / 256);
    const int cap = 2 * num_sms();
    return b < 1 ? 1 : (b > cap ? cap : b);
  };
  uint16_t* x = static_cast<uint16_t*>(buf);
  p2p_publish_kernel<<<grid(count / 8), 256, 0, stream>>>(x, count, pp, g_p2p.ctr, R, W);
  MB_CUDA(cudaGetLastError());
  if (oneshot) {
    p2p_oneshot_kernel<<<grid(count / 8), 256, 0, stream>>>(x, count, pp, g_p2p.ctr, R, W,
                                                            device_status_ptr());
  } else {
    p2p_reduce_push_kernel<<<grid(count / 8 / W), 256, 0, stream>>>(count, pp, g_p2p.ctr, R, W,
                                                                     device_status_ptr());
    MB_CUDA(cudaGetLastError());
    p2p_collect_kernel<<<grid(count / 8), 256, 0, stream>>>(x, count, pp, g_p2p.ctr, R, W,
                                                            device_status_ptr());
  }
  MB_CUDA(cudaGetLastError());
  return MB_OK;
}

bool tp_fused_ready(size_t T, int D) {
  static const bool off = getenv("MB_TP_NCCL") != nullptr;
  return g_p2p.ready && !off && (size_t)T * D <= kP2PMaxElems && D % 4 == 0;
}

float* tp_partial_slot() {
  return g_p2p.ready ? Region::staging32(g_p2p.region, 0) : nullptr;
}

int tp_reduce_residual(const float* part32, int64_t T, int D, const float* res32,
                       const uint16_t* res16, float* out32, uint16_t* out16, float* rstd_out,
                       float eps, cudaStream_t stream) {
  MB_REQUIRE(tp_fused_ready((size_t)T, D), "fused TP reduce: peers not mapped or size too large");
  MB_REQUIRE(res32 || res16, "fused TP reduce: no residual");
  MB_REQUIRE(T > 0, "fused TP reduce: no rows");
  PeerPtrs pp;
  for (int q = 0; q < 8; ++q) pp.r[q] = g_p2p.peer[q];
  const size_t n = (size_t)T * D;
  float* slot = tp_partial_slot();
  if (part32 != slot)
    MB_CUDA(cudaMemcpyAsync(slot, part32, n * sizeof(float), cudaMemcpyDeviceToDevice, stream));
  const int W = g_p2p.world;
  const int64_t per = (T + W - 1) / W;
  int rs = (int)((per * D / 4 + 255) / 256);
  if (rs > num_sms()) rs = num_sms();
  if (rs < 1) rs = 1;
  MB_CUDA(launch_pdl(p2p_rs_kernel, dim3(rs), dim3(256), 0, stream, pp, g_p2p.ctr, g_p2p.rank, W,
                     T, D, res32, res16, device_status_ptr()));
  MB_CUDA(cudaGetLastError());
  int threads = D / 4 < 1024 ? ((D / 4 + 31) / 32) * 32 : 1024;
  if (threads < 32) threads = 32;
  MB_CUDA(launch_pdl(p2p_ag_kernel, dim3((unsigned)T), dim3(threads), 0, stream, pp, g_p2p.ctr,
                     g_p2p.rank, W, T, D, out32, out16, rstd_out, eps, device_status_ptr()));
  MB_CUDA(cudaGetLastError());
  return MB_OK;
}

int tp_world() {
#ifdef MB_HAVE_NCCL
  return g_world;
#else
  return 1;
#endif
}

}  // namespace mb

extern "C" int mb_tp_allreduce_bf16(uint16_t* buf, size_t count, void* stream) {
  return mb::tp_allreduce_bf16(buf, count, static_cast<cudaStream_t>(stream));
}
