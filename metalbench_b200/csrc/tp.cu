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
  if (getenv("MB_TP_NO_P2P") == nullptr) {
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
// One-shot all-reduce over NVLink peer memory.
//
// Every rank owns, in its own HBM: staging[2][MAXE] bf16 (double buffer),
// flags[world] u32 (written by the peers) and two private counters. Peers'
// staging and flags are mapped with CUDA IPC at set-up (handles exchanged with
// one NCCL all-gather). A call is two kernels on the caller's stream:
//   publish: copy my partial into my staging slot (epoch % 2); the last CTA to
//            finish fences (system scope), stores epoch+1 into flags[my rank] of
//            every peer (release) and bumps my epoch;
//   gather:  wait (bounded) until every peer's flag in MY flags array reached
//            the epoch (acquire), then sum all ranks' staging slots over NVLink
//            into the output.
// The epoch lives on the device, so a CUDA graph of the step replays
// correctly. Two slots suffice: a rank can only republish a slot after every
// peer has published the following epoch, i.e. after every peer finished
// reading that slot.
// ---------------------------------------------------------------------------
static constexpr size_t kP2PMaxElems = size_t(4) << 20;  // 8 MiB of bf16 per slot
struct P2P {
  bool ready = false;
  int rank = 0, world = 1;
  uint16_t* staging = nullptr;  // local [2][MAXE]
  uint32_t* flags = nullptr;    // local [world]
  uint32_t* ctr = nullptr;      // local: [0] epoch, [1] CTAs done
  uint16_t* peer_staging[8] = {};
  uint32_t* peer_flags[8] = {};
};
static P2P g_p2p;

struct PeerPtrs {
  const uint16_t* staging[8];
  uint32_t* flags[8];
};

__global__ void p2p_publish_kernel(const uint16_t* __restrict__ src, size_t n, uint16_t* staging,
                                   PeerPtrs peers, uint32_t* ctr, int rank, int world) {
  const uint32_t e = *reinterpret_cast<volatile uint32_t*>(&ctr[0]);
  uint16_t* dst = staging + (size_t)(e & 1) * kP2PMaxElems;
  const size_t n8 = n / 8;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n8;
       i += (size_t)gridDim.x * blockDim.x)
    reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  for (size_t i = n8 * 8 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t done = atomicAdd(&ctr[1], 1u) + 1;
    if (done == gridDim.x) {  // last CTA: everything of this rank is written
      __threadfence_system();
      for (int r = 0; r < world; ++r)
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(peers.flags[r] + rank), "r"(e + 1)
                     : "memory");
      ctr[1] = 0;
      ctr[0] = e + 1;
    }
  }
}

__global__ void p2p_gather_kernel(uint16_t* __restrict__ out, size_t n, PeerPtrs peers,
                                  const uint32_t* flags, const uint32_t* ctr, int world,
                                  uint32_t* status) {
  __shared__ int ok;
  const uint32_t e = *reinterpret_cast<const volatile uint32_t*>(&ctr[0]);  // already bumped
  if (threadIdx.x < (unsigned)world) {
    const uint64_t t0 = mbd::globaltimer_ns();
    uint32_t v = 0;
    for (uint32_t it = 0;; ++it) {
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + threadIdx.x)
                   : "memory");
      if ((int32_t)(v - e) >= 0) break;
      if ((it & 63u) == 0 && mbd::globaltimer_ns() - t0 > 5000000000ull) {
        atomicOr(status, MB_DEV_TIMEOUT_EPI);
        break;
      }
    }
  }
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  const size_t slot = (size_t)((e - 1) & 1) * kP2PMaxElems;
  const size_t n8 = n / 8;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n8;
       i += (size_t)gridDim.x * blockDim.x) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int r = 0; r < world; ++r) {
      const uint4 w = reinterpret_cast<const uint4*>(peers.staging[r] + slot)[i];
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        acc[2 * m] += __uint_as_float(ws[m] << 16);
        acc[2 * m + 1] += __uint_as_float(ws[m] & 0xFFFF0000u);
      }
    }
    uint4 o;
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      __nv_bfloat162 h = __floats2bfloat162_rn(acc[2 * m], acc[2 * m + 1]);
      op[m] = *reinterpret_cast<uint32_t*>(&h);
    }
    reinterpret_cast<uint4*>(out)[i] = o;
  }
  for (size_t i = n8 * 8 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    float a = 0.f;
    for (int r = 0; r < world; ++r)
      a += __uint_as_float(((uint32_t)peers.staging[r][slot + i]) << 16);
    __nv_bfloat16 h = __float2bfloat16_rn(a);
    out[i] = *reinterpret_cast<uint16_t*>(&h);
  }
  (void)ok;
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
  MB_CUDA(cudaMalloc(&p.staging, 2 * kP2PMaxElems * sizeof(uint16_t)));
  MB_CUDA(cudaMalloc(&p.flags, 64 * sizeof(uint32_t)));
  MB_CUDA(cudaMalloc(&p.ctr, 2 * sizeof(uint32_t)));
  MB_CUDA(cudaMemset(p.flags, 0, 64 * sizeof(uint32_t)));
  MB_CUDA(cudaMemset(p.ctr, 0, 2 * sizeof(uint32_t)));
  cudaIpcMemHandle_t mine[2];
  MB_CUDA(cudaIpcGetMemHandle(&mine[0], p.staging));
  MB_CUDA(cudaIpcGetMemHandle(&mine[1], p.flags));
  void* dmine = nullptr;
  void* dall = nullptr;
  MB_CUDA(cudaMalloc(&dmine, sizeof(mine)));
  MB_CUDA(cudaMalloc(&dall, sizeof(mine) * world));
  MB_CUDA(cudaMemcpy(dmine, mine, sizeof(mine), cudaMemcpyHostToDevice));
  ncclResult_t r = ncclAllGather(dmine, dall, sizeof(mine), ncclUint8, g_comm, 0);
  if (r == ncclInProgress) {
    int rc = wait_ready(60000, "handle all-gather");
    if (rc) return rc;
  } else if (r != ncclSuccess) {
    return nccl_fail(r, "ncclAllGather(ipc handles)");
  }
  MB_CUDA(cudaDeviceSynchronize());
  std::vector<cudaIpcMemHandle_t> all(2 * world);
  MB_CUDA(cudaMemcpy(all.data(), dall, sizeof(mine) * world, cudaMemcpyDeviceToHost));
  cudaFree(dmine);
  cudaFree(dall);
  for (int q = 0; q < world; ++q) {
    if (q == rank) {
      p.peer_staging[q] = p.staging;
      p.peer_flags[q] = p.flags;
      continue;
    }
    void* a = nullptr;
    void* b = nullptr;
    MB_CUDA(cudaIpcOpenMemHandle(&a, all[2 * q], cudaIpcMemLazyEnablePeerAccess));
    MB_CUDA(cudaIpcOpenMemHandle(&b, all[2 * q + 1], cudaIpcMemLazyEnablePeerAccess));
    p.peer_staging[q] = static_cast<uint16_t*>(a);
    p.peer_flags[q] = static_cast<uint32_t*>(b);
  }
  p.ready = true;
  return MB_OK;
}
#endif

static void p2p_teardown() {
  P2P& p = g_p2p;
  if (!p.ready) return;
  for (int q = 0; q < p.world; ++q)
    if (q != p.rank) {
      if (p.peer_staging[q]) cudaIpcCloseMemHandle(p.peer_staging[q]);
      if (p.peer_flags[q]) cudaIpcCloseMemHandle(p.peer_flags[q]);
    }
  cudaFree(p.staging);
  cudaFree(p.flags);
  cudaFree(p.ctr);
  p = P2P();
}

// All-reduce used by the decoder: the peer kernels for messages that fit a
// staging slot (decode), NCCL otherwise or when MB_TP_NCCL=1.
int tp_allreduce_sum(void* buf, size_t count, cudaStream_t stream) {
  static const bool force_nccl = getenv("MB_TP_NCCL") != nullptr;
  if (!g_p2p.ready || force_nccl || count > kP2PMaxElems) return tp_allreduce_bf16(buf, count, stream);
  PeerPtrs pp;
  for (int q = 0; q < 8; ++q) {
    pp.staging[q] = g_p2p.peer_staging[q];
    pp.flags[q] = g_p2p.peer_flags[q];
  }
  const int sms = num_sms();
  const size_t n8 = (count + 7) / 8;
  int blocks = (int)((n8 + 255) / 256);
  if (blocks > 2 * sms) blocks = 2 * sms;
  if (blocks < 1) blocks = 1;
  p2p_publish_kernel<<<blocks, 256, 0, stream>>>(static_cast<const uint16_t*>(buf), count,
                                                  g_p2p.staging, pp, g_p2p.ctr, g_p2p.rank,
                                                  g_p2p.world);
  MB_CUDA(cudaGetLastError());
  p2p_gather_kernel<<<blocks, 256, 0, stream>>>(static_cast<uint16_t*>(buf), count, pp,
                                                 g_p2p.flags, g_p2p.ctr, g_p2p.world,
                                                 device_status_ptr());
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
