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
  return MB_OK;
#else
  (void)rank; (void)world; (void)nccl_id_path; (void)timeout_ms;
  set_error("mb_init: built without NCCL");
  return MB_ERR_NCCL;
#endif
}

void tp_shutdown() {
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
