// Tensor-parallel communicator set-up (filled in with the TP decoder).
#include "common.cuh"
#include "kernels.h"

namespace mb {
int tp_init(int rank, int world, const char* nccl_id_path, int timeout_ms) {
  (void)rank; (void)world; (void)nccl_id_path; (void)timeout_ms;
  set_error("mb_init: world > 1 needs the tensor-parallel build");
  return MB_ERR_NCCL;
}
void tp_shutdown() {}
}  // namespace mb
