// Internal (non-ABI) registry of the kernels mb_run can dispatch by name.
#pragma once
#include <cuda_runtime.h>

#include <functional>
#include <map>
#include <string>
#include <vector>

#include "../../include/mb200.h"

namespace mb {

struct Config {
  std::map<std::string, std::string> kv;
  double num(const char* k, double dflt) const;
  std::string str(const char* k, const char* dflt) const;
};
Config parse_config(const char* js);

struct RunArgs {
  struct Buf {
    int binding, role, dtype;
    size_t bytes;
    void* host;  // caller pointer
    void* dev;   // device pointer bound to the kernel
  };
  std::vector<Buf> bufs;
  std::vector<mb_scalar> scalars;
  Config config;
  const Buf* buf(int binding) const;
  bool scalar(int binding, double* out) const;
};

// What prepare() leaves behind: the per-iteration launch, an optional
// post-timing step, scratch allocations (freed on destruction) and the launch
// shape reported in mb_timing.
struct KernelState {
  std::function<int(cudaStream_t)> launch;
  std::function<int(cudaStream_t)> finish;
  std::vector<void*> scratch;
  std::vector<std::function<void()>> cleanup;
  int smem_bytes = 0, threads_per_cta = 0, launches_per_iter = 1;
  ~KernelState() {
    for (auto& f : cleanup) f();
    for (void* p : scratch) cudaFree(p);
  }
};

struct KernelEntry {
  std::string name;
  std::function<int(const RunArgs&, KernelState&, cudaStream_t)> prepare;
};

void register_kernel(const KernelEntry& e);
void register_all_kernels();  // defined in registry.cu

// tensor parallel communicator (tp.cu)
int tp_init(int rank, int world, const char* nccl_id_path, int timeout_ms);
void tp_shutdown();
int tp_allreduce_bf16(void* buf, size_t count, cudaStream_t stream);
int tp_world();
int tp_allreduce_sum(void* buf, size_t count, cudaStream_t stream);
// Fused fp32 peer reduction + residual (tp.cu): out = residual + sum over
// ranks of part32 [T, D] (fp32, summed in rank order over NVLink), written as
// fp32 (out32, optional) and bf16 (out16), with optional per-row rstd.
// One set of peer slots per process: calls must be serialised on the GPU (one
// stream) and issued in the same order on every rank.
// tp_partial_slot() is this rank's peer-mapped partial buffer: a producer that
// writes its partial there directly saves the copy in tp_reduce_residual.
bool tp_fused_ready(size_t T, int D);
float* tp_partial_slot();
int tp_reduce_residual(const float* part32, int64_t T, int D, const float* res32,
                       const uint16_t* res16, float* out32, uint16_t* out16, float* rstd_out,
                       float eps, cudaStream_t stream);

// gemm.cu: bf16 GEMM C[M, N] (row stride ldc) = act(A @ B) (+ residual, row
// stride ld_res); b_layout 0: B [N, K], 1: B [K, N]; act 0 none, 1 exact GELU.
int gemm_bf16_ex(const uint16_t* A, const uint16_t* B, uint16_t* C, int64_t M, int64_t N,
                 int64_t K, int64_t ldc, int b_layout, const uint16_t* residual, int64_t ld_res,
                 int act, cudaStream_t s);
// gemm.cu: 3xTF32 pieces. tf32x3_split_rows splits n fp32 values (n % 4 == 0,
// 16-byte aligned) into tf32 hi and the exact fp32 remainder lo;
// tf32x3_core runs C[batch*M, N] (fp32, row stride N) = A @ B^T from K-major
// split operands A_hi/A_lo [batch*M, K], B_hi/B_lo [batch*N, K].
int tf32x3_split_rows(const float* src, float* hi, float* lo, int64_t n, cudaStream_t s);
int tf32x3_core(const float* a_hi, const float* a_lo, const float* b_hi, const float* b_lo,
                float* C, int64_t batch, int64_t M, int64_t N, int64_t K, uint32_t* status,
                cudaStream_t s);
// attention_tc.cu: tcgen05 prefill attention (same contract as
// mb_attention_prefill_bf16, Dh = 128); _ok() says whether TMA can address
// the operands.
bool attention_prefill_tc_ok(const uint16_t* q, int ldq, const uint16_t* k_cache,
                             const uint16_t* v_cache, uint16_t* out, int ldo);
// splits > 1 (non-causal): key range cut into `splits` parts per query tile,
// partials in part_o [B][Hq][S][splits][128] / part_ml [..][2] (fp32), then
// a combine kernel; attention_split_plan picks splits to fill the SMs.
int attention_prefill_tc(const uint16_t* q, int ldq, const uint16_t* k_cache,
                         const uint16_t* v_cache, const int* block_table, int max_pages,
                         const int* start_pos, const int* kv_len, int B, int S, int Hq, int Hkv,
                         int causal, uint16_t* out, int ldo, cudaStream_t stream, int splits = 1,
                         int max_kv_len = 0, float* part_o = nullptr, float* part_ml = nullptr);
int attention_split_plan(int64_t B, int64_t S, int64_t Hq, int64_t kv_len);
// decoder.cu helpers shared with fused_ops.cu
int rownorm(const uint16_t* x, int M, int D, float eps, float* rstd, cudaStream_t s);
int pack_tiled_weight(const uint16_t* in, int64_t ld_in, int K, const int* col_idx_dev, int Nout,
                      uint8_t* out, cudaStream_t s);

}  // namespace mb
