// Shared helpers for the sm_100a kernels of libmb200: error plumbing, bounded
// mbarrier waits, TMA and tcgen05 PTX wrappers.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string>

#include "../../include/mb200.h"

// ---------------------------------------------------------------------------
// host-side error plumbing (thread-local message behind mb_last_error)
// ---------------------------------------------------------------------------
namespace mb {
void set_error(const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what, const char* file, int line);
// Device-side status word: kernels that give up a bounded wait write a code
// here; the host reads it after the launch (mb_check_device_status).
uint32_t* device_status_ptr();
// The current device's status word if it was allocated already, else null
// (never allocates).
uint32_t* existing_device_status_ptr();
int check_device_status(cudaStream_t stream);
// The status word mb_sqr_mm_f32_noalloc uses on the current device before
// that device has a shared one: read into *out (0 if never set up), cleared
// when `clear` is set. Allocates nothing.
int noalloc_status(uint32_t* out, bool clear);
// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes,
                 uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                 uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz);
int make_tmap_nd(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int rank,
                 const uint64_t* dims, const uint64_t* strides_bytes /*rank-1*/,
                 const uint32_t* box, CUtensorMapSwizzle swz);
int num_sms();
// Opt `fn` into `bytes` of dynamic shared memory on the current device, once
// per (function, device); safe to call from several host threads.
int ensure_smem_attr(const void* fn, int bytes);
}  // namespace mb

namespace mb {
bool pdl_enabled();  // false when MB_NO_PDL is set
// <<<grid, block, smem, stream>>> with programmatic stream serialisation, so
// the kernel's prologue overlaps the tail of the previous kernel (see
// pdl_wait); the kernel must call mbd::pdl_wait() before reading its inputs.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
}  // namespace mb

#define MB_CUDA(call)                                                      \
  do {                                                                     \
    cudaError_t _e = (call);                                               \
    if (_e != cudaSuccess) return mb::cuda_fail(_e, #call, __FILE__, __LINE__); \
  } while (0)

#define MB_REQUIRE(cond, ...)                                              \
  do {                                                                     \
    if (!(cond)) { mb::set_error(__VA_ARGS__); return MB_ERR_BAD_ARG; }    \
  } while (0)

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
// Status codes a kernel writes into the device status word.
#define MB_DEV_TIMEOUT_TMA 0x1u
#define MB_DEV_TIMEOUT_MMA 0x2u
#define MB_DEV_TIMEOUT_EPI 0x4u
#define MB_DEV_TIMEOUT_SELFTEST 0x100u

namespace mbd {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Programmatic dependent launch (PDL). A kernel launched with
// mb::launch_pdl may start while the previous kernel of the stream is still
// running: pdl_wait() blocks until that kernel has completed and its writes
// are visible, so it must come before the first read of anything the previous
// kernel wrote, and every CTA executes it (then the grid cannot complete
// before its predecessor, which keeps dependencies transitive). pdl_trigger()
// lets the next kernel start launching. Both are no-ops in a kernel launched
// without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded waits give up after MB_WAIT_NS of wall time on the SM's global
// timer (2 s; a correct pipeline waits microseconds), record a status code and
// let the caller fall through to teardown instead of hanging the GPU.
#define MB_WAIT_NS 2000000000ull

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: returns false (and records `code` in *status, and raises the
// CTA-wide *abort flag when given) if the phase never completes or another
// role of the CTA already gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status,
                                          uint32_t code, volatile int* abort_flag = nullptr,
                                          uint64_t limit_ns = MB_WAIT_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (abort_flag && *abort_flag) return false;
      if (globaltimer_ns() - t0 > limit_ns) break;
    }
  }
  if (status) atomicOr(status, code);
  if (abort_flag) *abort_flag = 1;
  return false;
}

// AND of `ok` over the `nthreads` threads that reach named barrier `id`; all of
// them get the same answer, so they can leave a loop together (no thread is
// left waiting at a later barrier for one that already left).
__device__ __forceinline__ bool vote_all(bool ok, int id, int nthreads) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)ok), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// 2-D tiled TMA load global -> shared, completion on an mbarrier.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2, int32_t c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}

// Contiguous bulk copy global -> shared (no tensor map), completion on an
// mbarrier. Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- tcgen05 -------------------------------------------------------------
// Warp-wide TMEM allocation; the base column address is written to *dst.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16/f16 in, f32 acc).
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same with kind::tf32 (fp32 storage, tf32 multiply, f32 acc).
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread
// have completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor (tcgen05 "version 1"), 128-byte swizzle.
//  start address >> 4 in bits [0,14), leading byte offset >> 4 in [16,30),
//  stride byte offset >> 4 in [32,46), version 1 at bit 46, layout type in
//  [61,64) (2 = SWIZZLE_128B). The base offset field stays 0: the swizzle is a
//  function of the shared-memory address bits, the same one TMA applies when
//  it writes a 1024-byte-aligned box, so an operand may start at any 128-byte
//  row of such a box (the conv2d producer starts taps at row r*TW + s).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes,
                                               uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor for kind::f16 / kind::tf32 with f32 accumulate.
//  c_format bits [4,6) = 1 (F32); a_format [7,10), b_format [10,13)
//  (0 F16, 1 BF16, 2 TF32); a_major bit 15, b_major bit 16 (0 = K-major,
//  1 = MN-major); N >> 3 in [17,23); M >> 4 in [24,29).
__host__ __device__ constexpr uint32_t make_idesc(uint32_t ab_format, uint32_t M, uint32_t N,
                                                  uint32_t a_mn_major, uint32_t b_mn_major) {
  return (1u << 4) | (ab_format << 7) | (ab_format << 10) | (a_mn_major << 15) |
         (b_mn_major << 16) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

}  // namespace mbd
