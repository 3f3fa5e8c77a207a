// libmb200 lifecycle, error plumbing, device info, tensor-map helpers and the
// manifest-style mb_run dispatcher.
//
// mb_run replaces the reference's Metal host binary: main.mm:129-159 binds
// buffers by index (inputs uploaded, outputs allocated, scalars by value),
// timing.mm:125-193 dispatches warmup+iters times with one GPU timestamp pair
// per dispatch, sorts the times and reports min/median/mean, and
// main.mm:167-171 writes the outputs back. Here the bindings come in as
// mb_buf/mb_scalar arrays, each dispatch is bracketed by CUDA events on the
// launch stream, and outputs are copied back into the caller's host buffers.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <unistd.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <cstdlib>
#include <functional>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace mb {

static thread_local std::string g_last_error;
static int g_device = -1;

// One device status word per GPU (bounded waits write into it), allocated on
// first use with that device current, so a kernel is never handed another
// GPU's word.
constexpr int kMaxDevices = 64;
static uint32_t* g_status[kMaxDevices] = {};
static std::mutex g_status_mu;

static int current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  return dev;
}

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

int cuda_fail(cudaError_t e, const char* what, const char* file, int line) {
  set_error("CUDA error %s (%d) in %s at %s:%d", cudaGetErrorString(e), (int)e, what, file, line);
  return MB_ERR_CUDA;
}

uint32_t* device_status_ptr() {
  const int dev = current_device();
  if (dev < 0) return nullptr;
  std::lock_guard<std::mutex> lk(g_status_mu);
  if (!g_status[dev]) {
    uint32_t* p = nullptr;
    if (cudaMalloc(&p, sizeof(uint32_t)) != cudaSuccess) return nullptr;
    cudaMemset(p, 0, sizeof(uint32_t));
    g_status[dev] = p;
  }
  return g_status[dev];
}

uint32_t* existing_device_status_ptr() {
  const int dev = current_device();
  if (dev < 0) return nullptr;
  std::lock_guard<std::mutex> lk(g_status_mu);
  return g_status[dev];
}

int check_device_status(cudaStream_t stream) {
  uint32_t* st = existing_device_status_ptr();
  if (!st) return MB_OK;
  uint32_t v = 0;
  MB_CUDA(cudaMemcpyAsync(&v, st, sizeof(v), cudaMemcpyDeviceToHost, stream));
  MB_CUDA(cudaStreamSynchronize(stream));
  if (v) {
    set_error("a bounded device wait timed out (status 0x%x)", v);
    return MB_ERR_TIMEOUT;
  }
  return MB_OK;
}

int num_sms() {
  static int n[kMaxDevices] = {};
  const int dev = current_device();
  if (dev < 0) return 148;
  if (!n[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n[dev] = v;  // an int store: racing threads write the same value
  }
  return n[dev];
}

int ensure_smem_attr(const void* fn, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  const int dev = current_device();
  std::lock_guard<std::mutex> lk(mu);
  if (done.count({fn, dev})) return MB_OK;
  MB_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.insert({fn, dev});
  return MB_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

int make_tmap_nd(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int rank,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled unavailable from the driver");
    return MB_ERR_CUDA;
  }
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, dt, (cuuint32_t)rank, const_cast<void*>(base),
                  reinterpret_cast<const cuuint64_t*>(dims),
                  reinterpret_cast<const cuuint64_t*>(strides_bytes),
                  reinterpret_cast<const cuuint32_t*>(box), estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d): rank %d dims[0]=%llu box[0]=%u", (int)r, rank,
              (unsigned long long)dims[0], box[0]);
    return MB_ERR_CUDA;
  }
  return MB_OK;
}

bool pdl_enabled() {
  static const bool on = getenv("MB_NO_PDL") == nullptr;
  return on;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes,
                 uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                 uint32_t box_outer, CUtensorMapSwizzle swz) {
  (void)elem_bytes;
  uint64_t dims[2] = {inner, outer};
  uint64_t strides[1] = {row_stride_bytes};
  uint32_t box[2] = {box_inner, box_outer};
  return make_tmap_nd(map, base, dt, 2, dims, strides, box, swz);
}

// ---------------------------------------------------------------------------
// tiny flat-JSON reader for mb_run's config (keys -> number / bool / string)
// ---------------------------------------------------------------------------
Config parse_config(const char* js) {
  Config c;
  if (!js) return c;
  const char* p = js;
  while (*p) {
    const char* q = strchr(p, '"');
    if (!q) break;
    const char* e = strchr(q + 1, '"');
    if (!e) break;
    std::string key(q + 1, e);
    p = e + 1;
    while (*p == ' ' || *p == ':' || *p == '\t' || *p == '\n') ++p;
    std::string val;
    if (*p == '"') {
      const char* e2 = strchr(p + 1, '"');
      if (!e2) break;
      val.assign(p + 1, e2);
      p = e2 + 1;
    } else {
      const char* s = p;
      while (*p && *p != ',' && *p != '}') ++p;
      val.assign(s, p);
      while (!val.empty() && (val.back() == ' ' || val.back() == '\n')) val.pop_back();
    }
    c.kv[key] = val;
  }
  return c;
}

double Config::num(const char* k, double dflt) const {
  auto it = kv.find(k);
  if (it == kv.end()) return dflt;
  if (it->second == "true") return 1;
  if (it->second == "false") return 0;
  return atof(it->second.c_str());
}

std::string Config::str(const char* k, const char* dflt) const {
  auto it = kv.find(k);
  return it == kv.end() ? std::string(dflt) : it->second;
}

const RunArgs::Buf* RunArgs::buf(int binding) const {
  for (auto& b : bufs)
    if (b.binding == binding) return &b;
  return nullptr;
}

bool RunArgs::scalar(int binding, double* out) const {
  for (auto& s : scalars)
    if (s.binding == binding) {
      *out = s.dtype == MB_F32 ? (double)s.v.f : s.dtype == MB_I32 ? (double)s.v.i : (double)s.v.u;
      return true;
    }
  return false;
}

static std::vector<KernelEntry>& table() {
  static std::vector<KernelEntry> t;
  return t;
}

void register_kernel(const KernelEntry& e) { table().push_back(e); }

static const KernelEntry* find_kernel(const char* name) {
  register_all_kernels();
  for (auto& e : table())
    if (e.name == name) return &e;
  return nullptr;
}

}  // namespace mb

using namespace mb;

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" const char* mb_last_error(void) { return g_last_error.c_str(); }

extern "C" int mb_init(int device, int rank, int world, const char* nccl_id_path, int timeout_ms) {
  int n = 0;
  MB_CUDA(cudaGetDeviceCount(&n));
  MB_REQUIRE(device >= 0 && device < n, "mb_init: device %d out of range (%d visible)", device, n);
  MB_CUDA(cudaSetDevice(device));
  MB_CUDA(cudaFree(nullptr));  // create the context now
  g_device = device;
  if (!device_status_ptr()) {
    set_error("mb_init: cannot allocate the device status word");
    return MB_ERR_CUDA;
  }
  if (world > 1) return tp_init(rank, world, nccl_id_path, timeout_ms);
  return MB_OK;
}

extern "C" void mb_shutdown(void) {
  tp_shutdown();
  {
    std::lock_guard<std::mutex> lk(g_status_mu);
    int cur = -1;
    cudaGetDevice(&cur);
    for (int d = 0; d < kMaxDevices; ++d) {
      if (!g_status[d]) continue;
      cudaSetDevice(d);
      cudaFree(g_status[d]);
      g_status[d] = nullptr;
    }
    if (cur >= 0) cudaSetDevice(cur);
  }
  g_device = -1;
}

extern "C" int mb_device_info(mb_device* out) {
  MB_REQUIRE(out != nullptr, "mb_device_info: null output");
  memset(out, 0, sizeof(*out));
  int dev = 0;
  MB_CUDA(cudaGetDevice(&dev));
  cudaDeviceProp p;
  MB_CUDA(cudaGetDeviceProperties(&p, dev));
  snprintf(out->name, sizeof(out->name), "%s", p.name);
  out->sm_count = p.multiProcessorCount;
  out->cc_major = p.major;
  out->cc_minor = p.minor;
  out->hbm_bytes = p.totalGlobalMem;
  out->l2_bytes = p.l2CacheSize;
  out->smem_per_block_optin = (int)p.sharedMemPerBlockOptin;
  out->cpu_cores = (int)sysconf(_SC_NPROCESSORS_ONLN);
  out->ram_bytes = (uint64_t)sysconf(_SC_PHYS_PAGES) * (uint64_t)sysconf(_SC_PAGE_SIZE);
  if (p.major == 10 && p.minor == 0 && strstr(p.name, "B200"))
    snprintf(out->type, sizeof(out->type), "b200");
  else
    snprintf(out->type, sizeof(out->type), "sm%d%d", p.major, p.minor);
  // The results bucket is forced to "b200" on B200 so that every B200 SKU
  // string lands in results/b200/.
  snprintf(out->bucket, sizeof(out->bucket), "%s", out->type);
  return MB_OK;
}

extern "C" const char* mb_kernel_names(void) {
  static std::string names;
  register_all_kernels();
  if (names.empty()) {
    for (auto& e : table()) {
      if (!names.empty()) names += ",";
      names += e.name;
    }
  }
  return names.c_str();
}

extern "C" int mb_device_status(uint32_t* out) {
  MB_REQUIRE(out != nullptr, "mb_device_status: null output");
  *out = 0;
  uint32_t* st = existing_device_status_ptr();
  uint32_t v = 0;
  if (st) {
    MB_CUDA(cudaDeviceSynchronize());
    MB_CUDA(cudaMemcpy(&v, st, sizeof(uint32_t), cudaMemcpyDeviceToHost));
  }
  uint32_t w = 0;
  const int rc = noalloc_status(&w, false);
  if (rc) return rc;
  *out = v | w;
  return MB_OK;
}

extern "C" int mb_clear_device_status(void) {
  uint32_t* st = existing_device_status_ptr();
  if (st) MB_CUDA(cudaMemset(st, 0, sizeof(uint32_t)));
  uint32_t w = 0;
  return noalloc_status(&w, true);
}

namespace {
struct DevAlloc {
  std::vector<void*> ptrs;
  ~DevAlloc() {
    for (void* p : ptrs) cudaFree(p);
  }
};
// Every event mb_run creates, destroyed on every return path.
struct EventPool {
  std::vector<cudaEvent_t> evs;
  cudaError_t make(cudaEvent_t* e) {
    const cudaError_t r = cudaEventCreate(e);
    if (r == cudaSuccess) evs.push_back(*e);
    return r;
  }
  ~EventPool() {
    for (cudaEvent_t e : evs) cudaEventDestroy(e);
  }
};
}  // namespace

extern "C" int mb_run(const char* kernel, const mb_buf* bufs, int nbufs, const mb_scalar* scalars,
                      int nsc, const char* config_json, int warmup, int iters, mb_timing* out) {
  if (g_device < 0) {
    set_error("mb_run: call mb_init first");
    return MB_ERR_NOT_INIT;
  }
  MB_REQUIRE(kernel != nullptr, "mb_run: null kernel name");
  MB_REQUIRE(nbufs >= 0 && nsc >= 0 && warmup >= 0 && iters >= 1, "mb_run: bad counts");
  const KernelEntry* ke = find_kernel(kernel);
  if (!ke) {
    set_error("mb_run: unknown kernel '%s' (known: %s)", kernel, mb_kernel_names());
    return MB_ERR_UNKNOWN_KERNEL;
  }
  RunArgs a;
  a.config = parse_config(config_json);
  for (int i = 0; i < nsc; ++i) a.scalars.push_back(scalars[i]);

  cudaStream_t stream;
  MB_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
  struct StreamGuard {
    cudaStream_t s;
    ~StreamGuard() { cudaStreamDestroy(s); }
  } sg{stream};
  DevAlloc alloc;
  EventPool evp;
  cudaEvent_t h0, h1;
  MB_CUDA(evp.make(&h0));
  MB_CUDA(evp.make(&h1));

  // Bind buffers: host inputs are uploaded, host outputs get device storage.
  MB_CUDA(cudaEventRecord(h0, stream));
  for (int i = 0; i < nbufs; ++i) {
    const mb_buf& b = bufs[i];
    MB_REQUIRE(b.role == MB_ROLE_INPUT || b.role == MB_ROLE_OUTPUT,
               "mb_run: buffer %d has unknown role %d", b.binding, b.role);
    RunArgs::Buf rb{b.binding, b.role, b.dtype, b.bytes, b.ptr, b.ptr};
    if (!(b.flags & MB_DEVICE_PTR) && b.bytes > 0) {
      void* d = nullptr;
      MB_CUDA(cudaMalloc(&d, b.bytes));
      alloc.ptrs.push_back(d);
      if (b.role == MB_ROLE_INPUT) {
        MB_REQUIRE(b.ptr != nullptr, "mb_run: input binding %d has a null pointer", b.binding);
        MB_CUDA(cudaMemcpyAsync(d, b.ptr, b.bytes, cudaMemcpyHostToDevice, stream));
      }
      rb.dev = d;
    }
    a.bufs.push_back(rb);
  }
  MB_CUDA(cudaEventRecord(h1, stream));
  MB_CUDA(cudaEventSynchronize(h1));
  float h2d = 0;
  MB_CUDA(cudaEventElapsedTime(&h2d, h0, h1));

  KernelState st;
  int rc = ke->prepare(a, st, stream);
  if (rc) return rc;
  MB_REQUIRE(bool(st.launch), "mb_run: kernel '%s' prepared no launch", kernel);

  // Optional L2 flush between timed launches (a write larger than L2).
  void* flush = nullptr;
  size_t flush_bytes = 0;
  if (a.config.num("flush_l2", 0) != 0) {
    int l2 = 0;
    cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, g_device);
    flush_bytes = (size_t)l2 * 2;
    MB_CUDA(cudaMalloc(&flush, flush_bytes));
    alloc.ptrs.push_back(flush);
  }

  for (int i = 0; i < warmup; ++i) {
    rc = st.launch(stream);
    if (rc) return rc;
  }
  MB_CUDA(cudaStreamSynchronize(stream));
  rc = check_device_status(stream);
  if (rc) return rc;

  std::vector<cudaEvent_t> ev(2 * (size_t)iters);
  for (auto& e : ev) MB_CUDA(evp.make(&e));
  const std::string timed_range = std::string("mb_timed:") + kernel;
  for (int i = 0; i < iters; ++i) {
    if (flush) MB_CUDA(cudaMemsetAsync(flush, i & 0xff, flush_bytes, stream));
    nvtxRangePushA(timed_range.c_str());
    MB_CUDA(cudaEventRecord(ev[2 * i], stream));
    rc = st.launch(stream);
    if (rc) {
      nvtxRangePop();
      return rc;
    }
    MB_CUDA(cudaEventRecord(ev[2 * i + 1], stream));
    nvtxRangePop();
  }
  MB_CUDA(cudaStreamSynchronize(stream));
  rc = check_device_status(stream);
  if (rc) return rc;
  std::vector<double> times(iters);
  for (int i = 0; i < iters; ++i) {
    float ms = 0;
    MB_CUDA(cudaEventElapsedTime(&ms, ev[2 * i], ev[2 * i + 1]));
    times[i] = ms;
  }
  // --profile: one more dispatch inside its own NVTX range (timing.mm:163-190
  // samples counters on one extra dispatch; here an outside profiler such as
  // ncu picks the range), timed with events; it does not touch the numbers above.
  double profile_ms = -1.0;
  if (a.config.num("profile", 0) != 0) {
    cudaEvent_t p0, p1;
    MB_CUDA(evp.make(&p0));
    MB_CUDA(evp.make(&p1));
    const std::string range = std::string("mb_profile:") + kernel;
    nvtxRangePushA(range.c_str());
    MB_CUDA(cudaEventRecord(p0, stream));
    rc = st.launch(stream);
    if (!rc) {
      const cudaError_t e = cudaEventRecord(p1, stream);
      if (e != cudaSuccess) rc = mb::cuda_fail(e, "cudaEventRecord", __FILE__, __LINE__);
    }
    if (!rc) {
      const cudaError_t e = cudaStreamSynchronize(stream);
      if (e != cudaSuccess) rc = mb::cuda_fail(e, "cudaStreamSynchronize", __FILE__, __LINE__);
    }
    nvtxRangePop();
    if (rc) return rc;
    rc = check_device_status(stream);
    if (rc) return rc;
    float pm = 0;
    MB_CUDA(cudaEventElapsedTime(&pm, p0, p1));
    profile_ms = pm;
  }
  if (st.finish) {
    rc = st.finish(stream);
    if (rc) return rc;
  }

  // Outputs back to the caller's host buffers.
  MB_CUDA(cudaEventRecord(h0, stream));
  for (auto& b : a.bufs) {
    if (b.role == MB_ROLE_OUTPUT && b.dev != b.host && b.bytes > 0)
      MB_CUDA(cudaMemcpyAsync(b.host, b.dev, b.bytes, cudaMemcpyDeviceToHost, stream));
  }
  MB_CUDA(cudaEventRecord(h1, stream));
  MB_CUDA(cudaEventSynchronize(h1));
  float d2h = 0;
  MB_CUDA(cudaEventElapsedTime(&d2h, h0, h1));

  std::sort(times.begin(), times.end());
  double sum = 0;
  for (double t : times) sum += t;
  if (out) {
    out->min_ms = times.front();
    out->median_ms = times[times.size() / 2];
    out->mean_ms = sum / times.size();
    out->iters = iters;
    out->smem_bytes = st.smem_bytes;
    out->threads_per_cta = st.threads_per_cta;
    out->launches_per_iter = st.launches_per_iter;
    out->h2d_ms = h2d;
    out->d2h_ms = d2h;
    out->profile_ms = profile_ms;
  }
  return MB_OK;
}
