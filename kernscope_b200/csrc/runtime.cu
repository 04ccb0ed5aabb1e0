// runtime.cu -- the C ABI of the device runtime (the B200 replacement of
// libs/gpuruntime's GpuRuntime class, gpu.h:182-255): device queries, memory,
// copies, streams, events, the device error word and the bounded-wait
// self-test, plus host helpers shared by the kernel families (status mapping,
// arch check, TMA tensor-map encoding).
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <vector>

#include "ks_common.cuh"

// The device error word (every device holds its own copy of this variable);
// kernels receive its address in KsWait.
__device__ int g_ks_device_error = 0;
static std::atomic<unsigned long long> g_wait_limit_ns{4000000000ull};

namespace ks {

int map_cuda(cudaError_t e) {
  switch (e) {
    case cudaSuccess: return KS_OK;
    case cudaErrorNoDevice: return KS_ERR_NO_DEVICE;
    case cudaErrorInsufficientDriver: return KS_ERR_NO_DRIVER;
    case cudaErrorMemoryAllocation: return KS_ERR_MEMORY;
    case cudaErrorInvalidDevice: return KS_ERR_DEVICE_NOT_FOUND;
    case cudaErrorLaunchFailure:
    case cudaErrorLaunchOutOfResources:
    case cudaErrorInvalidConfiguration: return KS_ERR_LAUNCH;
    case cudaErrorInvalidValue: return KS_ERR_INVALID_ARGS;
    default: return KS_ERR_OTHER;
  }
}

int check_arch_sm100() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return map_cuda(e);
  int major = 0;
  e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e != cudaSuccess) return map_cuda(e);
  return major == 10 ? KS_OK : KS_ERR_ARCH;
}

// The driver context current on this thread (cuCtxGetCurrent, reached through
// the runtime's driver entry point so that the library needs no libcuda link);
// nullptr when the driver does not answer.
static void *current_context() {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
  });
  CUcontext c = nullptr;
  if (fn == nullptr || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

int symbol_address(const void *symbol, void **out) {
  // A __device__ variable's address belongs to the module as loaded in one
  // driver context, so the cache is keyed on (context, symbol): a second
  // context on the same device (cuCtxCreate) resolves its own address.
  struct Entry { void *ctx; const void *sym; void *addr; };
  static std::vector<Entry> cache;
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return map_cuda(e);
  void *ctx = current_context();
  if (ctx == nullptr) {
    // no context is current on this thread yet: cudaSetDevice makes the
    // device's primary context current (CUDA 12 initialises it there), the
    // one the launches will then use
    e = cudaSetDevice(dev);
    if (e != cudaSuccess) return map_cuda(e);
    ctx = current_context();
    if (ctx == nullptr) return KS_ERR_NO_DRIVER;
  }
  std::lock_guard<std::mutex> lk(mu);
  for (const Entry &x : cache)
    if (x.ctx == ctx && x.sym == symbol) {
      *out = x.addr;
      return KS_OK;
    }
  void *p = nullptr;
  e = cudaGetSymbolAddress(&p, symbol);
  if (e != cudaSuccess) return map_cuda(e);
  if (p == nullptr) return KS_ERR_OTHER;
  cache.push_back({ctx, symbol, p});
  *out = p;
  return KS_OK;
}

KsWait wait_ctx() {
  KsWait w{nullptr, g_wait_limit_ns.load()};
  void *p = nullptr;
  if (symbol_address(reinterpret_cast<const void *>(&g_ks_device_error), &p) == KS_OK) w.err = static_cast<int *>(p);
  return w;
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

void set_reason(char *buf, size_t len, const char *fmt, ...) {
  if (buf == nullptr || len == 0) return;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, len, fmt, ap);
  va_end(ap);
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int encode_tmap_2d(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t inner, uint64_t outer,
                   uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  auto fn = get_encode();
  if (fn == nullptr) return KS_ERR_NO_DRIVER;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? KS_OK : KS_ERR_INVALID_ARGS;
}

int encode_tmap_3d(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t d0, uint64_t d1, uint64_t d2,
                   uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1, uint32_t b2,
                   CUtensorMapSwizzle swz) {
  auto fn = get_encode();
  if (fn == nullptr) return KS_ERR_NO_DRIVER;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, dt, 3, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? KS_OK : KS_ERR_INVALID_ARGS;
}

}  // namespace ks

// ---------------------------------------------------------------------------
// Bounded-wait self-test kernel: waits on an mbarrier whose phase never
// completes (count 2, one arrival), gives up after the limit, returns.
// ---------------------------------------------------------------------------
__global__ void ks_selftest_wait_kernel(unsigned long long limit_ns, int *err) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    ks_mbar_init(&bar, 2);
    ks_fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    ks_mbar_arrive(&bar);  // one of two arrivals: the phase stays open
    const uint32_t a = ks_smem_u32(&bar);
    const uint64_t t0 = ks_globaltimer();
    bool done = false;
    while (!done) {
      for (int i = 0; i < 32 && !done; ++i) done = ks_mbar_try_wait(a, 0);
      if (!done && ks_globaltimer() - t0 > limit_ns) break;
    }
    if (!done) ks_record_error(err, KS_DEVERR_SELFTEST);
  }
  __syncthreads();
}

extern "C" {

const char *ks_status_string(int s) {
  switch (s) {
    case KS_OK: return "ok";
    case KS_ERR_NO_DEVICE: return "no_device";
    case KS_ERR_NO_DRIVER: return "no_driver";
    case KS_ERR_MODULE_LOAD: return "module_load_failed";
    case KS_ERR_KERNEL_NOT_FOUND: return "kernel_not_found";
    case KS_ERR_LAUNCH: return "launch_failed";
    case KS_ERR_MEMORY: return "memory_op_failed";
    case KS_ERR_COPY: return "copy_op_failed";
    case KS_ERR_EVENT: return "event_op_failed";
    case KS_ERR_DEVICE_NOT_FOUND: return "device_not_found";
    case KS_ERR_UNSUPPORTED: return "unsupported";
    case KS_ERR_OTHER: return "other";
    case KS_ERR_INVALID_CONFIG: return "invalid_config";
    case KS_ERR_INVALID_ARGS: return "invalid_args";
    case KS_ERR_WORKSPACE: return "workspace";
    case KS_ERR_DEVICE_TIMEOUT: return "device_timeout";
    case KS_ERR_ARCH: return "arch";
    default: return "unknown";
  }
}

int ks_abi_version(void) { return KS_ABI_VERSION; }
#ifndef KS_SOURCE_HASH
#define KS_SOURCE_HASH "unknown"
#endif
// "src <hash>": the hash of the sources, headers, flags and nvcc version this
// library was compiled from (kernscope_b200/build.py: source_hash()).
const char *ks_build_info(void) { return "kernscope_b200 sm_100a nvcc src " KS_SOURCE_HASH; }

int ks_gpu_device_count(int *count) {
  if (!count) return KS_ERR_INVALID_ARGS;
  *count = 0;
  cudaError_t e = cudaGetDeviceCount(count);
  if (e != cudaSuccess) {
    *count = 0;
    cudaGetLastError();
    return KS_ERR_NO_DEVICE;
  }
  return KS_OK;
}
int ks_gpu_set_device(int d) { return ks::map_cuda(cudaSetDevice(d)); }
int ks_gpu_get_device(int *d) { return d ? ks::map_cuda(cudaGetDevice(d)) : KS_ERR_INVALID_ARGS; }

int ks_gpu_arch(int dev, char *buf, size_t len) {
  int ma = 0, mi = 0;
  cudaError_t e = cudaDeviceGetAttribute(&ma, cudaDevAttrComputeCapabilityMajor, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&mi, cudaDevAttrComputeCapabilityMinor, dev);
  if (e != cudaSuccess) return ks::map_cuda(e);
  if (ma == 10 && mi == 0)
    snprintf(buf, len, "sm_100a");
  else
    snprintf(buf, len, "sm_%d%d", ma, mi);
  return KS_OK;
}
int ks_gpu_sm_count(int dev, int *n) {
  return n ? ks::map_cuda(cudaDeviceGetAttribute(n, cudaDevAttrMultiProcessorCount, dev)) : KS_ERR_INVALID_ARGS;
}
int ks_gpu_l2_bytes(int dev, size_t *b) {
  if (!b) return KS_ERR_INVALID_ARGS;
  int v = 0;
  int s = ks::map_cuda(cudaDeviceGetAttribute(&v, cudaDevAttrL2CacheSize, dev));
  *b = static_cast<size_t>(v);
  return s;
}
int ks_gpu_malloc(void **p, size_t n) {
  if (!p) return KS_ERR_INVALID_ARGS;
  return cudaMalloc(p, n) == cudaSuccess ? KS_OK : KS_ERR_MEMORY;
}
int ks_gpu_free(void *p) { return cudaFree(p) == cudaSuccess ? KS_OK : KS_ERR_MEMORY; }
int ks_gpu_memset(void *p, int v, size_t n, void *s) {
  return cudaMemsetAsync(p, v, n, static_cast<cudaStream_t>(s)) == cudaSuccess ? KS_OK : KS_ERR_MEMORY;
}
int ks_gpu_memcpy_htod(void *d, const void *h, size_t n, void *s) {
  return cudaMemcpyAsync(d, h, n, cudaMemcpyHostToDevice, static_cast<cudaStream_t>(s)) == cudaSuccess ? KS_OK
                                                                                                        : KS_ERR_COPY;
}
int ks_gpu_memcpy_dtoh(void *h, const void *d, size_t n, void *s) {
  return cudaMemcpyAsync(h, d, n, cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(s)) == cudaSuccess ? KS_OK
                                                                                                        : KS_ERR_COPY;
}
int ks_gpu_host_alloc(void **p, size_t n) {
  return cudaHostAlloc(p, n, cudaHostAllocDefault) == cudaSuccess ? KS_OK : KS_ERR_MEMORY;
}
int ks_gpu_host_free(void *p) { return cudaFreeHost(p) == cudaSuccess ? KS_OK : KS_ERR_MEMORY; }
int ks_gpu_stream_create(void **s) {
  cudaStream_t st;
  cudaError_t e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
  *s = st;
  return ks::map_cuda(e);
}
int ks_gpu_stream_destroy(void *s) { return ks::map_cuda(cudaStreamDestroy(static_cast<cudaStream_t>(s))); }
int ks_gpu_stream_synchronize(void *s) {
  return ks::map_cuda(cudaStreamSynchronize(static_cast<cudaStream_t>(s)));
}
int ks_gpu_synchronize(void) { return ks::map_cuda(cudaDeviceSynchronize()); }
int ks_gpu_event_create(void **ev) {
  cudaEvent_t e;
  if (cudaEventCreate(&e) != cudaSuccess) return KS_ERR_EVENT;
  *ev = e;
  return KS_OK;
}
int ks_gpu_event_destroy(void *ev) {
  return cudaEventDestroy(static_cast<cudaEvent_t>(ev)) == cudaSuccess ? KS_OK : KS_ERR_EVENT;
}
int ks_gpu_event_record(void *ev, void *s) {
  return cudaEventRecord(static_cast<cudaEvent_t>(ev), static_cast<cudaStream_t>(s)) == cudaSuccess ? KS_OK
                                                                                                    : KS_ERR_EVENT;
}
int ks_gpu_event_synchronize(void *ev) {
  return cudaEventSynchronize(static_cast<cudaEvent_t>(ev)) == cudaSuccess ? KS_OK : KS_ERR_EVENT;
}
int ks_gpu_event_elapsed_ms(void *a, void *b, float *ms) {
  return cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(a), static_cast<cudaEvent_t>(b)) == cudaSuccess
             ? KS_OK
             : KS_ERR_EVENT;
}

int ks_device_error_take(int *word) {
  if (!word) return KS_ERR_INVALID_ARGS;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return ks::map_cuda(e);
  int zero = 0;
  e = cudaMemcpyFromSymbol(word, g_ks_device_error, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_ks_device_error, &zero, sizeof(int));
  return ks::map_cuda(e);
}

int ks_set_wait_limit_ns(uint64_t limit_ns) {
  if (limit_ns == 0) return KS_ERR_INVALID_ARGS;
  g_wait_limit_ns.store(limit_ns);
  return KS_OK;
}

int ks_selftest_bounded_wait(uint64_t limit_ns, void *stream) {
  int s = ks::check_arch_sm100();
  if (s != KS_OK) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ks_selftest_wait_kernel<<<1, 32, 0, st>>>(limit_ns, ks::wait_ctx().err);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return ks::map_cuda(e);
  int word = 0;
  s = ks_device_error_take(&word);
  if (s != KS_OK) return s;
  return word == KS_DEVERR_SELFTEST ? KS_ERR_DEVICE_TIMEOUT : (word == 0 ? KS_OK : KS_ERR_OTHER);
}

}  // extern "C"
