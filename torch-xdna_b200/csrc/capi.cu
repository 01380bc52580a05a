// Library-wide entry points and host helpers: last error, device checks, the device error word
// that bounded waits write, and TMA tensor-map encoding.
#include <atomic>
#include <cstdarg>
#include <cstring>
#include <mutex>

#include "host_util.h"
#include "sm100.cuh"

namespace xdna {

// The device error word: code, site, block, count. Written by kernels whose bounded waits ran out;
// read and cleared by xdna_take_device_error(). A file-scope __device__ array: every GPU that loads
// the library holds its own copy, and no allocation is needed to reach it.
__device__ int g_device_error[4];

static thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mutex;
// Per device: the SM count (0 = unchecked, -1 = not an sm_100 device) and the device address of
// g_device_error. The address is stored first and the count published after it with release order, so
// a thread that reads a positive count (acquire) also sees the address. The cached address belongs to
// the device's primary context: the library must not be used across a cudaDeviceReset of that device.
std::atomic<int> g_sm_count[kMaxDevices];
std::atomic<int*> g_err_ptr[kMaxDevices];
}  // namespace

int check_device(int* sm_count) {
  int dev = 0;
  XDNA_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(XDNA_ERR_DEVICE, "device ordinal %d out of range", dev);
  int sms = g_sm_count[dev].load(std::memory_order_acquire);
  if (sms == 0) {
    std::lock_guard<std::mutex> lock(g_mutex);
    sms = g_sm_count[dev].load(std::memory_order_relaxed);  // another thread may have finished meanwhile
    if (sms == 0) {
      cudaDeviceProp prop;
      XDNA_CUDA(cudaGetDeviceProperties(&prop, dev));
      if (prop.major != 10) {
        g_sm_count[dev].store(-1, std::memory_order_release);
        return fail(XDNA_ERR_DEVICE, "device %d (%s) is sm_%d%d; these kernels need sm_100a (B200)", dev, prop.name,
                    prop.major, prop.minor);
      }
      void* p = nullptr;
      XDNA_CUDA(cudaGetSymbolAddress(&p, g_device_error));
      g_err_ptr[dev].store(static_cast<int*>(p), std::memory_order_relaxed);
      sms = prop.multiProcessorCount;
      g_sm_count[dev].store(sms, std::memory_order_release);
    }
  }
  if (sms < 0) return fail(XDNA_ERR_DEVICE, "device %d is not an sm_100 GPU", dev);
  if (sm_count) *sm_count = sms;
  return XDNA_OK;
}

// The self-test of the bounded waits: one thread waits, with limit_ns, on a fresh mbarrier that nothing
// ever arrives at -- the same bounded wait as every role of the library's kernels -- so the wait runs out,
// records XDNA_ERR_TIMEOUT at site kSelftestSite in the device error word, and the kernel returns.
constexpr int kSelftestSite = 99;
__global__ void wait_selftest_kernel(int* err, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, err, kSelftestSite, limit_ns);
  __syncthreads();
}

int* device_error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  if (g_sm_count[dev].load(std::memory_order_acquire) <= 0) return nullptr;
  return g_err_ptr[dev].load(std::memory_order_relaxed);
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(XDNA_ERR_CUDA, "launch of %s failed: %s", what, cudaGetErrorString(e));
  return XDNA_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int encode_tma(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
               const uint64_t* strides_bytes, const uint32_t* box, const char* what, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(XDNA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (!aligned16(base)) return fail(XDNA_ERR_INVALID, "%s: base address is not 16-byte aligned", what);
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) {
    if (strides_bytes[i] % 16 != 0)
      return fail(XDNA_ERR_INVALID, "%s: row pitch %llu bytes is not a multiple of 16", what,
                  (unsigned long long)strides_bytes[i]);
    s[i] = strides_bytes[i];
  }
  CUresult r = fn(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, s, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(XDNA_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, (int)r);
  return XDNA_OK;
}

}  // namespace xdna

extern "C" {

const char* xdna_last_error(void) { return xdna::t_last_error.c_str(); }

int xdna_abi_version(void) { return 1; }

int xdna_ipc_alloc(size_t bytes, void** dev_ptr) {
  XDNA_CHECK_ARG(dev_ptr != nullptr && bytes > 0, "ipc_alloc: bad arguments");
  XDNA_CUDA(cudaMalloc(dev_ptr, bytes));
  return XDNA_OK;
}

int xdna_ipc_free(void* dev_ptr) {
  if (dev_ptr != nullptr) XDNA_CUDA(cudaFree(dev_ptr));
  return XDNA_OK;
}

int xdna_ipc_handle(const void* dev_ptr, void* handle64) {
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
  XDNA_CHECK_ARG(dev_ptr != nullptr && handle64 != nullptr, "ipc_handle: null pointer");
  cudaIpcMemHandle_t h;
  XDNA_CUDA(cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)));
  std::memcpy(handle64, &h, sizeof(h));
  return XDNA_OK;
}

int xdna_ipc_open(const void* handle64, void** dev_ptr) {
  XDNA_CHECK_ARG(dev_ptr != nullptr && handle64 != nullptr, "ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  XDNA_CUDA(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return XDNA_OK;
}

int xdna_ipc_close(void* dev_ptr) {
  if (dev_ptr != nullptr) XDNA_CUDA(cudaIpcCloseMemHandle(dev_ptr));
  return XDNA_OK;
}

int xdna_device_check(int device) {
  int cur = 0;
  XDNA_CUDA(cudaGetDevice(&cur));
  if (cur != device) XDNA_CUDA(cudaSetDevice(device));
  int rc = xdna::check_device(nullptr);
  if (cur != device) cudaSetDevice(cur);
  return rc;
}

int xdna_selftest_wait_timeout(uint64_t limit_ns, void* stream) {
  int rc = xdna::check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(limit_ns >= 1000 && limit_ns <= 2000000000ull, "selftest: limit must be 1 us .. 2 s");
  xdna::wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(xdna::device_error_word(), limit_ns);
  return xdna::check_launch("wait_selftest_kernel");
}

int xdna_take_device_error(int* code, int* site, void* stream) {
  int rc = xdna::check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  int* word = xdna::device_error_word();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int host[4] = {0, 0, 0, 0};
  XDNA_CUDA(cudaMemcpyAsync(host, word, sizeof(host), cudaMemcpyDeviceToHost, s));
  XDNA_CUDA(cudaStreamSynchronize(s));
  if (host[0] != 0) XDNA_CUDA(cudaMemsetAsync(word, 0, sizeof(host), s));
  XDNA_CUDA(cudaStreamSynchronize(s));
  if (code) *code = host[0];
  if (site) *site = host[1];
  return XDNA_OK;
}

}  // extern "C"
