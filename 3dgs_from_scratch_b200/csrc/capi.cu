// capi.cu -- status plumbing, launch accounting and small C-ABI utilities.
#include <atomic>
#include <mutex>

#include "gs_common.cuh"

namespace gs {

// One status word per device (module globals are instantiated per device).
__device__ uint32_t g_status_word;

static std::atomic<uint64_t> g_launches{0};
static std::atomic<int> g_last_cuda_error{0};

void count_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return GS_OK;
  g_last_cuda_error.store((int)e);
  return GS_ERR_CUDA;
}

int launch_status() { return cuda_status(cudaGetLastError()); }

// The current CUDA context's process-unique id (cuCtxGetId), 0 when there is
// no current context yet. Driver entry points are resolved once through the
// runtime, so the library needs no link against libcuda.
typedef int (*CtxGetCurrentFn)(void **);
typedef int (*CtxGetIdFn)(void *, unsigned long long *);
static CtxGetCurrentFn g_ctx_get_current = nullptr;
static CtxGetIdFn g_ctx_get_id = nullptr;
static std::once_flag g_ctx_once;

static void resolve_context_api() {
  void *f = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 12000, cudaEnableDefault, &q) ==
          cudaSuccess && q == cudaDriverEntryPointSuccess)
    g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(f);
  f = nullptr;
  if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &f, 12000, cudaEnableDefault, &q) ==
          cudaSuccess && q == cudaDriverEntryPointSuccess)
    g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(f);
}

unsigned long long current_context_id() {
  std::call_once(g_ctx_once, resolve_context_api);
  void *ctx = nullptr;
  if (g_ctx_get_current == nullptr || g_ctx_get_current(&ctx) != 0 || ctx == nullptr) return 0;
  unsigned long long id = 0;
  if (g_ctx_get_id == nullptr || g_ctx_get_id(ctx, &id) != 0) return 0;
  return id;
}

int symbol_address(const void *symbol, SymbolCache *cache, void **out) {
  const unsigned long long ctx = current_context_id();
  if (ctx != 0 && cache->context_id == ctx) {
    *out = cache->address;
    return GS_OK;
  }
  void *p = nullptr;
  int rc = cuda_status(cudaGetSymbolAddress(&p, symbol));
  if (rc) return rc;
  // The lookup made the context current if it was not yet; cache against it.
  cache->context_id = ctx != 0 ? ctx : current_context_id();
  cache->address = p;
  *out = p;
  return GS_OK;
}

__global__ void zero_words_kernel(uint32_t *__restrict__ p, size_t words) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < words;
       i += (size_t)gridDim.x * blockDim.x)
    p[i] = 0u;
}

int zero_async(void *p, size_t bytes, cudaStream_t st) {
  if (bytes == 0) return GS_OK;
  if (((uintptr_t)p & 3) || (bytes & 3)) return cuda_status(cudaMemsetAsync(p, 0, bytes, st));
  const size_t words = bytes / 4;
  const size_t want = (words + 255) / 256;
  const unsigned grid = (unsigned)(want < 1024 ? want : 1024);
  zero_words_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<uint32_t *>(p), words);
  count_launch();
  return launch_status();
}

uint32_t *device_status_word() {
  thread_local SymbolCache cache;
  void *p = nullptr;
  if (symbol_address(&g_status_word, &cache, &p) != GS_OK) return nullptr;
  return reinterpret_cast<uint32_t *>(p);
}

}  // namespace gs

using namespace gs;

extern "C" int gs_version(void) { return 2; }

extern "C" int gs_last_cuda_error(void) { return g_last_cuda_error.load(); }

extern "C" uint64_t gs_launch_count(void) { return g_launches.load(); }

// Launches recorded into a CUDA graph run at each replay, not at capture: the
// caller takes them off at capture (negative n) and adds them per replay, so
// that the launch count stays the number of this library's kernels that ran.
extern "C" void gs_note_launches(int64_t n) {
  g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed);
}

extern "C" int gs_sync(void *stream) {
  return cuda_status(cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)));
}

static int read_and_clear_status(cudaStream_t st) {
  uint32_t *w = device_status_word();
  if (w == nullptr) return GS_ERR_CUDA;
  uint32_t v = 0;
  int rc = cuda_status(cudaMemcpyAsync(&v, w, sizeof(v), cudaMemcpyDeviceToHost, st));
  if (rc) return rc;
  rc = cuda_status(cudaStreamSynchronize(st));
  if (rc) return rc;
  if (v != 0) {
    rc = cuda_status(cudaMemsetAsync(w, 0, sizeof(uint32_t), st));
    if (rc) return rc;
    return (int)v;
  }
  return GS_OK;
}

extern "C" int gs_check_status(void *stream) {
  return read_and_clear_status(reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int gs_read_total(const int64_t *total_dev, int64_t *total_host, void *stream) {
  if (total_dev == nullptr || total_host == nullptr) return GS_ERR_INVALID_ARGUMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int rc = cuda_status(cudaMemcpyAsync(total_host, total_dev, sizeof(int64_t),
                                       cudaMemcpyDeviceToHost, st));
  if (rc) return rc;
  return read_and_clear_status(st);
}

// Self-test of the bounded-wait mechanism: one thread waits on a flag that
// nothing sets, gives up after kSpinLimit polls, records
// GS_ERR_DEVICE_TIMEOUT in the status word and exits; the host reads it back.
__global__ void bounded_wait_probe_kernel(const uint32_t *flag, uint32_t *status) {
  uint32_t v, spins = 0;
  do {
    v = gs::ld_volatile_u32(flag);
  } while (v == 0 && ++spins < gs::kSpinLimit);
  if (v == 0) atomicExch(status, (uint32_t)GS_ERR_DEVICE_TIMEOUT);
}

// The device status word, copied to dst (one uint32 in device memory) on
// `stream`, without clearing it.
extern "C" int gs_status_export(uint32_t *dst, void *stream) {
  if (dst == nullptr) return GS_ERR_INVALID_ARGUMENT;
  uint32_t *w = device_status_word();
  if (w == nullptr) return GS_ERR_CUDA;
  return cuda_status(cudaMemcpyAsync(dst, w, sizeof(uint32_t), cudaMemcpyDeviceToDevice,
                                     reinterpret_cast<cudaStream_t>(stream)));
}

__global__ void status_merge_kernel(const uint32_t *src, uint32_t *status) {
  if (*src != 0u) atomicCAS(status, 0u, (uint32_t)GS_ERR_PEER);
}

// Makes the device status word non-zero when *src (device memory, e.g. the
// maximum of every rank's exported status) is: a code of this rank's own is
// kept, otherwise GS_ERR_PEER is recorded.
extern "C" int gs_status_merge(const uint32_t *src, void *stream) {
  if (src == nullptr) return GS_ERR_INVALID_ARGUMENT;
  uint32_t *w = device_status_word();
  if (w == nullptr) return GS_ERR_CUDA;
  status_merge_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(src, w);
  count_launch();
  return launch_status();
}

// The bounded-wait probe without the read-back: leaves GS_ERR_DEVICE_TIMEOUT
// in the status word, as a kernel whose wait gave up would, for tests of the
// paths gated on it.
extern "C" int gs_selftest_set_timeout(const uint32_t *flag_dev, void *stream) {
  if (flag_dev == nullptr) return GS_ERR_INVALID_ARGUMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  bounded_wait_probe_kernel<<<1, 1, 0, st>>>(flag_dev, device_status_word());
  count_launch();
  return launch_status();
}

extern "C" int gs_selftest_bounded_wait(const uint32_t *flag_dev, void *stream) {
  if (flag_dev == nullptr) return GS_ERR_INVALID_ARGUMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  bounded_wait_probe_kernel<<<1, 1, 0, st>>>(flag_dev, device_status_word());
  count_launch();
  int rc = launch_status();
  if (rc) return rc;
  return read_and_clear_status(st);
}
