// Engine lifecycle, memory and error plumbing.
//
// Replaces the reference's FFM driver wrapper (cuda/backend/cuda/CudaRuntime.java:38-713): one
// non-blocking stream per device instead of one process-wide context on device 0, stream-ordered
// allocation (cudaMallocAsync into the device's default pool) instead of the hand-written
// size-bucketed pool, and a thread-safe stream-ordered free instead of the Cleaner queue.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "j4b_internal.h"

namespace j4b {
namespace {

DeviceCtx g_ctx[kMaxDevices];
std::mutex g_mu;
thread_local char t_last_error[1024] = "";
Counters g_counters;

}  // namespace

Counters& counters() { return g_counters; }

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_error(cudaError_t e, const char* what) {
  if (e == cudaErrorMemoryAllocation)
    return set_error(J4B_ENOMEM, "%s failed: %s (code %d)", what, cudaGetErrorName(e), (int)e);
  return set_error(J4B_ECUDA, "%s failed: %s (code %d)", what, cudaGetErrorName(e), (int)e);
}

DeviceCtx* device_ctx(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  return &g_ctx[dev];
}

int ensure_device(int dev) {
  DeviceCtx* c = device_ctx(dev);
  if (!c) return set_error(J4B_EINVAL, "device index %d out of range", dev);
  if (c->ready) return J4B_OK;
  std::lock_guard<std::mutex> lock(g_mu);
  if (c->ready) return J4B_OK;
  int count = 0;
  J4B_CUDA(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
  if (dev >= count) return set_error(J4B_EINVAL, "device %d not present (%d devices)", dev, count);
  DeviceGuard guard(dev);
  cudaDeviceProp prop;
  J4B_CUDA(cudaGetDeviceProperties(&prop, dev), "cudaGetDeviceProperties");
  if (prop.major != 10)
    return set_error(J4B_EUNSUPPORTED, "device %d is sm_%d%d; this engine is built for sm_100a",
                     dev, prop.major, prop.minor);
  c->sm_count = prop.multiProcessorCount;
  snprintf(c->name, sizeof(c->name), "%s", prop.name);
  J4B_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "cudaStreamCreate");
  // Keep freed blocks in the stream-ordered pool instead of returning them to the driver on
  // every synchronisation (the reference keeps a 256 MiB free-list for the same reason).
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
    uint64_t threshold = 1ull << 30;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
  }
  c->ready = true;
  return J4B_OK;
}

int device_of(const void* ptr, int* dev) {
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, ptr);
  if (e != cudaSuccess || attr.type != cudaMemoryTypeDevice) {
    cudaGetLastError();
    return set_error(J4B_EINVAL, "pointer %p is not device memory", ptr);
  }
  *dev = attr.device;
  return ensure_device(*dev);
}

cudaStream_t resolve_stream(int dev, j4b_stream s) {
  if (s) return (cudaStream_t)s;
  DeviceCtx* c = device_ctx(dev);
  return c ? c->stream : nullptr;
}

}  // namespace j4b

using namespace j4b;

extern "C" int j4b_init(const int* devices, int n) {
  if (!devices || n <= 0) return ensure_device(0);
  for (int i = 0; i < n; i++) {
    int st = ensure_device(devices[i]);
    if (st) return st;
  }
  return J4B_OK;
}

extern "C" int j4b_device_count(int* count) {
  if (!count) return set_error(J4B_EINVAL, "count is null");
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  *count = n;
  return J4B_OK;
}

extern "C" int j4b_device_name(int dev, char* buf, size_t len) {
  int st = ensure_device(dev);
  if (st) return st;
  if (!buf || len == 0) return set_error(J4B_EINVAL, "empty name buffer");
  snprintf(buf, len, "%s", device_ctx(dev)->name);
  return J4B_OK;
}

extern "C" int j4b_sm_count(int dev, int* count) {
  int st = ensure_device(dev);
  if (st) return st;
  *count = device_ctx(dev)->sm_count;
  return J4B_OK;
}

extern "C" int j4b_get_stream(int dev, j4b_stream* stream) {
  int st = ensure_device(dev);
  if (st) return st;
  *stream = (j4b_stream)device_ctx(dev)->stream;
  return J4B_OK;
}

extern "C" int j4b_sync(int dev) {
  int st = ensure_device(dev);
  if (st) return st;
  DeviceGuard guard(dev);
  J4B_CUDA(cudaStreamSynchronize(device_ctx(dev)->stream), "cudaStreamSynchronize");
  J4B_CUDA(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  return J4B_OK;
}

extern "C" int j4b_last_error(char* buf, size_t len) {
  if (!buf || len == 0) return J4B_EINVAL;
  snprintf(buf, len, "%s", t_last_error);
  return J4B_OK;
}

extern "C" int j4b_get_diagnostics(j4b_diagnostics* out) {
  if (!out) return set_error(J4B_EINVAL, "diagnostics is null");
  Counters& c = counters();
  out->dispatches = c.dispatches.load();
  out->allocations = c.allocations.load();
  out->releases = c.releases.load();
  out->h2d_bytes = c.h2d.load();
  out->d2h_bytes = c.d2h.load();
  out->compilations = c.compilations.load();
  return J4B_OK;
}

extern "C" int j4b_alloc(int dev, size_t bytes, j4b_buf* out) {
  if (!out) return set_error(J4B_EINVAL, "out is null");
  int st = ensure_device(dev);
  if (st) return st;
  DeviceGuard guard(dev);
  void* p = nullptr;
  if (bytes == 0) bytes = 4;
  J4B_CUDA(cudaMallocAsync(&p, bytes, device_ctx(dev)->stream), "cudaMallocAsync");
  counters().allocations++;
  *out = (j4b_buf)(uintptr_t)p;
  return J4B_OK;
}

extern "C" int j4b_free(j4b_buf buf) {
  if (!buf) return J4B_OK;
  int dev = 0;
  int st = device_of((const void*)(uintptr_t)buf, &dev);
  if (st) return st;
  DeviceGuard guard(dev);
  J4B_CUDA(cudaFreeAsync((void*)(uintptr_t)buf, device_ctx(dev)->stream), "cudaFreeAsync");
  counters().releases++;
  return J4B_OK;
}

extern "C" int j4b_h2d(j4b_buf dst, const void* src, size_t bytes, j4b_stream s) {
  if (bytes == 0) return J4B_OK;
  if (!dst || !src) return set_error(J4B_EINVAL, "null pointer in h2d");
  int dev = 0;
  int st = device_of((const void*)(uintptr_t)dst, &dev);
  if (st) return st;
  DeviceGuard guard(dev);
  cudaStream_t stream = resolve_stream(dev, s);
  J4B_CUDA(cudaMemcpyAsync((void*)(uintptr_t)dst, src, bytes, cudaMemcpyHostToDevice, stream),
           "cudaMemcpyAsync(HtoD)");
  counters().h2d += bytes;
  return J4B_OK;
}

extern "C" int j4b_d2h(void* dst, j4b_buf src, size_t bytes, j4b_stream s) {
  if (bytes == 0) return J4B_OK;
  if (!dst || !src) return set_error(J4B_EINVAL, "null pointer in d2h");
  int dev = 0;
  int st = device_of((const void*)(uintptr_t)src, &dev);
  if (st) return st;
  DeviceGuard guard(dev);
  cudaStream_t stream = resolve_stream(dev, s);
  J4B_CUDA(cudaMemcpyAsync(dst, (const void*)(uintptr_t)src, bytes, cudaMemcpyDeviceToHost,
                           stream),
           "cudaMemcpyAsync(DtoH)");
  J4B_CUDA(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
  counters().d2h += bytes;
  return J4B_OK;
}

extern "C" int j4b_d2d(j4b_buf dst, j4b_buf src, size_t bytes, j4b_stream s) {
  if (bytes == 0) return J4B_OK;
  if (!dst || !src) return set_error(J4B_EINVAL, "null pointer in d2d");
  int dev = 0;
  int st = device_of((const void*)(uintptr_t)dst, &dev);
  if (st) return st;
  DeviceGuard guard(dev);
  J4B_CUDA(cudaMemcpyAsync((void*)(uintptr_t)dst, (const void*)(uintptr_t)src, bytes,
                           cudaMemcpyDeviceToDevice, resolve_stream(dev, s)),
           "cudaMemcpyAsync(DtoD)");
  return J4B_OK;
}
