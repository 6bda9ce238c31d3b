// Internal helpers shared by the engine's translation units: status/error plumbing, the
// per-device context table and launch bookkeeping.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "jax4j_b200.h"

namespace j4b {

constexpr int kMaxDevices = 16;

struct DeviceCtx {
  bool ready = false;
  int sm_count = 0;
  cudaStream_t stream = nullptr;
  char name[256] = {0};
};

DeviceCtx* device_ctx(int dev);          // nullptr if dev is out of range
int ensure_device(int dev);              // lazily initialises dev; returns status
int device_of(const void* ptr, int* dev);  // device owning a device pointer
cudaStream_t resolve_stream(int dev, j4b_stream s);

// Sets the calling thread's last error and returns code.
int set_error(int code, const char* fmt, ...);
int cuda_error(cudaError_t e, const char* what);

struct Counters {
  std::atomic<uint64_t> dispatches{0}, allocations{0}, releases{0}, h2d{0}, d2h{0},
      compilations{0};
};
Counters& counters();

inline void count_launch(uint64_t n = 1) { counters().dispatches += n; }

// RAII guard restoring the caller's current device.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// C[b] = A[b] . B[b] on the tcgen05 tensor cores; terms 1 = bf16 operands, 3 = fp32-accurate split
int tc_matmul(const float* a, const float* b, float* out, int64_t batch, int64_t m, int64_t k, int64_t n,
              int terms, int dev, cudaStream_t stream);
int tc_status_read(int dev, int* value);
// C (m x n) = op(A) . op(B) on tcgen05 with op = transpose where ta / tb (A stored [k, m], B [n, k])
int tc_matmul_t(const float* a, const float* b, float* out, int64_t m, int64_t k, int64_t n, bool ta, bool tb,
                int terms, int dev, cudaStream_t stream);
// C (m x n) = op(A) . op(B), precision as j4b_matmul (SIMT, skinny or tensor-core kernels); batch > 1
// only without transposes
int matmul_strided(const float* a, const float* b, float* out, int64_t batch, int64_t m, int64_t k, int64_t n,
                   bool ta, bool tb, int precision, int dev, cudaStream_t stream);
}  // namespace j4b
#include <cuda_bf16.h>
namespace j4b {
// C (m x n) = A (m x k f32) . Bt^T, Bt bf16 hi (and lo for terms 3) [n, kp] K-major, kp = k
// rounded up to 64 with zero padding
int tc_gemm_bt(const float* a, int64_t m, int64_t k, const __nv_bfloat16* bt_hi, const __nv_bfloat16* bt_lo,
               int64_t n, int terms, float* out, int dev, cudaStream_t stream);
// C (m x n) = A . Bt^T with both operands bf16 hi (and lo for terms 3) K-major [m, kp] / [n, kp],
// kp a multiple of 64, zero-padded
int tc_gemm_bf16(const __nv_bfloat16* a_hi, const __nv_bfloat16* a_lo, int64_t m, int64_t kp,
                 const __nv_bfloat16* bt_hi, const __nv_bfloat16* bt_lo, int64_t n, int terms, float* out, int dev,
                 cudaStream_t stream);
// f32 [rows, cols] (row stride ld) -> bf16 hi (and lo) [rows, kp], zero-padded columns
int tc_split_rows(const float* src, int64_t rows, int64_t cols, int64_t ld, int64_t kp, __nv_bfloat16* hi,
                  __nv_bfloat16* lo, cudaStream_t stream);

// ---- collectives over peer memory (peer.cu) ----
constexpr int kMaxPeerRanks = 8;

// Where a GEMV's y goes when it is all-gathered over peer memory.
struct GemvPeers {
  int nranks, rank;
  unsigned long long* y[kMaxPeerRanks];  // each rank's gathered buffer (the channel's data slice)
  unsigned* step;                        // this rank's step counter of the channel
  unsigned* done;                        // this rank's finished-warp counter of the channel
  int64_t half_words;                    // flagged words per parity half of the slice
  float* out;                            // the gathered output, [batch][rows * nranks]
  int64_t gathered;                      // its floats
  int* status;                           // the group's status word (a wait that gave up)
};

// A flagged word of the peer buffers: a float value in the low half, the step flag (step + 1) in
// the high half, written and read as one 64-bit access (single-copy atomic), so a reader that
// sees the flag of its step sees that step's value: no fence and no arrival counter between the
// writer's data and the reader's wait.
__device__ __forceinline__ void gather_store(unsigned long long* p, float v, unsigned flag) {
  const unsigned long long w = ((unsigned long long)flag << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long gather_load(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
// Two consecutive flagged words (16-byte aligned) in one load; each 8-byte word is read
// single-copy atomically, so value and flag of a word always belong together.
__device__ __forceinline__ ulonglong2 gather_load2(const unsigned long long* p) {
  ulonglong2 w;
  asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(w.x), "=l"(w.y) : "l"(p) : "memory");
  return w;
}
constexpr uint64_t kPeerWaitNs = 1000000000ull;  // a peer's words: one second before giving up
int peer_group_ranks(const j4b_peer_group* g);
int peer_gemv_targets(const j4b_peer_group* g, int channel, float* out, int64_t gathered_floats, GemvPeers* t);

// out[k] = sum of a[sources[p]] for p in [offsets[k], offsets[k+1]), in that order
int launch_segment_sum(const float* a, const int64_t* offsets, const int64_t* sources, int64_t n_dst,
                       float* out, j4b_stream s);

}  // namespace j4b

#define J4B_CHECK_LAUNCH(what)                                 \
  do {                                                         \
    cudaError_t e_ = cudaGetLastError();                       \
    if (e_ != cudaSuccess) return ::j4b::cuda_error(e_, what); \
    ::j4b::count_launch();                                     \
  } while (0)

#define J4B_CUDA(call, what)                                   \
  do {                                                         \
    cudaError_t e_ = (call);                                   \
    if (e_ != cudaSuccess) return ::j4b::cuda_error(e_, what); \
  } while (0)

#define J4B_REQUIRE(cond, ...)                                   \
  do {                                                           \
    if (!(cond)) return ::j4b::set_error(J4B_EINVAL, __VA_ARGS__); \
  } while (0)
