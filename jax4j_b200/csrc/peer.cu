// Collectives over NVLink peer memory (one process per GPU, buffers mapped with CUDA IPC).
//
// Replaces the NCCL calls of the sharded paths: the row-sharded GEMV's all-gather of y
// (j4b_quant_matvec_allgather: the GEMV epilogue itself stores each output into every rank's
// buffer) and the data-parallel tape's all-reduce of [dg, loss] (j4b_peer_allreduce: every rank
// writes its vector into every rank's slot, then sums the slots in rank order -- deterministic,
// identical on all ranks).
//
// Every rank allocates one buffer (j4b_peer_alloc) and maps the others' (j4b_peer_open); a peer
// group holds all of them. Layout of each rank's buffer:
//   [0, 64)        step counter per channel (local; selects the parity half and the flag, advanced
//                  once per collective call by the rank's own kernel)
//   [64, 128)      finished-CTA counter of the reading kernel per channel (local)
//   [131072, end)  data, one slice per channel, each split into two parity halves of flagged
//                  words (gather_store: value and step flag in one 64-bit store)
// A reader of step k waits, word by word, until the flag k + 1 appears: no fence, arrival
// counter or remote atomic sits between a writer's data and the reader. The data of consecutive
// steps alternates halves, so a rank that runs one step ahead never overwrites what a slower rank
// still reads, and no rank gets two steps ahead: step k + 1 of every rank waits for every rank's
// words of step k + 1, which each rank writes only after its own step k is read.
// Every wait is bounded (about a second); a wait that gives up sets the group's status word.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "j4b_internal.h"
#include "j4b_wait.cuh"

namespace j4b {
namespace {

constexpr int kChannels = 16;
constexpr size_t kDataOffset = 131072;
constexpr uint64_t kPeerWaitNs = 1000000000ull;  // one second

struct PeerBases {
  uint8_t* base[kMaxPeerRanks];
};

// Waits (bounded) for the flag of step `want` in a flagged word and returns its value; on a
// timeout sets *timed_out (and every later word of the thread is taken as it is).
__device__ __forceinline__ float wait_word(const unsigned long long* p, unsigned want, uint64_t t0, bool& timed_out) {
  unsigned long long w = gather_load(p);
  while ((unsigned)(w >> 32) != want && !timed_out) {
    if (global_ns() - t0 > kPeerWaitNs) {
      timed_out = true;
      break;
    }
    w = gather_load(p);
  }
  return __uint_as_float((unsigned)w);
}

// The last CTA of the reading kernel to finish advances the channel's step counter.
__device__ __forceinline__ void finish_step(unsigned* step, unsigned* done, unsigned s) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *done = 0u;
      *(volatile unsigned*)step = s + 1u;
    }
  }
}

// Two consecutive flagged words (16-byte aligned) in one load; each 8-byte word is read
// single-copy atomically, so value and flag of a word always belong together.
__device__ __forceinline__ ulonglong2 gather_load2(const unsigned long long* p) {
  ulonglong2 w;
  asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(w.x), "=l"(w.y) : "l"(p) : "memory");
  return w;
}

constexpr int kWaitCopyThreads = 512;
constexpr int kWaitCopyPairs = 4;  // word pairs a thread loads before it checks any of their flags

// Copies this rank's gathered half (every source's flagged words of this step) to `out` once the
// flags show up, then advances the step counter. Launched as a programmatic dependent of the
// GEMV; it lets its own dependents launch at once (the next GEMV's weight prefetch overlaps the
// wait), and it waits for the GEMV to finish before it reads the step counter, which the previous
// step's copy advanced (a launch two kernels back is not otherwise ordered before this one).
// Each thread issues the loads of up to kWaitCopyPairs word pairs before it looks at a flag, and
// re-reads only a pair whose flags have not arrived: the copy costs about one load round trip
// when the peers' stores have landed.
__global__ void __launch_bounds__(kWaitCopyThreads) wait_copy_kernel(unsigned* step, unsigned* done,
                                                                     const unsigned long long* data,
                                                                     int64_t half_words, float* out, int64_t n,
                                                                     int* status) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const unsigned s = *(volatile unsigned*)step;
  const unsigned want = s + 1u;
  const unsigned long long* src = data + (int64_t)(s & 1u) * half_words;  // 16-byte aligned
  const uint64_t t0 = global_ns();
  bool timed_out = false;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
  if (((uintptr_t)out & 7u) == 0) {
    const int64_t npairs = n / 2;
    float2* out2 = reinterpret_cast<float2*>(out);
    for (int64_t p0 = tid; p0 < npairs; p0 += stride * kWaitCopyPairs) {
      ulonglong2 w[kWaitCopyPairs];
#pragma unroll
      for (int u = 0; u < kWaitCopyPairs; ++u)
        if (p0 + u * stride < npairs) w[u] = gather_load2(src + 2 * (p0 + u * stride));
#pragma unroll
      for (int u = 0; u < kWaitCopyPairs; ++u) {
        const int64_t p = p0 + u * stride;
        if (p >= npairs) break;
        while (((unsigned)(w[u].x >> 32) != want || (unsigned)(w[u].y >> 32) != want) && !timed_out) {
          if (global_ns() - t0 > kPeerWaitNs) {
            timed_out = true;
            break;
          }
          w[u] = gather_load2(src + 2 * p);
        }
        out2[p] = make_float2(__uint_as_float((unsigned)w[u].x), __uint_as_float((unsigned)w[u].y));
      }
    }
    if ((n & 1) && tid == 0) out[n - 1] = wait_word(src + n - 1, want, t0, timed_out);
  } else {
    for (int64_t i = tid; i < n; i += stride) out[i] = wait_word(src + i, want, t0, timed_out);
  }
  if (timed_out) atomicExch(status, 1);
  finish_step(step, done, s);
}

constexpr int kAllreduceThreads = 256;

// One thread per element: write it into slot `rank` of every rank as flagged words, then load slot
// q of every source q from this rank's buffer (all loads issued before any flag is checked; a
// slot whose flag has not arrived is re-read) and sum the slots in rank order.
__global__ void __launch_bounds__(kAllreduceThreads) allreduce_kernel(PeerBases bases, int nranks, int rank,
                                                                      int channel, int64_t slice_words,
                                                                      const float* src, int64_t n, float* out,
                                                                      int* status) {
  uint8_t* mine = bases.base[rank];
  unsigned* step = reinterpret_cast<unsigned*>(mine) + channel;
  unsigned* done = reinterpret_cast<unsigned*>(mine + 64) + channel;
  const unsigned s = *(volatile unsigned*)step;
  const unsigned want = s + 1u;
  const int64_t par = (int64_t)(s & 1u) * (slice_words / 2);
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  bool timed_out = false;
  if (i < n) {
    const float v = src[i];
#pragma unroll
    for (int p = 0; p < kMaxPeerRanks; ++p) {
      if (p < nranks) {
        unsigned long long* dst = reinterpret_cast<unsigned long long*>(bases.base[p] + kDataOffset) +
                                  channel * slice_words + par + (int64_t)rank * n;
        gather_store(dst + i, v, want);
      }
    }
    const unsigned long long* slots =
        reinterpret_cast<const unsigned long long*>(mine + kDataOffset) + channel * slice_words + par + i;
    unsigned long long w[kMaxPeerRanks];
#pragma unroll
    for (int q = 0; q < kMaxPeerRanks; ++q)
      if (q < nranks) w[q] = gather_load(slots + (int64_t)q * n);
    const uint64_t t0 = global_ns();
    float acc = 0.0f;
#pragma unroll
    for (int q = 0; q < kMaxPeerRanks; ++q) {
      if (q < nranks) {
        unsigned long long wq = w[q];
        while ((unsigned)(wq >> 32) != want && !timed_out) {
          if (global_ns() - t0 > kPeerWaitNs) timed_out = true;
          else wq = gather_load(slots + (int64_t)q * n);
        }
        const float x = __uint_as_float((unsigned)wq);
        acc = q == 0 ? x : __fadd_rn(acc, x);
      }
    }
    out[i] = acc;
  }
  if (timed_out) atomicExch(status, 1);
  finish_step(step, done, s);
}

}  // namespace
}  // namespace j4b

struct j4b_peer_group {
  int dev = 0, nranks = 0, rank = 0;
  size_t bytes = 0;
  uint8_t* base[j4b::kMaxPeerRanks] = {};
  int* status = nullptr;
};

using namespace j4b;

extern "C" int j4b_peer_alloc(int dev, size_t bytes, j4b_buf* out, uint8_t* handle) {
  J4B_REQUIRE(out != nullptr && handle != nullptr, "null argument");
  J4B_REQUIRE(bytes > kDataOffset, "peer buffers need more than %zu bytes", kDataOffset);
  int st = ensure_device(dev);
  if (st) return st;
  DeviceGuard guard(dev);
  void* p = nullptr;
  J4B_CUDA(cudaMalloc(&p, bytes), "cudaMalloc(peer buffer)");
  J4B_CUDA(cudaMemset(p, 0, bytes), "cudaMemset(peer buffer)");
  cudaIpcMemHandle_t h;
  J4B_CUDA(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle");
  static_assert(sizeof(h) == 64, "IPC handle size");
  std::memcpy(handle, &h, 64);
  *out = (j4b_buf)(uintptr_t)p;
  return J4B_OK;
}

extern "C" int j4b_peer_open(int dev, const uint8_t* handle, j4b_buf* out) {
  J4B_REQUIRE(out != nullptr && handle != nullptr, "null argument");
  int st = ensure_device(dev);
  if (st) return st;
  DeviceGuard guard(dev);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, 64);
  void* p = nullptr;
  J4B_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  *out = (j4b_buf)(uintptr_t)p;
  return J4B_OK;
}

extern "C" int j4b_peer_close(j4b_buf remote) {
  if (!remote) return J4B_OK;
  J4B_CUDA(cudaIpcCloseMemHandle((void*)(uintptr_t)remote), "cudaIpcCloseMemHandle");
  return J4B_OK;
}

extern "C" int j4b_peer_free(j4b_buf local) {
  if (!local) return J4B_OK;
  J4B_CUDA(cudaFree((void*)(uintptr_t)local), "cudaFree(peer buffer)");
  return J4B_OK;
}

extern "C" int j4b_peer_group_create(int dev, int nranks, int rank, const j4b_buf* bases, size_t bytes,
                                     j4b_peer_group** out) {
  J4B_REQUIRE(out != nullptr && bases != nullptr, "null argument");
  J4B_REQUIRE(nranks >= 1 && nranks <= kMaxPeerRanks, "peer groups hold 1..%d ranks", kMaxPeerRanks);
  J4B_REQUIRE(rank >= 0 && rank < nranks, "rank %d out of range", rank);
  J4B_REQUIRE(bytes > kDataOffset, "peer buffers need more than %zu bytes", kDataOffset);
  for (int p = 0; p < nranks; ++p) J4B_REQUIRE(bases[p] != 0 && bases[p] % 256 == 0, "peer buffer %d", p);
  int st = ensure_device(dev);
  if (st) return st;
  DeviceGuard guard(dev);
  j4b_peer_group* g = new j4b_peer_group();
  g->dev = dev;
  g->nranks = nranks;
  g->rank = rank;
  g->bytes = bytes;
  for (int p = 0; p < nranks; ++p) g->base[p] = (uint8_t*)(uintptr_t)bases[p];
  if (cudaMalloc(&g->status, sizeof(int)) != cudaSuccess || cudaMemset(g->status, 0, sizeof(int)) != cudaSuccess) {
    delete g;
    return set_error(J4B_ENOMEM, "peer group status allocation failed");
  }
  *out = g;
  return J4B_OK;
}

extern "C" int j4b_peer_group_free(j4b_peer_group* g) {
  if (!g) return J4B_OK;
  {
    DeviceGuard guard(g->dev);
    cudaFree(g->status);
  }
  delete g;
  return J4B_OK;
}

extern "C" int j4b_peer_status(j4b_peer_group* g, int* status) {
  J4B_REQUIRE(g != nullptr && status != nullptr, "null argument");
  DeviceGuard guard(g->dev);
  J4B_CUDA(cudaMemcpy(status, g->status, sizeof(int), cudaMemcpyDeviceToHost), "cudaMemcpy(peer status)");
  return J4B_OK;
}

namespace j4b {

int peer_group_ranks(const j4b_peer_group* g) { return g->nranks; }

// Flagged words per channel slice (both parity halves).
int64_t peer_slice_words(const j4b_peer_group* g) {
  return (int64_t)(((g->bytes - kDataOffset) / kChannels) / 256 * 256 / 8);
}

// Fills the GEMV's peer targets for `channel`.
int peer_gemv_targets(const j4b_peer_group* g, int channel, int64_t gathered_floats, GemvPeers* t) {
  J4B_REQUIRE(channel >= 0 && channel < kChannels, "channel %d out of range", channel);
  const int64_t slice = peer_slice_words(g);
  J4B_REQUIRE(2 * gathered_floats <= slice,
              "peer buffer slice too small for the gathered output (%lld words per parity half, %lld needed)",
              (long long)(slice / 2), (long long)gathered_floats);
  t->nranks = g->nranks;
  t->rank = g->rank;
  t->half_words = slice / 2;
  t->step = reinterpret_cast<const unsigned*>(g->base[g->rank]) + channel;
  for (int p = 0; p < g->nranks; ++p)
    t->y[p] = reinterpret_cast<unsigned long long*>(g->base[p] + kDataOffset) + channel * slice;
  return J4B_OK;
}

// Launches the waiting copy of the gathered output after the GEMV.
int peer_wait_copy(const j4b_peer_group* g, int channel, float* out, int64_t n, cudaStream_t stream) {
  uint8_t* mine = g->base[g->rank];
  const int64_t slice = peer_slice_words(g);
  unsigned* step = reinterpret_cast<unsigned*>(mine) + channel;
  unsigned* done = reinterpret_cast<unsigned*>(mine + 64) + channel;
  const unsigned long long* data = reinterpret_cast<const unsigned long long*>(mine + kDataOffset) + channel * slice;
  // about one word pair per thread, up to kWaitCopyPairs pairs per thread on one CTA per SM
  const int64_t ctas = ((n + 1) / 2 + kWaitCopyThreads - 1) / kWaitCopyThreads;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(ctas, 148));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kWaitCopyThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  J4B_CUDA(cudaLaunchKernelEx(&cfg, wait_copy_kernel, step, done, data, slice / 2, out, n, g->status),
           "wait_copy_kernel");
  count_launch();
  return J4B_OK;
}

}  // namespace j4b

extern "C" int j4b_peer_allreduce(j4b_peer_group* g, int channel, j4b_buf src, int64_t n, j4b_buf out,
                                  j4b_stream s) {
  J4B_REQUIRE(g != nullptr, "null peer group");
  J4B_REQUIRE(channel >= 0 && channel < kChannels, "channel %d out of range", channel);
  J4B_REQUIRE(n >= 1 && src && out, "all-reduce needs n >= 1 and buffers");
  const int64_t slice = peer_slice_words(g);
  J4B_REQUIRE(2 * (int64_t)g->nranks * n <= slice, "peer buffer slice too small for the all-reduce");
  J4B_REQUIRE((n + kAllreduceThreads - 1) / kAllreduceThreads <= 0x7fffffffLL, "all-reduce of %lld elements is too long",
              (long long)n);
  DeviceGuard guard(g->dev);
  cudaStream_t stream = resolve_stream(g->dev, s);
  PeerBases b;
  for (int p = 0; p < kMaxPeerRanks; ++p) b.base[p] = p < g->nranks ? g->base[p] : nullptr;
  allreduce_kernel<<<(unsigned)((n + kAllreduceThreads - 1) / kAllreduceThreads), kAllreduceThreads, 0, stream>>>(
      b, g->nranks, g->rank, channel, slice, (const float*)(uintptr_t)src, n, (float*)(uintptr_t)out, g->status);
  J4B_CHECK_LAUNCH("allreduce_kernel");
  return J4B_OK;
}
