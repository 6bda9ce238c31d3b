// Collectives over NVLink peer memory (one process per GPU, buffers mapped with CUDA IPC).
//
// Replaces the NCCL calls of the sharded paths: the row-sharded GEMV's all-gather of y
// (j4b_quant_matvec_allgather: the GEMV epilogue itself stores each output into every rank's
// buffer, and the GEMV's warps then copy the gathered words out as their flags arrive, in the
// same kernel) and the data-parallel tape's all-reduce of [dg, loss] (j4b_peer_allreduce: every rank
// writes its vector into every rank's slot, then sums the slots in rank order -- deterministic,
// identical on all ranks).
//
// Every rank allocates one buffer (j4b_peer_alloc) and maps the others' (j4b_peer_open); a peer
// group holds all of them. Layout of each rank's buffer:
//   [0, 64)        step counter per channel (local; selects the parity half and the flag, advanced
//                  once per collective call by the rank's own kernel)
//   [64, 128)      finished-reader counter per channel (local; the reading kernel's last CTA or
//                  warp to finish advances the step counter and resets it)
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

struct PeerBases {
  uint8_t* base[kMaxPeerRanks];
};

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

// Fills the GEMV's peer targets for `channel`: every rank's gathered buffer, this rank's step and
// finished-warp counters, and the gathered output `out` the GEMV's warps copy into.
int peer_gemv_targets(const j4b_peer_group* g, int channel, float* out, int64_t gathered_floats, GemvPeers* t) {
  J4B_REQUIRE(channel >= 0 && channel < kChannels, "channel %d out of range", channel);
  const int64_t slice = peer_slice_words(g);
  J4B_REQUIRE(2 * gathered_floats <= slice,
              "peer buffer slice too small for the gathered output (%lld words per parity half, %lld needed)",
              (long long)(slice / 2), (long long)gathered_floats);
  uint8_t* mine = g->base[g->rank];
  t->nranks = g->nranks;
  t->rank = g->rank;
  t->half_words = slice / 2;
  t->step = reinterpret_cast<unsigned*>(mine) + channel;
  t->done = reinterpret_cast<unsigned*>(mine + 64) + channel;
  t->out = out;
  t->gathered = gathered_floats;
  t->status = g->status;
  for (int p = 0; p < g->nranks; ++p)
    t->y[p] = reinterpret_cast<unsigned long long*>(g->base[p] + kDataOffset) + channel * slice;
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
