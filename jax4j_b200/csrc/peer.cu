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
//   [0, 64)        step counter per channel (local; selects the parity half, advanced once per
//                  collective call by the rank's own kernel)
//   [64, 128)      arrival counter of the calling kernel's CTAs per channel (local)
//   [4096, 69632)  arrival counters per channel: [channel][slot], slot = chunk * 8 + source
//   [131072, end)  data, one slice per channel, each split into two parity halves
// Step k of a channel is complete for source s once
//   - GEMV all-gather: s's arrival counter reaches (k + 1) x kPeerCallUnits (every call adds
//     exactly that many units, whatever its grid);
//   - all-reduce: the chunk's slot holds the epoch k + 1 (stored by s after its chunk's data, so
//     a chunk that earlier calls did not use carries no stale count);
// both compared modulo 2^32. The data of consecutive steps alternates halves, so a rank that runs
// one step ahead never overwrites what a slower rank still reads (and no rank gets further ahead:
// each step waits for every rank's arrival at that step).
// Every wait is bounded (about a second); a wait that gives up sets the group's status word.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "j4b_internal.h"

namespace j4b {
namespace {

constexpr int kChannels = 16;
constexpr size_t kCtrOffset = 4096, kDataOffset = 131072;
constexpr int kSlotsPerChannel = 1024;
constexpr uint32_t kPeerWaitLimit = 1u << 24;

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// v has not yet reached target, modulo 2^32.
__device__ __forceinline__ bool before(unsigned v, unsigned target) { return (int)(v - target) < 0; }

struct PeerBases {
  uint8_t* base[kMaxPeerRanks];
};

// Waits until every source's arrival counter reaches (step + 1) x kPeerCallUnits, then copies
// this rank's gathered half to `out`; the last CTA advances the step counter.
// Launched as a programmatic dependent of the GEMV: it may start while the GEMV still runs (it
// reads only the arrival counters, the step counter and the gathered data the counters vouch
// for), and it releases its own dependents at once so the next kernel's prologue -- the next
// GEMV's weight prefetch -- overlaps the wait.
__global__ void wait_copy_kernel(unsigned* step, unsigned* done, const unsigned* ctr, int nranks,
                                 const float* data, int64_t half_floats, float* out, int64_t n,
                                 int* status) {
  __shared__ unsigned s_step;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (threadIdx.x == 0) {
    const unsigned s = *(volatile unsigned*)step;
    const unsigned target = (s + 1u) * kPeerCallUnits;
    for (int src = 0; src < nranks; ++src) {
      uint32_t it = 0;
      while (before(ld_acquire_sys(ctr + src), target)) {
        if (++it > kPeerWaitLimit) {
          atomicExch(status, 1);
          break;
        }
        __nanosleep(32);
      }
    }
    s_step = s;
  }
  __syncthreads();
  const float* src = data + (int64_t)(s_step & 1u) * half_floats;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = src[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *done = 0u;
      *(volatile unsigned*)step = s_step + 1u;
    }
  }
}

// One CTA per 1024-element chunk: write the chunk into slot `rank` of every rank, publish the
// step's epoch in the chunk's counter slot at every rank, wait for every source's epoch, sum the
// slots in rank order.
__global__ void allreduce_kernel(PeerBases bases, int nranks, int rank, int channel, int64_t slice_floats,
                                 const float* src, int64_t n, float* out, int* status) {
  constexpr int kChunk = 1024;
  __shared__ unsigned s_step;
  uint8_t* mine = bases.base[rank];
  unsigned* step = reinterpret_cast<unsigned*>(mine) + channel;
  unsigned* done = reinterpret_cast<unsigned*>(mine + 64) + channel;
  if (threadIdx.x == 0) s_step = *(volatile unsigned*)step;
  __syncthreads();
  const unsigned s = s_step;
  const int64_t half = slice_floats / 2;
  const int64_t par = (int64_t)(s & 1u) * half;
  const int64_t c = blockIdx.x, i0 = c * kChunk, i1 = min(n, i0 + kChunk);
  for (int p = 0; p < nranks; ++p) {
    float* dst = reinterpret_cast<float*>(bases.base[p] + kDataOffset) + channel * slice_floats + par + (int64_t)rank * n;
    for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int p = 0; p < nranks; ++p) {
      unsigned* ctr = reinterpret_cast<unsigned*>(bases.base[p] + kCtrOffset) + channel * kSlotsPerChannel;
      st_release_sys(ctr + c * 8 + rank, s + 1u);
    }
    const unsigned* mctr = reinterpret_cast<const unsigned*>(mine + kCtrOffset) + channel * kSlotsPerChannel;
    for (int q = 0; q < nranks; ++q) {
      uint32_t it = 0;
      while (before(ld_acquire_sys(mctr + c * 8 + q), s + 1u)) {
        if (++it > kPeerWaitLimit) {
          atomicExch(status, 1);
          break;
        }
        __nanosleep(32);
      }
    }
  }
  __syncthreads();
  const float* slots = reinterpret_cast<const float*>(mine + kDataOffset) + channel * slice_floats + par;
  for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    float acc = slots[i];
    for (int q = 1; q < nranks; ++q) acc = __fadd_rn(acc, slots[(int64_t)q * n + i]);
    out[i] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *done = 0u;
      *(volatile unsigned*)step = s + 1u;
    }
  }
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

int64_t peer_slice_floats(const j4b_peer_group* g) {
  return (int64_t)(((g->bytes - kDataOffset) / kChannels) / 256 * 256 / 4);
}

// Fills the GEMV's peer targets for `channel` and launches the waiting copy after it.
int peer_gemv_targets(const j4b_peer_group* g, int channel, int64_t gathered_floats, GemvPeers* t) {
  J4B_REQUIRE(channel >= 0 && channel < kChannels, "channel %d out of range", channel);
  const int64_t slice = peer_slice_floats(g);
  J4B_REQUIRE(2 * gathered_floats <= slice, "peer buffer slice too small for the gathered output");
  t->nranks = g->nranks;
  t->rank = g->rank;
  t->half_floats = slice / 2;
  t->step = reinterpret_cast<const unsigned*>(g->base[g->rank]) + channel;
  for (int p = 0; p < g->nranks; ++p) {
    t->y[p] = reinterpret_cast<float*>(g->base[p] + kDataOffset) + channel * slice;
    t->ctr[p] = reinterpret_cast<unsigned*>(g->base[p] + kCtrOffset) + channel * kSlotsPerChannel + g->rank;
  }
  return J4B_OK;
}

int peer_wait_copy(const j4b_peer_group* g, int channel, float* out, int64_t n, cudaStream_t stream) {
  uint8_t* mine = g->base[g->rank];
  const int64_t slice = peer_slice_floats(g);
  unsigned* step = reinterpret_cast<unsigned*>(mine) + channel;
  unsigned* done = reinterpret_cast<unsigned*>(mine + 64) + channel;
  const unsigned* ctr = reinterpret_cast<const unsigned*>(mine + kCtrOffset) + channel * kSlotsPerChannel;
  const float* data = reinterpret_cast<const float*>(mine + kDataOffset) + channel * slice;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 1023) / 1024, 148));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  J4B_CUDA(cudaLaunchKernelEx(&cfg, wait_copy_kernel, step, done, ctr, g->nranks, data, slice / 2, out, n,
                              g->status),
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
  J4B_REQUIRE((n + 1023) / 1024 * 8 <= kSlotsPerChannel, "all-reduce of %lld elements exceeds the counter slots",
              (long long)n);
  const int64_t slice = peer_slice_floats(g);
  J4B_REQUIRE(2 * (int64_t)g->nranks * n <= slice, "peer buffer slice too small for the all-reduce");
  DeviceGuard guard(g->dev);
  cudaStream_t stream = resolve_stream(g->dev, s);
  PeerBases b;
  for (int p = 0; p < kMaxPeerRanks; ++p) b.base[p] = p < g->nranks ? g->base[p] : nullptr;
  allreduce_kernel<<<(unsigned)((n + 1023) / 1024), 256, 0, stream>>>(b, g->nranks, g->rank, channel, slice,
                                                                      (const float*)(uintptr_t)src, n,
                                                                      (float*)(uintptr_t)out, g->status);
  J4B_CHECK_LAUNCH("allreduce_kernel");
  return J4B_OK;
}
