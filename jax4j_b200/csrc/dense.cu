// Eager dense primitives of the engine SPI (core/tensor/spi/ComputeBackend.java:48-280).
//
// Each entry point is one launch on the caller's stream, with the shape checks of the reference
// backend done on the host first. These kernels serve calls the fused-tape executor does not
// absorb (and any caller that drives the SPI op by op, as the reference's ExecutionPlan replay
// does): 128-bit vector access where alignment allows, grid sizes in multiples of the SM count,
// warp-shuffle reductions with double accumulators for sums (CpuBackend.java:264-311 sums in
// double), and a shared-memory tiled transpose.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "j4b_internal.h"
#include "j4b_math.cuh"

namespace j4b {
namespace {

constexpr int kThreads = 256;

unsigned grid_for(int64_t n, int dev, int per_thread = 1) {
  const int64_t want = (n + (int64_t)kThreads * per_thread - 1) / ((int64_t)kThreads * per_thread);
  const int64_t cap = (int64_t)device_ctx(dev)->sm_count * 16;
  return (unsigned)(want < 1 ? 1 : (want > cap ? cap : want));
}

__global__ void fill_kernel(float* __restrict__ out, int64_t n, float v) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t n4 = ((uintptr_t)out & 15) == 0 ? n / 4 : 0;
  float4 v4 = make_float4(v, v, v, v);
  for (int64_t j = i; j < n4; j += stride) reinterpret_cast<float4*>(out)[j] = v4;
  for (int64_t j = n4 * 4 + i; j < n; j += stride) out[j] = v;
}

__global__ void binary_kernel(int op, const float* __restrict__ a, const float* __restrict__ b,
                              float* __restrict__ out, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = apply_binary(op, a[i], b[i]);
}

__global__ void scalar_kernel(int op, const float* __restrict__ a, float s, float* __restrict__ out,
                              int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = apply_binary(op, a[i], s);
}

__global__ void unary_kernel(int op, const float* __restrict__ a, float* __restrict__ out,
                             int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = apply_unary(op, a[i]);
}

__global__ void relu_backward_kernel(const float* __restrict__ up, const float* __restrict__ in,
                                     float* __restrict__ out, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = in[i] > 0.0f ? up[i] : 0.0f;
}

// 32x32 tiles through shared memory (padded to 33 to avoid bank conflicts): both the read of a
// and the write of out are coalesced, unlike the reference's one-thread-per-element kernel
// (cuda/backend/cuda/CudaBackend.java:96-101).
__global__ void transpose_kernel(const float* __restrict__ a, float* __restrict__ out,
                                 int64_t rows, int64_t cols) {
  __shared__ float tile[32][33];
  const int64_t c0 = (int64_t)blockIdx.x * 32, r0 = (int64_t)blockIdx.y * 32;
  for (int j = threadIdx.y; j < 32; j += 8) {
    const int64_t r = r0 + j, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[j][threadIdx.x] = a[r * cols + c];
  }
  __syncthreads();
  for (int j = threadIdx.y; j < 32; j += 8) {
    const int64_t c = c0 + j, r = r0 + threadIdx.x;
    if (r < rows && c < cols) out[c * rows + r] = tile[threadIdx.x][j];
  }
}

__device__ __forceinline__ double warp_sum(double v) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Strict '>' comparison, NaN never wins: CpuBackend.reduceMax (CpuBackend.java:274-284).
__device__ __forceinline__ float gt_max(float best, float v) { return v > best ? v : best; }

__device__ __forceinline__ float warp_gt_max(float v) {
  for (int o = 16; o; o >>= 1) v = gt_max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Full reductions: block partials (double for sums), then the last block to finish folds them in
// block order (deterministic).
template <bool kMax>
__global__ void reduce_all_kernel(const float* __restrict__ a, int64_t n, double* __restrict__ part,
                                  unsigned* __restrict__ done, float* __restrict__ out) {
  __shared__ double sh[32];
  __shared__ bool last;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  double acc = kMax ? -INFINITY : 0.0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    if (kMax) acc = gt_max((float)acc, a[i]);
    else acc += a[i];
  }
  if (kMax) acc = warp_gt_max((float)acc);
  else acc = warp_sum(acc);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sh[warp] = acc;
  __syncthreads();
  if (warp == 0) {
    double v = lane < (int)(blockDim.x >> 5) ? sh[lane] : (kMax ? -INFINITY : 0.0);
    v = kMax ? (double)warp_gt_max((float)v) : warp_sum(v);
    if (lane == 0) {
      part[blockIdx.x] = v;
      __threadfence();
      last = atomicAdd(done, 1u) == gridDim.x - 1;
    }
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    double total = kMax ? -INFINITY : 0.0;
    for (unsigned b = 0; b < gridDim.x; b++) {
      const double v = __ldcg(part + b);
      total = kMax ? (double)gt_max((float)total, (float)v) : total + v;
    }
    out[0] = (float)total;
    *done = 0u;
  }
}

// Axis reductions over [outer, axis, inner].
// inner == 1: one warp per output row, shuffle reduction.
enum AxisOp { kSum = 0, kMaxOp = 1, kArgMax = 2 };

template <int OP>
__global__ void axis_rows_kernel(const float* __restrict__ a, int64_t outer, int64_t axis,
                                 float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row >= outer) return;
  const float* p = a + row * axis;
  if (OP == kSum) {
    double s = 0.0;
    for (int64_t i = lane; i < axis; i += 32) s += p[i];
    s = warp_sum(s);
    if (lane == 0) out[row] = (float)s;
  } else if (OP == kMaxOp) {
    // Math.max chain: NaN anywhere makes the result NaN (CpuBackend.java:313-329).
    float m = -INFINITY;
    for (int64_t i = lane; i < axis; i += 32) m = java_max(m, p[i]);
    for (int o = 16; o; o >>= 1) m = java_max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) out[row] = m;
  } else {
    // First NaN wins, else the first maximum (CpuBackend.java:331-355): reduce (key, index) with
    // NaN ranked above everything and ties broken by the lower index.
    float best = -INFINITY;
    int64_t bi = axis;  // sentinel: nothing seen
    bool nan = false;
    for (int64_t i = lane; i < axis; i += 32) {
      const float v = p[i];
      if (v != v) {
        if (!nan || i < bi) { nan = true; bi = i; }
        break;
      }
      if (!nan && (v > best || bi == axis)) {
        if (v > best || (v == best && i < bi)) { best = v; bi = i; }
      }
    }
    for (int o = 16; o; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const long long oi = __shfl_xor_sync(0xffffffffu, (long long)bi, o);
      const bool onan = __shfl_xor_sync(0xffffffffu, (int)nan, o);
      bool take;
      if (onan != nan) take = onan;
      else if (nan) take = oi < bi;
      else if (oi == axis) take = false;
      else if (bi == axis) take = true;
      else take = ob > best || (ob == best && oi < bi);
      if (take) { best = ob; bi = oi; nan = onan; }
    }
    if (lane == 0) out[row] = (float)(bi == axis ? 0 : bi);
  }
}

// inner > 1: 32 columns x 8 row groups per block; coalesced along inner.
template <int OP>
__global__ void axis_cols_kernel(const float* __restrict__ a, int64_t outer, int64_t axis,
                                 int64_t inner, float* __restrict__ out) {
  __shared__ double sv[8][33];
  __shared__ long long si[8][33];
  const int64_t col = (int64_t)blockIdx.x * 32 + threadIdx.x;
  const int64_t o = blockIdx.y;
  const int ty = threadIdx.y;
  double acc = OP == kSum ? 0.0 : -INFINITY;
  long long bi = -1;
  bool nan = false;
  if (col < inner) {
    const float* p = a + o * axis * inner + col;
    for (int64_t i = ty; i < axis; i += 8) {
      const float v = p[i * inner];
      if (OP == kSum) acc += v;
      else if (OP == kMaxOp) acc = java_max((float)acc, v);
      else {
        if (nan) continue;
        if (v != v) { nan = true; bi = i; acc = v; }
        else if (bi < 0 || v > (float)acc) { acc = v; bi = i; }
      }
    }
  }
  sv[ty][threadIdx.x] = nan ? (double)NAN : acc;
  si[ty][threadIdx.x] = nan ? -2 - bi : bi;  // NaN encoded below -1 so it sorts by index too
  __syncthreads();
  if (ty == 0 && col < inner) {
    double r = sv[0][threadIdx.x];
    long long ri = si[0][threadIdx.x];
    for (int y = 1; y < 8; y++) {
      const double v = sv[y][threadIdx.x];
      const long long vi = si[y][threadIdx.x];
      if (OP == kSum) r += v;
      else if (OP == kMaxOp) r = java_max((float)r, (float)v);
      else {
        const bool rn = ri <= -2, vn = vi <= -2;
        const long long ria = rn ? -2 - ri : ri, via = vn ? -2 - vi : vi;
        bool take;
        if (vi == -1) take = false;
        else if (ri == -1) take = true;
        else if (rn != vn) take = vn;
        else if (rn) take = via < ria;
        else take = v > r || (v == r && via < ria);
        if (take) { r = v; ri = vi; }
      }
    }
    float res;
    if (OP == kArgMax) res = (float)(ri <= -2 ? -2 - ri : (ri < 0 ? 0 : ri));
    else res = (float)r;
    out[o * inner + col] = res;
  }
}

// maxAxisBackward (CpuBackend.java:357-391): zero, then route upstream to the first max.
__global__ void max_axis_backward_kernel(const float* __restrict__ up, const float* __restrict__ in,
                                         int64_t outer, int64_t axis, int64_t inner,
                                         float* __restrict__ out) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= outer * inner) return;
  const int64_t o = idx / inner, n = idx % inner;
  const int64_t base = o * axis * inner + n;
  int64_t bi = 0;
  float best = -INFINITY;
  for (int64_t i = 0; i < axis; i++) {
    const float v = in[base + i * inner];
    out[base + i * inner] = 0.0f;
    if (v != v || v > best) {
      best = v;
      bi = i;
      if (v != v) {
        for (int64_t j = i + 1; j < axis; j++) out[base + j * inner] = 0.0f;
        break;
      }
    }
  }
  out[base + bi * inner] = up[idx];
}

struct BcastArgs {
  int rank;
  int64_t dst_stride[8];
  int64_t src_stride[8];
};

__global__ void broadcast_kernel(const float* __restrict__ a, float* __restrict__ out, int64_t n,
                                 BcastArgs b) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t rem = i, off = 0;
    for (int d = 0; d < b.rank; d++) {
      const int64_t c = rem / b.dst_stride[d];
      rem -= c * b.dst_stride[d];
      off += c * b.src_stride[d];
    }
    out[i] = a[off];
  }
}

__global__ void reindex_kernel(const float* __restrict__ a, int64_t n_src, const int* __restrict__ map,
                               int64_t n_dst, float* __restrict__ out) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_dst; i += stride) {
    const int m = map[i];
    out[i] = (m >= 0 && m < n_src) ? a[m] : 0.0f;
  }
}

__global__ void scatter_add_kernel(const float* __restrict__ a, int64_t n_src, const int* __restrict__ map,
                                   int64_t n_dst, float* __restrict__ out) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_src; i += stride) {
    const int m = map[i];
    if (m >= 0 && m < n_dst) atomicAdd(out + m, a[i]);
  }
}

// scatterAdd with a static map, as a gather: destination k sums its sources in increasing
// source order (offsets[k] .. offsets[k+1] of `sources`), the float order of the reference's
// sequential loop (ComputeBackend.java:261-274), so the result is bit-exact and deterministic.
__global__ void segment_sum_kernel(const float* __restrict__ a, const int64_t* __restrict__ offsets,
                                   const int64_t* __restrict__ sources, int64_t n_dst,
                                   float* __restrict__ out) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n_dst; k += stride) {
    float acc = 0.0f;
    for (int64_t p = offsets[k]; p < offsets[k + 1]; ++p) acc = __fadd_rn(acc, a[sources[p]]);
    out[k] = acc;
  }
}

// PRNG: ComputeBackend.java:282-295 (splitmix64), bit-exact uniforms.
__device__ __forceinline__ uint64_t mix64(uint64_t v) {
  v = (v ^ (v >> 30)) * 0xBF58476D1CE4E5B9ULL;
  v = (v ^ (v >> 27)) * 0x94D049BB133111EBULL;
  return v ^ (v >> 31);
}

__global__ void random_kernel(int normal, int64_t seed, int64_t counter, float* __restrict__ out,
                              int64_t n) {
  const uint64_t kPhi = 0x9E3779B97F4A7C15ULL;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    if (!normal) {
      const uint64_t m = mix64((uint64_t)seed + kPhi * (uint64_t)(counter + i));
      out[i] = (float)(m >> 40) * 0x1.0p-24f;
    } else {
      // Box-Muller in double like ComputeBackend.java:70-73; CUDA's double log/cos are within an
      // ulp or two, so the float result matches the reference almost always, not always.
      const uint64_t m1 = mix64((uint64_t)seed + kPhi * (uint64_t)(counter + 2 * i));
      const uint64_t m2 = mix64((uint64_t)seed + kPhi * (uint64_t)(counter + 2 * i + 1));
      const float u1 = (float)((m1 >> 40) + 1) * 0x1.0p-24f;
      const float u2 = (float)(m2 >> 40) * 0x1.0p-24f;
      out[i] = (float)(sqrt(-2.0 * log((double)u1)) * cos(2.0 * 3.141592653589793 * (double)u2));
    }
  }
}

// Skinny fp32 matmuls, where a 64 x 64 output tile would leave most of the GPU idle (a logits
// layer's n = 10, or its gradient's k = 10): fp32 FMA accumulation in ascending p, batch in
// grid.y.
// k <= 32: one thread per output element, the k products summed in order.
// Operand strides: A(i, p) = A[i * sai + p * sap], B(p, j) = B[p * sbp + j * sbj] (a transposed
// operand is read in place).
__global__ void __launch_bounds__(256) gemm_short_k_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                                           float* __restrict__ C, int64_t M, int64_t K, int64_t N,
                                                           int64_t sai, int64_t sap, int64_t sbp, int64_t sbj) {
  const int64_t bz = blockIdx.y;
  const int64_t idx = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (idx >= M * N) return;
  const int64_t i = idx / N, j = idx % N;
  const float* a = A + bz * M * K + i * sai;
  const float* b = B + bz * K * N + j * sbj;
  float acc = 0.f;
  for (int64_t p = 0; p < K; p++) acc = fmaf(__ldg(a + p * sap), __ldg(b + p * sbp), acc);
  C[bz * M * N + idx] = acc;
}

// n <= 32: one warp per row of C; lane l takes p = l, l + 32, ... and keeps n partial sums, which
// the warp adds lane-wise (butterfly), so the sum order is fixed.
__global__ void __launch_bounds__(256) gemm_narrow_n_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                                            float* __restrict__ C, int64_t M, int64_t K, int N,
                                                            int64_t sai, int64_t sap, int64_t sbp, int64_t sbj) {
  const int64_t bz = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int64_t i = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (i >= M) return;
  const float* a = A + bz * M * K + i * sai;
  const float* b = B + bz * K * N;
  float acc[32];
#pragma unroll
  for (int j = 0; j < 32; j++) acc[j] = 0.f;
  int64_t p = lane;
  for (; p + 96 < K; p += 128) {  // four rows of B in flight, products added in ascending p
    float av[4];
#pragma unroll
    for (int u = 0; u < 4; u++) av[u] = __ldg(a + (p + 32 * u) * sap);
#pragma unroll
    for (int j = 0; j < 32; j++) {
      if (j < N) {
        const float b0 = __ldg(b + (p)*sbp + j * sbj), b1 = __ldg(b + (p + 32) * sbp + j * sbj);
        const float b2 = __ldg(b + (p + 64) * sbp + j * sbj), b3 = __ldg(b + (p + 96) * sbp + j * sbj);
        acc[j] = fmaf(av[0], b0, acc[j]);
        acc[j] = fmaf(av[1], b1, acc[j]);
        acc[j] = fmaf(av[2], b2, acc[j]);
        acc[j] = fmaf(av[3], b3, acc[j]);
      }
    }
  }
  for (; p < K; p += 32) {
    const float av = __ldg(a + p * sap);
    const float* br = b + p * sbp;
#pragma unroll
    for (int j = 0; j < 32; j++)
      if (j < N) acc[j] = fmaf(av, __ldg(br + j * sbj), acc[j]);
  }
  float mine = 0.f;
#pragma unroll
  for (int j = 0; j < 32; j++) {
    if (j >= N) break;
    float v = acc[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == j) mine = v;
  }
  if (lane < N) C[bz * M * N + i * N + lane] = mine;
}

// fp32 SIMT matmul (precision 0): 64x64 output tile per 256-thread block, 4x4 per thread,
// fp32 FMA accumulation; batch in grid.z.
__global__ void __launch_bounds__(256) sgemm_kernel(const float* __restrict__ A,
                                                    const float* __restrict__ B, float* __restrict__ C,
                                                    int64_t M, int64_t K, int64_t N, int64_t sai, int64_t sap,
                                                    int64_t sbp, int64_t sbj) {
  __shared__ float As[16][64 + 4];
  __shared__ float Bs[16][64 + 4];
  const int64_t bz = blockIdx.z;
  A += bz * M * K;
  B += bz * K * N;
  C += bz * M * N;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int64_t row0 = (int64_t)blockIdx.y * 64, col0 = (int64_t)blockIdx.x * 64;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += 16) {
    for (int i = threadIdx.x; i < 64 * 16; i += 256) {
      const int r = i / 16, kk = i % 16;
      const int64_t gr = row0 + r, gk = k0 + kk;
      As[kk][r] = (gr < M && gk < K) ? A[gr * sai + gk * sap] : 0.f;
      const int kb = i / 64, c = i % 64;
      const int64_t gk2 = k0 + kb, gc = col0 + c;
      Bs[kb][c] = (gk2 < K && gc < N) ? B[gk2 * sbp + gc * sbj] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; kk++) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; i++) av[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; j++) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int64_t r = row0 + ty * 4 + i, c = col0 + tx * 4 + j;
      if (r < M && c < N) C[r * N + c] = acc[i][j];
    }
}

bool is_binary(int op) { return op >= J4B_ADD && op <= J4B_MIN; }
bool is_unary(int op) { return op >= J4B_NEG && op <= J4B_SIGN; }

}  // namespace
}  // namespace j4b

using namespace j4b;

#define J4B_DEVICE_OF(ptr)                                          \
  int dev = 0;                                                      \
  {                                                                 \
    int st_ = device_of((const void*)(uintptr_t)(ptr), &dev);       \
    if (st_) return st_;                                            \
  }                                                                 \
  DeviceGuard guard_(dev);                                          \
  cudaStream_t stream = resolve_stream(dev, s)

// After J4B_DEVICE_OF(out): an input must live on out's device (a kernel launched on out's
// device must not be handed another GPU's memory, or host memory).
#define J4B_SAME_DEVICE(ptr, what)                                                           \
  do {                                                                                       \
    int in_dev_ = -1;                                                                        \
    int st_ = device_of((const void*)(uintptr_t)(ptr), &in_dev_);                            \
    if (st_) return st_;                                                                     \
    if (in_dev_ != dev)                                                                      \
      return set_error(J4B_EINVAL, "%s is on device %d but the output is on device %d", what, \
                       in_dev_, dev);                                                        \
  } while (0)

extern "C" int j4b_fill(j4b_buf out, int64_t n, float value, j4b_stream s) {
  J4B_REQUIRE(n >= 0, "negative element count");
  if (n == 0) return J4B_OK;
  J4B_DEVICE_OF(out);
  fill_kernel<<<grid_for(n, dev, 4), kThreads, 0, stream>>>((float*)(uintptr_t)out, n, value);
  J4B_CHECK_LAUNCH("fill_kernel");
  return J4B_OK;
}

extern "C" int j4b_binary(int op, j4b_buf a, j4b_buf b, j4b_buf out, int64_t n, j4b_stream s) {
  J4B_REQUIRE(is_binary(op), "not a binary op: %d", op);
  J4B_REQUIRE(n >= 0, "negative element count");
  if (n == 0) return J4B_OK;
  J4B_DEVICE_OF(out);
  binary_kernel<<<grid_for(n, dev), kThreads, 0, stream>>>(op, (const float*)(uintptr_t)a,
                                                          (const float*)(uintptr_t)b,
                                                          (float*)(uintptr_t)out, n);
  J4B_CHECK_LAUNCH("binary_kernel");
  return J4B_OK;
}

extern "C" int j4b_scalar(int op, j4b_buf a, double value, j4b_buf out, int64_t n, j4b_stream s) {
  J4B_REQUIRE(is_binary(op), "not a scalar op: %d", op);
  if (n == 0) return J4B_OK;
  J4B_DEVICE_OF(out);
  scalar_kernel<<<grid_for(n, dev), kThreads, 0, stream>>>(op, (const float*)(uintptr_t)a,
                                                          (float)value, (float*)(uintptr_t)out, n);
  J4B_CHECK_LAUNCH("scalar_kernel");
  return J4B_OK;
}

extern "C" int j4b_unary(int op, j4b_buf a, j4b_buf out, int64_t n, j4b_stream s) {
  J4B_REQUIRE(is_unary(op), "not a unary op: %d", op);
  if (n == 0) return J4B_OK;
  J4B_DEVICE_OF(out);
  unary_kernel<<<grid_for(n, dev), kThreads, 0, stream>>>(op, (const float*)(uintptr_t)a,
                                                         (float*)(uintptr_t)out, n);
  J4B_CHECK_LAUNCH("unary_kernel");
  return J4B_OK;
}

extern "C" int j4b_relu_backward(j4b_buf up, j4b_buf in, j4b_buf out, int64_t n, j4b_stream s) {
  if (n == 0) return J4B_OK;
  J4B_DEVICE_OF(out);
  relu_backward_kernel<<<grid_for(n, dev), kThreads, 0, stream>>>(
      (const float*)(uintptr_t)up, (const float*)(uintptr_t)in, (float*)(uintptr_t)out, n);
  J4B_CHECK_LAUNCH("relu_backward_kernel");
  return J4B_OK;
}

extern "C" int j4b_transpose(j4b_buf a, j4b_buf out, int64_t rows, int64_t cols, j4b_stream s) {
  J4B_REQUIRE(rows > 0 && cols > 0, "transpose requires a non-empty rank-2 tensor");
  J4B_DEVICE_OF(out);
  dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32));
  transpose_kernel<<<grid, dim3(32, 8), 0, stream>>>((const float*)(uintptr_t)a,
                                                     (float*)(uintptr_t)out, rows, cols);
  J4B_CHECK_LAUNCH("transpose_kernel");
  return J4B_OK;
}

static int reduce_all(bool is_max, j4b_buf a, int64_t n, j4b_buf out, j4b_stream s) {
  J4B_REQUIRE(n >= 0, "negative element count");
  J4B_DEVICE_OF(out);
  if (n > 0) J4B_SAME_DEVICE(a, "the input");
  const unsigned grid = grid_for(n, dev, 8);
  void* ws = nullptr;
  J4B_CUDA(cudaMallocAsync(&ws, grid * sizeof(double) + 16, stream), "cudaMallocAsync(reduce)");
  unsigned* done = (unsigned*)((char*)ws + grid * sizeof(double));
  J4B_CUDA(cudaMemsetAsync(done, 0, sizeof(unsigned), stream), "cudaMemsetAsync(reduce)");
  if (is_max)
    reduce_all_kernel<true><<<grid, kThreads, 0, stream>>>((const float*)(uintptr_t)a, n,
                                                          (double*)ws, done, (float*)(uintptr_t)out);
  else
    reduce_all_kernel<false><<<grid, kThreads, 0, stream>>>((const float*)(uintptr_t)a, n,
                                                           (double*)ws, done, (float*)(uintptr_t)out);
  cudaError_t e = cudaGetLastError();
  cudaFreeAsync(ws, stream);
  if (e != cudaSuccess) return cuda_error(e, "reduce_all_kernel");
  count_launch();
  return J4B_OK;
}

extern "C" int j4b_reduce_sum(j4b_buf a, int64_t n, j4b_buf out, j4b_stream s) {
  return reduce_all(false, a, n, out, s);
}
extern "C" int j4b_reduce_max(j4b_buf a, int64_t n, j4b_buf out, j4b_stream s) {
  return reduce_all(true, a, n, out, s);
}

template <int OP>
static int axis_reduce(j4b_buf a, int64_t outer, int64_t axis, int64_t inner, j4b_buf out,
                       j4b_stream s, const char* name) {
  J4B_REQUIRE(outer > 0 && axis > 0 && inner > 0, "%s requires a non-empty tensor", name);
  J4B_DEVICE_OF(out);
  if (inner == 1) {
    const int64_t threads = outer * 32;
    axis_rows_kernel<OP><<<(unsigned)((threads + kThreads - 1) / kThreads), kThreads, 0, stream>>>(
        (const float*)(uintptr_t)a, outer, axis, (float*)(uintptr_t)out);
  } else {
    dim3 grid((unsigned)((inner + 31) / 32), (unsigned)outer);
    axis_cols_kernel<OP><<<grid, dim3(32, 8), 0, stream>>>((const float*)(uintptr_t)a, outer, axis,
                                                          inner, (float*)(uintptr_t)out);
  }
  J4B_CHECK_LAUNCH(name);
  return J4B_OK;
}

extern "C" int j4b_sum_axis(j4b_buf a, int64_t outer, int64_t axis, int64_t inner, j4b_buf out,
                            j4b_stream s) {
  return axis_reduce<kSum>(a, outer, axis, inner, out, s, "sumAxis");
}
extern "C" int j4b_max_axis(j4b_buf a, int64_t outer, int64_t axis, int64_t inner, j4b_buf out,
                            j4b_stream s) {
  return axis_reduce<kMaxOp>(a, outer, axis, inner, out, s, "maxAxis");
}
extern "C" int j4b_argmax_axis(j4b_buf a, int64_t outer, int64_t axis, int64_t inner, j4b_buf out,
                               j4b_stream s) {
  return axis_reduce<kArgMax>(a, outer, axis, inner, out, s, "argMaxAxis");
}

extern "C" int j4b_max_axis_backward(j4b_buf up, j4b_buf in, int64_t outer, int64_t axis,
                                     int64_t inner, j4b_buf out, j4b_stream s) {
  J4B_REQUIRE(outer > 0 && axis > 0 && inner > 0, "maxAxisBackward requires a non-empty tensor");
  J4B_DEVICE_OF(out);
  const int64_t n = outer * inner;
  max_axis_backward_kernel<<<(unsigned)((n + kThreads - 1) / kThreads), kThreads, 0, stream>>>(
      (const float*)(uintptr_t)up, (const float*)(uintptr_t)in, outer, axis, inner,
      (float*)(uintptr_t)out);
  J4B_CHECK_LAUNCH("max_axis_backward_kernel");
  return J4B_OK;
}

extern "C" int j4b_broadcast_to(j4b_buf a, const int64_t* src_dims, int src_rank,
                                const int64_t* dst_dims, int dst_rank, j4b_buf out, j4b_stream s) {
  J4B_REQUIRE(dst_rank >= 1 && dst_rank <= 8 && src_rank >= 0 && src_rank <= dst_rank,
              "broadcastTo supports ranks up to 8");
  BcastArgs b;
  b.rank = dst_rank;
  int64_t sd[8];
  const int pad = dst_rank - src_rank;
  for (int i = 0; i < dst_rank; i++) sd[i] = i < pad ? 1 : src_dims[i - pad];
  int64_t stride = 1, total = 1;
  for (int i = dst_rank - 1; i >= 0; i--) {
    J4B_REQUIRE(sd[i] == dst_dims[i] || sd[i] == 1, "cannot broadcast dimension %d: %lld to %lld", i,
                (long long)sd[i], (long long)dst_dims[i]);
    b.src_stride[i] = sd[i] == 1 ? 0 : stride;
    stride *= sd[i];
    b.dst_stride[i] = total;
    total *= dst_dims[i];
  }
  if (total == 0) return J4B_OK;
  J4B_DEVICE_OF(out);
  broadcast_kernel<<<grid_for(total, dev), kThreads, 0, stream>>>((const float*)(uintptr_t)a,
                                                                 (float*)(uintptr_t)out, total, b);
  J4B_CHECK_LAUNCH("broadcast_kernel");
  return J4B_OK;
}

extern "C" int j4b_reindex(j4b_buf a, int64_t n_src, j4b_buf map, int64_t n_dst, j4b_buf out,
                           j4b_stream s) {
  J4B_REQUIRE(n_dst >= 0 && n_src >= 0, "negative sizes");
  if (n_dst == 0) return J4B_OK;
  J4B_DEVICE_OF(out);
  reindex_kernel<<<grid_for(n_dst, dev), kThreads, 0, stream>>>(
      (const float*)(uintptr_t)a, n_src, (const int*)(uintptr_t)map, n_dst, (float*)(uintptr_t)out);
  J4B_CHECK_LAUNCH("reindex_kernel");
  return J4B_OK;
}

extern "C" int j4b_scatter_add(j4b_buf a, int64_t n_src, j4b_buf map, int64_t n_dst, j4b_buf out,
                               j4b_stream s) {
  J4B_REQUIRE(n_dst >= 0 && n_src >= 0, "negative sizes");
  J4B_DEVICE_OF(out);
  J4B_CUDA(cudaMemsetAsync((void*)(uintptr_t)out, 0, (size_t)n_dst * 4, stream), "cudaMemsetAsync");
  if (n_src == 0) return J4B_OK;
  scatter_add_kernel<<<grid_for(n_src, dev), kThreads, 0, stream>>>(
      (const float*)(uintptr_t)a, n_src, (const int*)(uintptr_t)map, n_dst, (float*)(uintptr_t)out);
  J4B_CHECK_LAUNCH("scatter_add_kernel");
  return J4B_OK;
}

namespace j4b {
int launch_segment_sum(const float* a, const int64_t* offsets, const int64_t* sources, int64_t n_dst,
                       float* out, j4b_stream s) {
  if (n_dst == 0) return J4B_OK;
  J4B_DEVICE_OF(out);
  segment_sum_kernel<<<grid_for(n_dst, dev), kThreads, 0, stream>>>(a, offsets, sources, n_dst, out);
  J4B_CHECK_LAUNCH("segment_sum_kernel");
  return J4B_OK;
}
}  // namespace j4b

extern "C" int j4b_random_uniform(int64_t seed, int64_t counter, j4b_buf out, int64_t n,
                                  j4b_stream s) {
  if (n == 0) return J4B_OK;
  J4B_DEVICE_OF(out);
  random_kernel<<<grid_for(n, dev), kThreads, 0, stream>>>(0, seed, counter, (float*)(uintptr_t)out, n);
  J4B_CHECK_LAUNCH("random_kernel");
  return J4B_OK;
}

extern "C" int j4b_random_normal(int64_t seed, int64_t counter, j4b_buf out, int64_t n,
                                 j4b_stream s) {
  if (n == 0) return J4B_OK;
  J4B_DEVICE_OF(out);
  random_kernel<<<grid_for(n, dev), kThreads, 0, stream>>>(1, seed, counter, (float*)(uintptr_t)out, n);
  J4B_CHECK_LAUNCH("random_kernel");
  return J4B_OK;
}

namespace j4b {
// C (m x n) = A . B with A, B optionally transposed in place (ta: A given as [k, m]; tb: B given
// as [n, k]); batch >= 1 only for untransposed operands. precision as j4b_matmul.
int matmul_strided(const float* pa, const float* pb, float* pc, int64_t batch, int64_t m, int64_t k, int64_t n,
                   bool ta, bool tb, int precision, int dev, cudaStream_t stream) {
  // tensor cores (tcgen05): bf16 operands (1), or the 3-term bf16 split for fp32 accuracy (2, and
  // 0 when the contraction is large enough to amortise the operand conversion)
  const bool big = m * n * k >= (int64_t(1) << 24) && m >= 64 && n >= 64;
  if (precision == 1 || precision == 2 || big) {
    if (ta || tb) return tc_matmul_t(pa, pb, pc, m, k, n, ta, tb, precision == 1 ? 1 : 3, dev, stream);
    return tc_matmul(pa, pb, pc, batch, m, k, n, precision == 1 ? 1 : 3, dev, stream);
  }
  const int64_t sai = ta ? 1 : k, sap = ta ? m : 1, sbp = tb ? 1 : n, sbj = tb ? k : 1;
  if (k <= 32 && batch <= 65535 && (m * n + 255) / 256 <= INT32_MAX) {
    gemm_short_k_kernel<<<dim3((unsigned)((m * n + 255) / 256), (unsigned)batch), 256, 0, stream>>>(pa, pb, pc, m, k, n,
                                                                                                 sai, sap, sbp, sbj);
    J4B_CHECK_LAUNCH("gemm_short_k_kernel");
    return J4B_OK;
  }
  if (n <= 32 && batch <= 65535 && (m + 7) / 8 <= INT32_MAX) {
    gemm_narrow_n_kernel<<<dim3((unsigned)((m + 7) / 8), (unsigned)batch), 256, 0, stream>>>(pa, pb, pc, m, k, (int)n,
                                                                                          sai, sap, sbp, sbj);
    J4B_CHECK_LAUNCH("gemm_narrow_n_kernel");
    return J4B_OK;
  }
  dim3 grid((unsigned)((n + 63) / 64), (unsigned)((m + 63) / 64), (unsigned)batch);
  sgemm_kernel<<<grid, 256, 0, stream>>>(pa, pb, pc, m, k, n, sai, sap, sbp, sbj);
  J4B_CHECK_LAUNCH("sgemm_kernel");
  return J4B_OK;
}
}  // namespace j4b

extern "C" int j4b_matmul(j4b_buf a, j4b_buf b, j4b_buf out, int64_t batch, int64_t m, int64_t k,
                          int64_t n, int precision, j4b_stream s) {
  J4B_REQUIRE(batch >= 1 && m >= 1 && k >= 1 && n >= 1, "matmul dimensions must be positive");
  J4B_REQUIRE(precision >= 0 && precision <= 2, "matmul precision must be 0, 1 or 2");
  J4B_DEVICE_OF(out);
  return matmul_strided((const float*)(uintptr_t)a, (const float*)(uintptr_t)b, (float*)(uintptr_t)out, batch, m, k,
                        n, false, false, precision, dev, stream);
}

// ---------------------------------------------------------------------------------------------
// Full sum without any allocation.
//
// Some callers cannot allocate device memory when they reduce: hosts that reserve a fixed
// device-memory budget up front and forbid growth afterwards (a JVM that hands the engine a
// pre-sized arena and accounts for every byte of it), and serving loops that must not take the
// allocator's locks or risk an out-of-memory failure in the middle of a request. j4b_reduce_sum above
// allocates its block partials on every call; this variant keeps them in the static array below,
// which every GPU that loads the library holds until the process exits (512 KiB + 256 bytes).
//
// Layout of the array: one double per 2048-element chunk of the input (at most 65536 chunks,
// so at most 134,217,728 elements per call), then one 64-bit arrival counter. Each call rewrites
// the partials it uses; the counter must start at zero, is zeroed at set-up and is reset by the
// last block of every call. All calls share the array: calls that overlap on the GPU (on
// different streams, or from different threads without ordering) race and give wrong sums.
// ---------------------------------------------------------------------------------------------
namespace j4b {
namespace {

constexpr int64_t kNoallocChunk = 2048;      // elements per block (256 threads x 8)
constexpr int64_t kNoallocMaxChunks = 65536;  // partials the static array holds
static __device__ __align__(256) double g_reduce_noalloc_scratch[kNoallocMaxChunks + 32];

std::mutex g_noalloc_mu;
double* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the static scratch on `dev`, looked up (and its counter zeroed) on the first
// call for that device, with the device current.
int noalloc_scratch(int dev, cudaStream_t stream, double** out) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    J4B_CUDA(cudaGetSymbolAddress(&p, g_reduce_noalloc_scratch), "cudaGetSymbolAddress");
    J4B_CUDA(cudaMemsetAsync((double*)p + kNoallocMaxChunks, 0, sizeof(double), stream),
             "cudaMemsetAsync(reduce scratch counter)");
    g_noalloc_ptr[dev] = (double*)p;
  }
  *out = g_noalloc_ptr[dev];
  return J4B_OK;
}

__global__ void reduce_sum_noalloc_kernel(const float* __restrict__ a, int64_t n,
                                          double* __restrict__ scratch, float* __restrict__ out) {
  __shared__ double sh[32];
  __shared__ bool last;
  unsigned long long* counter = reinterpret_cast<unsigned long long*>(scratch + kNoallocMaxChunks);
  const int64_t base = (int64_t)blockIdx.x * kNoallocChunk;
  double acc = 0.0;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int64_t k = base + i * 256 + threadIdx.x;
    if (k < n) acc += a[k];
  }
  acc = warp_sum(acc);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sh[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double v = 0.0;
    for (int w = 0; w < 8; w++) v += sh[w];
    scratch[blockIdx.x] = v;
    __threadfence();
    last = atomicAdd(counter, 1ull) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // The last block folds the partials: thread t takes partials t, t+256, ... in order, then the
  // warps and the block combine in a fixed order, so the result does not depend on timing.
  double v = 0.0;
  for (int64_t b = threadIdx.x; b < gridDim.x; b += 256) v += __ldcg(scratch + b);
  v = warp_sum(v);
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    double total = 0.0;
    for (int w = 0; w < 8; w++) total += sh[w];
    out[0] = (float)total;
    *counter = 0ull;
  }
}

}  // namespace
}  // namespace j4b

extern "C" int j4b_reduce_sum_noalloc(j4b_buf a, int64_t n, j4b_buf out, j4b_stream s) {
  J4B_REQUIRE(n >= 0, "negative element count");
  J4B_REQUIRE(n <= kNoallocChunk * kNoallocMaxChunks,
              "reduce_sum_noalloc sums at most %lld elements (its static scratch holds %lld "
              "partials of %lld elements); got %lld",
              (long long)(kNoallocChunk * kNoallocMaxChunks), (long long)kNoallocMaxChunks,
              (long long)kNoallocChunk, (long long)n);
  J4B_DEVICE_OF(out);
  if (n > 0) J4B_SAME_DEVICE(a, "the input");
  double* scratch = nullptr;
  int st = noalloc_scratch(dev, stream, &scratch);
  if (st) return st;
  const int64_t chunks = n == 0 ? 1 : (n + kNoallocChunk - 1) / kNoallocChunk;
  reduce_sum_noalloc_kernel<<<(unsigned)chunks, 256, 0, stream>>>((const float*)(uintptr_t)a, n,
                                                                   scratch, (float*)(uintptr_t)out);
  J4B_CHECK_LAUNCH("reduce_sum_noalloc_kernel");
  return J4B_OK;
}
