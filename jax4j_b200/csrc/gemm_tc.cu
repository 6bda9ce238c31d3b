// Dense f32 matmul on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), the engine's
// ComputeBackend.matmul / batchedMatmul for shapes large enough to be real contractions
// (core/tensor/spi/ComputeBackend.java:97-101; the reference's CUDA backend runs 16x16 SIMT
// tiles, cuda/backend/cuda/CudaBackend.java:102-173, 572-623).
//
// C[M,N] = A[M,K] B[K,N], f32 row-major in and out. The operands are first rewritten as bf16,
// K-major (A as is, B transposed), K padded to the 64-element tile with zeros; for the
// fp32-accurate mode each operand is split into hi = bf16(x) and lo = bf16(x - hi) and the
// product is hi.hi + hi.lo + lo.hi (about 16 mantissa bits, relative error ~1e-5), for the bf16
// mode only hi.hi.
//
// One CTA computes one 128 x 256 (bf16 mode) or 128 x 128 (3-term mode) tile of C with six
// warps:
//   warp 0  one thread streams 64-wide K slices of the A and B tiles into a ring of
//           shared-memory stages with 2-D TMA tile loads (128-byte swizzle), completion counted
//           on the stage's `full` mbarrier;
//   warp 1  allocates 256 / 128 TMEM columns (the fp32 accumulator, one lane per tile row) and
//           one thread issues tcgen05.mma (M=128, N=256 / 128, K=16 each) from shared-memory
//           descriptors; tcgen05.commit releases each stage (`empty`) and finally signals the
//           epilogue (`acc_full`);
//   warps 2-5  read the accumulator with tcgen05.ld (32 lanes x 8 columns per load; warp w
//           may access TMEM lanes 32 (w % 4) .. + 31) and store C.
// Every mbarrier wait is bounded; a wait that gives up records an error in the status word.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <mutex>

#include "j4b_internal.h"
#include "j4b_wait.cuh"
#include "tc_common.cuh"

namespace j4b {
namespace {

constexpr int kBM = 128, kBK = 64;
// row tiles per rasterisation group (measured on the 16384 x 14336 x 4096 prefill projection:
// 16, 32 and 64 within 2% of each other; 32 and 64 slower on the fp32-accurate 128-wide tiles)
constexpr int kGroupM = 16;
constexpr int kTcThreads = 192;
constexpr int kTileBytes = kBM * kBK * 2;  // one 128 x 64 bf16 tile

// bf16 mode: 128 x 256 output tiles (A 16 KB + B 32 KB per stage), a 2-stage ring (96 KB) so two
// CTAs share an SM and one's prologue / epilogue overlaps the other's tensor work (TMEM: 2 x 256
// columns). 3-term mode: 128 x 128 tiles, 3 stages of four 16 KB tiles, one CTA per SM.
template <int TERMS>
constexpr int tc_bn() { return TERMS == 1 ? 256 : 128; }
template <int TERMS>
constexpr int tc_stages() { return TERMS == 1 ? 2 : 3; }
template <int TERMS>
constexpr uint32_t tc_stage_bytes() { return TERMS == 1 ? kTileBytes * 3 : kTileBytes * 4; }

struct TcArgs {
  int M, N, Kp;   // Kp: K padded to a multiple of 64
  int terms;      // 1: hi.hi (bf16 mode); 3: hi.hi + hi.lo + lo.hi (fp32-accurate mode)
  float* C;
  int64_t ldc;
  int* status;
};

template <int TERMS>
__global__ void __launch_bounds__(kTcThreads, TERMS == 1 ? 2 : 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap a_hi, const __grid_constant__ CUtensorMap a_lo,
                   const __grid_constant__ CUtensorMap b_hi, const __grid_constant__ CUtensorMap b_lo, TcArgs p) {
  constexpr int kBN = tc_bn<TERMS>();
  constexpr int kStages = tc_stages<TERMS>();
  constexpr uint32_t kStageBytes = tc_stage_bytes<TERMS>();
  constexpr uint32_t kBTile = (uint32_t)kBN * kBK * 2;  // B tile bytes
  extern __shared__ uint8_t smem_raw[];
  // 128-byte swizzled tiles need 1024-byte aligned bases
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Grouped rasterisation of the 1-D grid: tiles are taken in groups of kGroupM row tiles with the
  // row index fastest, so the CTAs resident at one time share a few A row panels and about
  // (resident / kGroupM) B column panels, which stay in L2 (row-major order would sweep all of
  // B's panels at once).
  int m_tile, n_tile;
  {
    const int mt = (p.M + kBM - 1) / kBM;
    const int nt = (p.N + kBN - 1) / kBN;
    const int per_group = kGroupM * nt;
    const int grp = (int)blockIdx.x / per_group, idx = (int)blockIdx.x % per_group;
    const int gm = min(kGroupM, mt - grp * kGroupM);
    m_tile = grp * kGroupM + idx % gm;
    n_tile = idx / gm;
  }
  const int m0 = m_tile * kBM, n0 = n_tile * kBN;
  const int nk = p.Kp / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      bar_init(&full[s], 1);
      bar_init(&empty[s], 1);
    }
    bar_init(acc_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tmem_slot)),
                 "r"(kBN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kStages, use = kb / kStages;
        if (use > 0 && !bar_wait(&empty[s], (uint32_t)((use - 1) & 1))) ok = false;
        uint8_t* st = smem + s * kStageBytes;
        bar_expect_tx(&full[s], kStageBytes);
        tma_tile(st, &a_hi, kb * kBK, m0, &full[s]);
        tma_tile(st + kTileBytes, &b_hi, kb * kBK, n0, &full[s]);
        if (TERMS == 3) {
          tma_tile(st + kTileBytes + kBTile, &a_lo, kb * kBK, m0, &full[s]);
          tma_tile(st + 2 * kTileBytes + kBTile, &b_lo, kb * kBK, n0, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(kBM, kBN);
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kStages;
        if (!bar_wait(&full[s], (uint32_t)((kb / kStages) & 1))) ok = false;
        tc_fence_after();
        const uint32_t st = saddr(smem + s * kStageBytes);
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {  // 16 bf16 = 32 bytes along the swizzled row
          const uint64_t ah = kmajor_sw128(st + k * 32), bh = kmajor_sw128(st + kTileBytes + k * 32);
          umma_bf16(tmem, ah, bh, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          if (TERMS == 3) {
            const uint64_t al = kmajor_sw128(st + kTileBytes + kBTile + k * 32);
            const uint64_t bl = kmajor_sw128(st + 2 * kTileBytes + kBTile + k * 32);
            umma_bf16(tmem, ah, bl, idesc, 1u);
            umma_bf16(tmem, al, bh, idesc, 1u);
          }
        }
        umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
      }
      umma_commit(acc_full);
    }
  } else {
    // epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 = tile rows
    const int quarter = warp & 3;
    const int row = m0 + quarter * 32 + lane;
    if (!bar_wait(acc_full, 0)) ok = false;
    tc_fence_after();
    const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16);
    float* crow = p.C + (int64_t)row * p.ldc;
#pragma unroll 1
    for (int c = 0; c < kBN; c += 8) {
      uint32_t v[8];
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
          : "r"(taddr + (uint32_t)c));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      const int col = n0 + c;
      if (row < p.M) {
        if (col + 8 <= p.N && (p.ldc & 3) == 0 && (reinterpret_cast<uintptr_t>(p.C) & 15) == 0) {
          float4* dst = reinterpret_cast<float4*>(crow + col);
          dst[0] = make_float4(__uint_as_float(v[0]), __uint_as_float(v[1]), __uint_as_float(v[2]), __uint_as_float(v[3]));
          dst[1] = make_float4(__uint_as_float(v[4]), __uint_as_float(v[5]), __uint_as_float(v[6]), __uint_as_float(v[7]));
        } else {
#pragma unroll
          for (int u = 0; u < 8; ++u)
            if (col + u < p.N) crow[col + u] = __uint_as_float(v[u]);
        }
      }
    }
  }
  if (!ok) atomicExch(p.status, 1);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kBN));
  }
}

// f32 [rows, cols] (row stride ld) -> bf16 hi (and lo) [rows, kp], zero-padded columns. One
// thread per 8 consecutive columns of a row (blockIdx.y strides the rows): one 16-byte store.
__global__ void split_rows_kernel(const float* __restrict__ src, int64_t rows, int64_t cols, int64_t ld,
                                  int64_t kp, __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
  const int64_t c0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c0 >= kp) return;
  const bool vec = (ld % 4) == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0 && c0 + 8 <= cols;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const float* s = src + r * ld + c0;
    float v[8];
    if (vec) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(s));
      const float4 b = __ldg(reinterpret_cast<const float4*>(s) + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = c0 + u < cols ? s[u] : 0.0f;
    }
    alignas(16) __nv_bfloat16 h8[8], l8[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      h8[u] = __float2bfloat16_rn(v[u]);
      l8[u] = __float2bfloat16_rn(v[u] - __bfloat162float(h8[u]));
    }
    *reinterpret_cast<uint4*>(hi + r * kp + c0) = *reinterpret_cast<const uint4*>(h8);
    if (lo) *reinterpret_cast<uint4*>(lo + r * kp + c0) = *reinterpret_cast<const uint4*>(l8);
  }
}

// f32 B [k, n] -> bf16 B^T hi (and lo) [n, kp] through 32 x 32 shared-memory tiles.
__global__ void split_transpose_kernel(const float* __restrict__ b, int64_t k, int64_t n, int64_t kp,
                                       __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
  __shared__ float tile[32][33];
  const int64_t k0 = (int64_t)blockIdx.x * 32, n0 = (int64_t)blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int64_t kk = k0 + r, nn = n0 + threadIdx.x;
    tile[r][threadIdx.x] = (kk < k && nn < n) ? b[kk * n + nn] : 0.0f;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int64_t nn = n0 + r, kk = k0 + threadIdx.x;
    if (nn < n && kk < kp) {
      const float v = tile[threadIdx.x][r];
      const __nv_bfloat16 h = __float2bfloat16_rn(v);
      hi[nn * kp + kk] = h;
      if (lo) lo[nn * kp + kk] = __float2bfloat16_rn(v - __bfloat162float(h));
    }
  }
}

int* tc_status(int dev) {
  static int* status[kMaxDevices] = {};
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  if (!status[dev]) {
    if (cudaMalloc(&status[dev], sizeof(int)) != cudaSuccess) return nullptr;
    cudaMemset(status[dev], 0, sizeof(int));
  }
  return status[dev];
}

template <int TERMS>
cudaError_t launch_tc(const CUtensorMap& ah, const CUtensorMap& al, const CUtensorMap& bh, const CUtensorMap& bl,
                      const TcArgs& a, cudaStream_t stream) {
  constexpr int kStages = tc_stages<TERMS>();
  constexpr int kBN = tc_bn<TERMS>();
  const size_t smem = (size_t)kStages * tc_stage_bytes<TERMS>() + 1024 + 256;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<TERMS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const int64_t tiles = (int64_t)((a.N + kBN - 1) / kBN) * ((a.M + kBM - 1) / kBM);
  if (tiles > 0x7fffffffLL) return cudaErrorInvalidValue;
  tc_gemm_kernel<TERMS><<<(unsigned)tiles, kTcThreads, smem, stream>>>(ah, al, bh, bl, a);
  return cudaGetLastError();
}

}  // namespace

// C (m x n, row stride n) = A . Bt^T with both operands already bf16 hi (and lo, terms 3),
// K-major [m, kp] and [n, kp], kp a multiple of 64 with zero padding.
int tc_gemm_bf16(const __nv_bfloat16* a_hi, const __nv_bfloat16* a_lo, int64_t m, int64_t kp,
                 const __nv_bfloat16* bt_hi, const __nv_bfloat16* bt_lo, int64_t n, int terms, float* out, int dev,
                 cudaStream_t stream) {
  if (m == 0 || n == 0) return J4B_OK;
  if (kp % kBK) return set_error(J4B_EINVAL, "tensor-core operand width %lld is not a multiple of %d", (long long)kp, kBK);
  int* status = tc_status(dev);
  if (!status) return set_error(J4B_ENOMEM, "tensor-core status word allocation failed");
  const bool split = terms == 3;
  CUtensorMap mah, mal, mbh, mbl;
  const int bn = split ? tc_bn<3>() : tc_bn<1>();
  if (!make_map(&mah, a_hi, m, kp, kBM) || !make_map(&mbh, bt_hi, n, kp, bn) ||
      (split && (!make_map(&mal, a_lo, m, kp, kBM) || !make_map(&mbl, bt_lo, n, kp, bn))))
    return set_error(J4B_ECUDA, "cuTensorMapEncodeTiled failed for the matmul operands");
  if (!split) {
    mal = mah;
    mbl = mbh;
  }
  TcArgs args;
  args.M = (int)m;
  args.N = (int)n;
  args.Kp = (int)kp;
  args.terms = terms;
  args.C = out;
  args.ldc = n;
  args.status = status;
  cudaError_t e = split ? launch_tc<3>(mah, mal, mbh, mbl, args, stream) : launch_tc<1>(mah, mal, mbh, mbl, args, stream);
  if (e != cudaSuccess) return cuda_error(e, "tc_gemm_kernel");
  count_launch(1);
  return J4B_OK;
}

// f32 [rows, cols] (row stride ld) -> bf16 hi (and lo) [rows, kp] with zero-padded columns.
int tc_split_rows(const float* src, int64_t rows, int64_t cols, int64_t ld, int64_t kp, __nv_bfloat16* hi,
                  __nv_bfloat16* lo, cudaStream_t stream) {
  dim3 grid((unsigned)((kp / 8 + 127) / 128), (unsigned)std::min<int64_t>(rows, 65535));
  split_rows_kernel<<<grid, 128, 0, stream>>>(src, rows, cols, ld, kp, hi, lo);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "split_rows_kernel");
  count_launch(1);
  return J4B_OK;
}

// C (m x n, row stride n) = A (m x k, f32 row-major) . Bt^T, with Bt given as bf16 hi (and lo)
// [n, kp] K-major (kp = k rounded up to 64, zero-padded). A is converted here.
int tc_gemm_bt(const float* a, int64_t m, int64_t k, const __nv_bfloat16* bt_hi, const __nv_bfloat16* bt_lo,
               int64_t n, int terms, float* out, int dev, cudaStream_t stream) {
  if (m == 0 || n == 0) return J4B_OK;
  const int64_t kp = (k + kBK - 1) / kBK * kBK;
  const bool split = terms == 3;
  const size_t abytes = (size_t)(m * kp) * 2;
  void* scratch = nullptr;
  J4B_CUDA(cudaMallocAsync(&scratch, 2 * abytes + 512, stream), "cudaMallocAsync(matmul operand)");
  __nv_bfloat16* ahi = (__nv_bfloat16*)scratch;
  __nv_bfloat16* alo = split ? (__nv_bfloat16*)((uint8_t*)scratch + ((abytes + 255) & ~size_t(255))) : nullptr;
  int rc = tc_split_rows(a, m, k, k, kp, ahi, alo, stream);
  if (rc == J4B_OK) rc = tc_gemm_bf16(ahi, alo, m, kp, bt_hi, bt_lo, n, terms, out, dev, stream);
  cudaFreeAsync(scratch, stream);
  return rc;
}

// C[b] = A[b] (m x k) . B[b] (k x n) on tcgen05; terms 1 (bf16 operands) or 3 (fp32-accurate).
int tc_matmul(const float* a, const float* b, float* out, int64_t batch, int64_t m, int64_t k, int64_t n,
              int terms, int dev, cudaStream_t stream) {
  if (m == 0 || n == 0) return J4B_OK;
  if (k == 0) {
    J4B_CUDA(cudaMemsetAsync(out, 0, (size_t)(batch * m * n) * 4, stream), "cudaMemsetAsync");
    return J4B_OK;
  }
  if (m > INT32_MAX / 2 || n > INT32_MAX / 2 || k > INT32_MAX / 2)
    return set_error(J4B_EINVAL, "matmul dimension too large for the tensor-core path");
  const int64_t kp = (k + kBK - 1) / kBK * kBK;
  const bool split = terms == 3;
  const size_t bbytes = (size_t)(n * kp) * 2;
  void* scratch = nullptr;
  J4B_CUDA(cudaMallocAsync(&scratch, 2 * bbytes + 512, stream), "cudaMallocAsync(matmul operand)");
  __nv_bfloat16* bhi = (__nv_bfloat16*)scratch;
  __nv_bfloat16* blo = split ? (__nv_bfloat16*)((uint8_t*)scratch + ((bbytes + 255) & ~size_t(255))) : nullptr;
  int rc = J4B_OK;
  for (int64_t bi = 0; bi < batch && rc == J4B_OK; ++bi) {
    dim3 tg((unsigned)((kp + 31) / 32), (unsigned)((n + 31) / 32));
    split_transpose_kernel<<<tg, dim3(32, 8), 0, stream>>>(b + bi * k * n, k, n, kp, bhi, blo);
    count_launch(1);
    rc = tc_gemm_bt(a + bi * m * k, m, k, bhi, blo, n, terms, out + bi * m * n, dev, stream);
  }
  cudaFreeAsync(scratch, stream);
  return rc;
}

// op(A) . op(B): each operand converted to its bf16 K-major form straight from its stored layout
// (A [m, k] rows or A^T stored [k, m] through the transposing split; B likewise), so a transpose
// feeding a matmul is never materialised.
int tc_matmul_t(const float* a, const float* b, float* out, int64_t m, int64_t k, int64_t n, bool ta, bool tb,
                int terms, int dev, cudaStream_t stream) {
  if (m == 0 || n == 0) return J4B_OK;
  if (k == 0) {
    J4B_CUDA(cudaMemsetAsync(out, 0, (size_t)(m * n) * 4, stream), "cudaMemsetAsync");
    return J4B_OK;
  }
  if (m > INT32_MAX / 2 || n > INT32_MAX / 2 || k > INT32_MAX / 2)
    return set_error(J4B_EINVAL, "matmul dimension too large for the tensor-core path");
  const int64_t kp = (k + kBK - 1) / kBK * kBK;
  const bool split = terms == 3;
  const size_t abytes = (size_t)(m * kp) * 2, bbytes = (size_t)(n * kp) * 2;
  const size_t aspan = (abytes + 255) & ~size_t(255), bspan = (bbytes + 255) & ~size_t(255);
  void* scratch = nullptr;
  J4B_CUDA(cudaMallocAsync(&scratch, 2 * aspan + 2 * bspan + 256, stream), "cudaMallocAsync(matmul operands)");
  __nv_bfloat16* ahi = (__nv_bfloat16*)scratch;
  __nv_bfloat16* alo = split ? (__nv_bfloat16*)((uint8_t*)scratch + aspan) : nullptr;
  __nv_bfloat16* bhi = (__nv_bfloat16*)((uint8_t*)scratch + 2 * aspan);
  __nv_bfloat16* blo = split ? (__nv_bfloat16*)((uint8_t*)scratch + 2 * aspan + bspan) : nullptr;
  int rc = J4B_OK;
  if (ta) {  // stored [k, m] -> [m, kp]
    split_transpose_kernel<<<dim3((unsigned)((kp + 31) / 32), (unsigned)((m + 31) / 32)), dim3(32, 8), 0, stream>>>(
        a, k, m, kp, ahi, alo);
    count_launch(1);
  } else {
    rc = tc_split_rows(a, m, k, k, kp, ahi, alo, stream);
  }
  if (rc == J4B_OK) {
    if (tb) {  // stored [n, k] -> [n, kp]
      rc = tc_split_rows(b, n, k, k, kp, bhi, blo, stream);
    } else {  // stored [k, n] -> [n, kp]
      split_transpose_kernel<<<dim3((unsigned)((kp + 31) / 32), (unsigned)((n + 31) / 32)), dim3(32, 8), 0, stream>>>(
          b, k, n, kp, bhi, blo);
      count_launch(1);
    }
  }
  if (rc == J4B_OK) rc = tc_gemm_bf16(ahi, alo, m, kp, bhi, blo, n, terms, out, dev, stream);
  cudaFreeAsync(scratch, stream);
  return rc;
}

int tc_status_read(int dev, int* value) {
  int* st = tc_status(dev);
  if (!st) return set_error(J4B_ENOMEM, "status");
  J4B_CUDA(cudaMemcpy(value, st, sizeof(int), cudaMemcpyDeviceToHost), "cudaMemcpy(status)");
  return J4B_OK;
}

}  // namespace j4b
