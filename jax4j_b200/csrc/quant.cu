// GGUF block-quantised matrices: upload + repack, batched dequant-GEMV, bit-exact row gather and
// a device-side encoder.
//
// Reference interface: core/tensor/spi/QuantizedOps.java:19-34, CPU semantics in
// core/backend/cpu/CpuBackend.java:690-755, CpuQ4Gemm.java:17-77, CpuQ2Gemm.java:17-83. The
// reference has no GPU quantised path; Q8_0 and Q4_K have no implementation at all there
// (core/tensor/QuantType.java:8-9 only) and follow the public GGUF block layouts.
//
// Device layout ("fragment-major repack", same byte count as the GGUF blob):
//   A weight of R rows x K columns is cut into row tiles of 16 rows. Inside a row tile, every
//   group of 32 columns (one Q8_0/Q4_0 block, one Q4_K sub-block, a quarter Q2_0 block) holds
//   exactly the bytes lane l of a warp needs to build its mma.m16n8k16 A fragments for those 32
//   columns, stored contiguously in lane order, so a warp streams its tile with fully coalesced
//   128-bit loads. Per-row scales live in a separate plane in the same tile order. Padding rows
//   and columns carry zero scales.
//
// GEMV: y[b, r] = sum_k W[r, k] x[b, k] (+ add[b, r]). Codes are expanded in registers to fp16
// "magic" values that are exact (Q8_0: the integer code; 4-bit codes: 1 + q/16; 2-bit codes:
// 1 + c/4), x is split into fp16 hi + lo parts (x = hi + lo to ~2^-22 relative), products are
// accumulated by the tensor cores in fp32 per 32-column block, and the per-block scale (and the
// 1 + q/16 offset, via precomputed block sums of x) is applied in fp32 on the block partials.
// Accuracy: normwise relative error ~1e-6, inside the 1e-4 fp32-accumulate bar.
//
// Work split: a CTA of 8 warps owns one K range of 1024 columns (8 warp chunks of 128) and a run
// of row tiles; each warp keeps its chunk's x fragments in registers for the whole run. Warp
// partials are summed in shared memory; K ranges are combined by the last CTA to finish a row
// tile (per-tile arrival counter, partials in per-weight scratch), which also applies `add`.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "j4b_internal.h"

struct j4b_qweight {
  int dev;
  int type;
  int64_t rows, cols;
  int64_t rt;     // row tiles of 16
  int64_t kpad;   // K rounded up to the 128-column warp chunk
  int ksplit;     // K ranges of 1024 columns
  uint8_t* quants;
  uint8_t* meta;
  size_t quant_bytes, meta_bytes;
  float* partials;     // [ksplit][rt][256] split-K scratch
  unsigned* arrivals;  // [rt] arrival counters, zero between launches
};

namespace j4b {
namespace {

constexpr int kWarpCols = 128;           // columns per warp chunk
constexpr int kWarps = 8;                // warps per CTA
constexpr int kCtaCols = kWarpCols * kWarps;

__host__ __device__ inline int block_elems(int t) {
  switch (t) {
    case J4B_Q4_0: case J4B_Q8_0: return 32;
    case J4B_Q4_K: return 256;
    case J4B_Q2_0: return 128;
  }
  return -1;
}
__host__ __device__ inline int block_bytes(int t) {
  switch (t) {
    case J4B_Q4_0: return 18;
    case J4B_Q8_0: return 34;
    case J4B_Q4_K: return 144;
    case J4B_Q2_0: return 34;
  }
  return -1;
}

// ---------------------------------------------------------------------------------------------
// fragment geometry: element e (0..7) of lane l's A fragment for one 16-column k-step
// ---------------------------------------------------------------------------------------------
__host__ __device__ inline int frag_row(int lane, int e) { return (lane >> 2) + 8 * ((e >> 1) & 1); }
__host__ __device__ inline int frag_col(int lane, int e) { return 2 * (lane & 3) + (e & 1) + 8 * (e >> 2); }

// Bit position of element e's nibble inside a lane's 32-bit word (4-bit formats): pair i = e/2
// lives at bits 6+4i (first) and 22+4i (second), modulo 32, so that rotating right by 4i and
// masking 0x03C003C0 drops both nibbles into the fp16 mantissa bits 6..9.
__host__ __device__ inline int nib_pos(int e) {
  int i = e >> 1;
  return ((e & 1) ? 22 + 4 * i : 6 + 4 * i) & 31;
}
// 2-bit codes: pair p (0..7) at bits 8+2p and 24+2p modulo 32 (rotate by 2p, mask 0x03000300).
__host__ __device__ inline int crumb_pos(int p, int second) { return (second ? 24 + 2 * p : 8 + 2 * p) & 31; }

__device__ inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
// Rotations: a 4-bit field at bit 30 wraps into bits 0..1.
__host__ __device__ inline uint32_t rotl32(uint32_t v, int s) { return s ? (v << s) | (v >> (32 - s)) : v; }
__host__ __device__ inline uint32_t rotr32(uint32_t v, int s) { return s ? (v >> s) | (v << (32 - s)) : v; }

__device__ inline void q4k_scale_min(int j, const uint8_t* q, int* sc, int* m) {
  if (j < 4) {
    *sc = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// Raw code of GGUF element (row r, column k); returns false outside the matrix.
__device__ inline int raw_code(int type, const uint8_t* blob, int64_t rows, int64_t cols, int64_t r,
                               int64_t k, bool* inside) {
  *inside = r < rows && k < cols;
  if (!*inside) return 0;
  int be = block_elems(type), bb = block_bytes(type);
  const uint8_t* blk = blob + (r * (cols / be) + k / be) * bb;
  int w = (int)(k % be);
  switch (type) {
    case J4B_Q8_0: return (int)(int8_t)blk[2 + w];
    case J4B_Q4_0: return w < 16 ? (blk[2 + w] & 0xF) : (blk[2 + w - 16] >> 4);
    case J4B_Q2_0: return (blk[2 + w / 4] >> ((w & 3) * 2)) & 3;
    case J4B_Q4_K: {
      int c = w / 64, h = (w % 64) / 32, l = w % 32;
      int b = blk[16 + 32 * c + l];
      return h ? (b >> 4) : (b & 0xF);
    }
  }
  return 0;
}

// ---------------------------------------------------------------------------------------------
// repack kernels
// ---------------------------------------------------------------------------------------------

// One thread per (row tile, 32-column group, lane): writes that lane's quant bytes.
__global__ void repack_quants_kernel(int type, const uint8_t* __restrict__ blob, int64_t rows,
                                     int64_t cols, int64_t rt, int64_t kpad,
                                     uint8_t* __restrict__ out) {
  int64_t groups = kpad / 32;
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rt * groups * 32) return;
  int lane = (int)(idx % 32);
  int64_t grp = (idx / 32) % groups;
  int64_t tile = idx / 32 / groups;
  int64_t r0 = tile * 16, k0 = grp * 32;
  bool in;
  if (type == J4B_Q8_0) {
    // [tile][grp][lane][16 bytes]: kstep ks, element e at byte 8*ks + e, value q ^ 0x80.
    uint8_t bytes[16];
    for (int ks = 0; ks < 2; ks++)
      for (int e = 0; e < 8; e++) {
        int q = raw_code(type, blob, rows, cols, r0 + frag_row(lane, e), k0 + 16 * ks + frag_col(lane, e), &in);
        bytes[8 * ks + e] = (uint8_t)((q & 0xFF) ^ 0x80);
      }
    uint8_t* dst = out + ((tile * groups + grp) * 32 + lane) * 16;
    for (int i = 0; i < 16; i++) dst[i] = bytes[i];
  } else if (type == J4B_Q4_0 || type == J4B_Q4_K) {
    // Two 32-bit words (k-steps 0, 1) per lane per group. Q4_0 groups are paired into one
    // 16-byte line per lane ([tile][grp/2][lane][grp&1][8 bytes]); Q4_K half super-blocks of 4
    // groups form one 32-byte line per lane ([tile][grp/4][lane][grp&3][8 bytes]).
    uint32_t words[2] = {0, 0};
    for (int ks = 0; ks < 2; ks++)
      for (int e = 0; e < 8; e++) {
        int q = raw_code(type, blob, rows, cols, r0 + frag_row(lane, e), k0 + 16 * ks + frag_col(lane, e), &in);
        words[ks] |= rotl32((uint32_t)(q & 0xF), nib_pos(e));
      }
    int per_line = type == J4B_Q4_0 ? 2 : 4;
    int64_t line = grp / per_line;
    int slot = (int)(grp % per_line);
    uint32_t* dst = (uint32_t*)(out + ((tile * (groups / per_line) + line) * 32 + lane) * (8 * per_line) + 8 * slot);
    dst[0] = words[0];
    dst[1] = words[1];
  } else if (type == J4B_Q2_0) {
    // One word per lane per group; the 4 groups of a 128-block form one 16-byte line.
    uint32_t word = 0;
    for (int ks = 0; ks < 2; ks++)
      for (int e = 0; e < 8; e++) {
        int c = raw_code(type, blob, rows, cols, r0 + frag_row(lane, e), k0 + 16 * ks + frag_col(lane, e), &in);
        if (!in) c = 1;  // padding decodes to 0
        word |= rotl32((uint32_t)(c & 3), crumb_pos(4 * ks + (e >> 1), e & 1));
      }
    int64_t line = grp / 4;
    int slot = (int)(grp % 4);
    uint32_t* dst = (uint32_t*)(out + ((tile * (groups / 4) + line) * 32 + lane) * 16 + 4 * slot);
    dst[0] = word;
  }
}

// Scale planes. Q8_0/Q4_0/Q2_0: [tile][block][8 groups][2 halves: row g, row g+8].
// Q4_K: [tile][super-block][8 groups][2 rows][16 bytes: d, dmin, 12 packed scale bytes].
__global__ void repack_meta_kernel(int type, const uint8_t* __restrict__ blob, int64_t rows,
                                   int64_t cols, int64_t rt, int64_t kpad,
                                   uint8_t* __restrict__ out) {
  int be = block_elems(type), bb = block_bytes(type);
  int64_t blocks = kpad / be;
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // (tile, block, row-in-tile)
  if (idx >= rt * blocks * 16) return;
  int rr = (int)(idx % 16);
  int64_t blk = (idx / 16) % blocks;
  int64_t tile = idx / 16 / blocks;
  int64_t r = tile * 16 + rr;
  bool in = r < rows && blk * be < cols;
  const uint8_t* src = in ? blob + (r * (cols / be) + blk) * bb : nullptr;
  int g = rr & 7, which = rr >> 3;
  if (type == J4B_Q4_K) {
    uint8_t* dst = out + (((tile * blocks + blk) * 8 + g) * 2 + which) * 16;
    for (int i = 0; i < 16; i++) dst[i] = in ? src[i] : 0;
  } else {
    uint8_t* dst = out + (((tile * blocks + blk) * 8 + g) * 2 + which) * 2;
    dst[0] = in ? src[0] : 0;
    dst[1] = in ? src[1] : 0;
  }
}

// ---------------------------------------------------------------------------------------------
// bit-exact gather (quantGatherRow) from the repacked layout
// ---------------------------------------------------------------------------------------------
__device__ inline int repacked_code(const j4b_qweight& w, int64_t r, int64_t k) {
  int64_t tile = r / 16;
  int rr = (int)(r % 16);
  int64_t grp = k / 32, groups = w.kpad / 32;
  int kk = (int)(k % 32), ks = kk / 16, k16 = kk % 16;
  int g = rr & 7, hi8 = rr >> 3;
  int t = (k16 & 7) >> 1;
  int lane = 4 * g + t;
  int e = (k16 & 1) + 2 * hi8 + 4 * (k16 >> 3);
  if (w.type == J4B_Q8_0) {
    const uint8_t* p = w.quants + ((tile * groups + grp) * 32 + lane) * 16;
    return (int)(int8_t)(p[8 * ks + e] ^ 0x80);
  }
  if (w.type == J4B_Q4_0 || w.type == J4B_Q4_K) {
    int per_line = w.type == J4B_Q4_0 ? 2 : 4;
    const uint32_t* p = (const uint32_t*)(w.quants + ((tile * (groups / per_line) + grp / per_line) * 32 + lane) * (8 * per_line) + 8 * (grp % per_line));
    return rotr32(p[ks], nib_pos(e)) & 0xF;
  }
  const uint32_t* p = (const uint32_t*)(w.quants + ((tile * (groups / 4) + grp / 4) * 32 + lane) * 16 + 4 * (grp % 4));
  return rotr32(p[0], crumb_pos(4 * ks + (e >> 1), e & 1)) & 3;
}

__global__ void gather_row_kernel(j4b_qweight w, int64_t row, float* __restrict__ out) {
  int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= w.cols) return;
  int64_t tile = row / 16;
  int rr = (int)(row % 16), g = rr & 7, which = rr >> 3;
  int q = repacked_code(w, row, k);
  float v;
  if (w.type == J4B_Q4_K) {
    int64_t sb = k / 256;
    const uint8_t* m = w.meta + (((tile * (w.kpad / 256) + sb) * 8 + g) * 2 + which) * 16;
    float d = __half2float(__ushort_as_half(rd16(m)));
    float dmin = __half2float(__ushort_as_half(rd16(m + 2)));
    int j = (int)((k % 256) / 32), sc, mn;
    q4k_scale_min(j, m + 4, &sc, &mn);
    float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)mn);
    v = __fsub_rn(__fmul_rn(d1, (float)q), m1);  // d1*q is exact; one rounding, as the oracle
  } else {
    int be = block_elems(w.type);
    int64_t blk = k / be;
    const uint8_t* m = w.meta + (((tile * (w.kpad / be) + blk) * 8 + g) * 2 + which) * 2;
    float d = __half2float(__ushort_as_half(rd16(m)));
    int code = w.type == J4B_Q8_0 ? q : (w.type == J4B_Q4_0 ? q - 8 : q - 1);
    v = __fmul_rn(d, (float)code);
  }
  out[k] = v;
}

// ---------------------------------------------------------------------------------------------
// GEMV
// ---------------------------------------------------------------------------------------------
struct GemvArgs {
  const uint8_t* quants;
  const uint8_t* meta;
  int64_t rows, cols, kpad, rt;
  const float* x;
  const float* add;
  float* y;
  int batch;  // batch rows handled by this launch (<= 8 * NT)
  int ksplit;
  int tiles_per_cta;
  float* partials;
  unsigned* arrivals;
};

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t rotr(uint32_t v, int s) { return __funnelshift_r(v, v, s); }
__device__ __forceinline__ uint32_t lop_or(uint32_t v, uint32_t mask, uint32_t bias) {
  return (v & mask) | bias;
}
__device__ __forceinline__ uint32_t h2sub(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// Q8_0: 4 bytes (a0..a3 or a4..a7) -> two half2 holding the exact integer codes.
__device__ __forceinline__ void q8_pairs(uint32_t w, uint32_t& p0, uint32_t& p1) {
  const uint32_t kBias = 0x64806480u;  // half2(1152, 1152): 1024 + the 0x80 code offset
  p0 = h2sub(__byte_perm(w, 0x64646464u, 0x4140), kBias);
  p1 = h2sub(__byte_perm(w, 0x64646464u, 0x4342), kBias);
}
// 4-bit: one word -> four half2 of (1 + q/16).
__device__ __forceinline__ void q4_pairs(uint32_t w, uint32_t (&a)[4]) {
  const uint32_t kMask = 0x03C003C0u, kOne = 0x3C003C00u;
  a[0] = lop_or(w, kMask, kOne);
  a[1] = lop_or(rotr(w, 4), kMask, kOne);
  a[2] = lop_or(rotr(w, 8), kMask, kOne);
  a[3] = lop_or(rotr(w, 12), kMask, kOne);
}
// 2-bit: one word -> eight half2 of (1 + c/4); pairs 0..3 are k-step 0, 4..7 k-step 1.
__device__ __forceinline__ uint32_t q2_pair(uint32_t w, int p) {
  return lop_or(rotr(w, 2 * p), 0x03000300u, 0x3C003C00u);
}

template <int QT, int NT>
__global__ void __launch_bounds__(256, 2) qgemv_kernel(GemvArgs a) {
  __shared__ float red[2][kWarps][NT * 4][32];
  __shared__ int last_flag;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int split = blockIdx.x % a.ksplit;
  const int64_t tile0 = (int64_t)(blockIdx.x / a.ksplit) * a.tiles_per_cta;
  const int64_t tile1 = min(tile0 + a.tiles_per_cta, a.rt);
  const int64_t k0 = (int64_t)split * kCtaCols + warp * kWarpCols;
  const bool active = k0 < a.kpad;
  const int groups_total = (int)(a.kpad / 32);

  // ---- x fragments of this warp's 128-column chunk: hi/lo fp16, per n-tile and k-step ----
  uint32_t bh[NT][8][2], bl[NT][8][2];
  float xs[NT][8];  // per-lane partial sums of x over its fragment columns, per 16-col k-step
#pragma unroll
  for (int n = 0; n < NT; n++) {
    const int b = 8 * n + g;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      const int64_t k = k0 + 16 * j + 2 * t;
      if (active && b < a.batch) {
        const float* xr = a.x + (int64_t)b * a.cols;
        if (k < a.cols) {
          float2 p = *reinterpret_cast<const float2*>(xr + k);
          v[0] = p.x;
          v[1] = p.y;
        }
        if (k + 8 < a.cols) {
          float2 p = *reinterpret_cast<const float2*>(xr + k + 8);
          v[2] = p.x;
          v[3] = p.y;
        }
      }
      __half2 h0 = __floats2half2_rn(v[0], v[1]);
      __half2 h1 = __floats2half2_rn(v[2], v[3]);
      float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
      __half2 l0 = __floats2half2_rn(v[0] - f0.x, v[1] - f0.y);
      __half2 l1 = __floats2half2_rn(v[2] - f1.x, v[3] - f1.y);
      bh[n][j][0] = *reinterpret_cast<uint32_t*>(&h0);
      bh[n][j][1] = *reinterpret_cast<uint32_t*>(&h1);
      bl[n][j][0] = *reinterpret_cast<uint32_t*>(&l0);
      bl[n][j][1] = *reinterpret_cast<uint32_t*>(&l1);
      float2 g0 = __half22float2(l0), g1 = __half22float2(l1);
      xs[n][j] = (f0.x + g0.x) + (f0.y + g0.y) + (f1.x + g1.x) + (f1.y + g1.y);
    }
  }
  // Block sums of x for the output columns this lane holds (batch 2t, 2t+1 of each n-tile).
  // Q4_0 / Q4_K: per 32-col block (4 per chunk); Q2_0: one 128-col block.
  constexpr int kXB = (QT == J4B_Q2_0) ? 1 : 4;
  float xblk[NT][kXB][2];
  if constexpr (QT != J4B_Q8_0) {
#pragma unroll
    for (int n = 0; n < NT; n++) {
#pragma unroll
      for (int q = 0; q < kXB; q++) {
        float s = 0.f;
        constexpr int kSteps = 8 / kXB;
#pragma unroll
        for (int j = 0; j < kSteps; j++) s += xs[n][q * kSteps + j];
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);  // block sum of x for batch 8n+g
        xblk[n][q][0] = __shfl_sync(0xffffffffu, s, 4 * (2 * t));
        xblk[n][q][1] = __shfl_sync(0xffffffffu, s, 4 * (2 * t + 1));
      }
    }
  }

  int buf = 0;
  for (int64_t tile = tile0; tile < tile1; tile++) {
    float acc[NT][4];
#pragma unroll
    for (int n = 0; n < NT; n++) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;

    if (active) {
      const int64_t gbase = tile * groups_total + k0 / 32;  // first 32-col group of the chunk
      if constexpr (QT == J4B_Q8_0) {
        const uint4* qp = reinterpret_cast<const uint4*>(a.quants + (gbase * 32) * 16) ;
        uint4 line[4];
        uint32_t sc[4];
#pragma unroll
        for (int q = 0; q < 4; q++) line[q] = __ldg(qp + q * 32 + lane);
#pragma unroll
        for (int q = 0; q < 4; q++)
          sc[q] = __ldg(reinterpret_cast<const uint32_t*>(a.meta + ((gbase + q) * 8 + g) * 4));
#pragma unroll
        for (int q = 0; q < 4; q++) {
          float tmp[NT][4];
#pragma unroll
          for (int n = 0; n < NT; n++) tmp[n][0] = tmp[n][1] = tmp[n][2] = tmp[n][3] = 0.f;
          const uint32_t wv[4] = {line[q].x, line[q].y, line[q].z, line[q].w};
#pragma unroll
          for (int ks = 0; ks < 2; ks++) {
            uint32_t a0, a1, a2, a3;
            q8_pairs(wv[2 * ks], a0, a1);
            q8_pairs(wv[2 * ks + 1], a2, a3);
            const int j = 2 * q + ks;
#pragma unroll
            for (int n = 0; n < NT; n++) {
              mma16816(tmp[n], a0, a1, a2, a3, bh[n][j][0], bh[n][j][1]);
              mma16816(tmp[n], a0, a1, a2, a3, bl[n][j][0], bl[n][j][1]);
            }
          }
          const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&sc[q]));
#pragma unroll
          for (int n = 0; n < NT; n++) {
            acc[n][0] = fmaf(d.x, tmp[n][0], acc[n][0]);
            acc[n][1] = fmaf(d.x, tmp[n][1], acc[n][1]);
            acc[n][2] = fmaf(d.y, tmp[n][2], acc[n][2]);
            acc[n][3] = fmaf(d.y, tmp[n][3], acc[n][3]);
          }
        }
      } else if constexpr (QT == J4B_Q4_0) {
        const uint4* qp = reinterpret_cast<const uint4*>(a.quants + gbase * 32 * 8);
        uint4 line[2];
        uint32_t sc[4];
#pragma unroll
        for (int q = 0; q < 2; q++) line[q] = __ldg(qp + q * 32 + lane);
#pragma unroll
        for (int q = 0; q < 4; q++)
          sc[q] = __ldg(reinterpret_cast<const uint32_t*>(a.meta + ((gbase + q) * 8 + g) * 4));
        const uint32_t wv[8] = {line[0].x, line[0].y, line[0].z, line[0].w,
                                line[1].x, line[1].y, line[1].z, line[1].w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
          float tmp[NT][4];
#pragma unroll
          for (int n = 0; n < NT; n++) tmp[n][0] = tmp[n][1] = tmp[n][2] = tmp[n][3] = 0.f;
#pragma unroll
          for (int ks = 0; ks < 2; ks++) {
            uint32_t av[4];
            q4_pairs(wv[2 * q + ks], av);
            const int j = 2 * q + ks;
#pragma unroll
            for (int n = 0; n < NT; n++) {
              mma16816(tmp[n], av[0], av[1], av[2], av[3], bh[n][j][0], bh[n][j][1]);
              mma16816(tmp[n], av[0], av[1], av[2], av[3], bl[n][j][0], bl[n][j][1]);
            }
          }
          // sum w x = d (16 C' - 24 X)
          const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&sc[q]));
          const float c0 = 16.f * d.x, c1 = 16.f * d.y, x0 = -24.f * d.x, x1 = -24.f * d.y;
#pragma unroll
          for (int n = 0; n < NT; n++) {
            acc[n][0] += fmaf(c0, tmp[n][0], x0 * xblk[n][q][0]);
            acc[n][1] += fmaf(c0, tmp[n][1], x0 * xblk[n][q][1]);
            acc[n][2] += fmaf(c1, tmp[n][2], x1 * xblk[n][q][0]);
            acc[n][3] += fmaf(c1, tmp[n][3], x1 * xblk[n][q][1]);
          }
        }
      } else if constexpr (QT == J4B_Q2_0) {
        const uint4 line = __ldg(reinterpret_cast<const uint4*>(a.quants + gbase * 32 * 4) + lane);
        const uint32_t sc = __ldg(reinterpret_cast<const uint32_t*>(a.meta + ((gbase / 4) * 8 + g) * 4));
        const uint32_t wv[4] = {line.x, line.y, line.z, line.w};
        float tmp[NT][4];
#pragma unroll
        for (int n = 0; n < NT; n++) tmp[n][0] = tmp[n][1] = tmp[n][2] = tmp[n][3] = 0.f;
#pragma unroll
        for (int q = 0; q < 4; q++) {
#pragma unroll
          for (int ks = 0; ks < 2; ks++) {
            const uint32_t a0 = q2_pair(wv[q], 4 * ks), a1 = q2_pair(wv[q], 4 * ks + 1);
            const uint32_t a2 = q2_pair(wv[q], 4 * ks + 2), a3 = q2_pair(wv[q], 4 * ks + 3);
            const int j = 2 * q + ks;
#pragma unroll
            for (int n = 0; n < NT; n++) {
              mma16816(tmp[n], a0, a1, a2, a3, bh[n][j][0], bh[n][j][1]);
              mma16816(tmp[n], a0, a1, a2, a3, bl[n][j][0], bl[n][j][1]);
            }
          }
        }
        // sum w x = d (4 C' - 5 X)
        const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&sc));
        const float c0 = 4.f * d.x, c1 = 4.f * d.y, x0 = -5.f * d.x, x1 = -5.f * d.y;
#pragma unroll
        for (int n = 0; n < NT; n++) {
          acc[n][0] = fmaf(c0, tmp[n][0], x0 * xblk[n][0][0]);
          acc[n][1] = fmaf(c0, tmp[n][1], x0 * xblk[n][0][1]);
          acc[n][2] = fmaf(c1, tmp[n][2], x1 * xblk[n][0][0]);
          acc[n][3] = fmaf(c1, tmp[n][3], x1 * xblk[n][0][1]);
        }
      } else {  // Q4_K: this chunk is half h of super-block sb
        const int64_t sb = k0 / 256;
        const int h = (int)((k0 / 128) & 1);
        const int64_t sbs = a.kpad / 256;
        const uint4* qp = reinterpret_cast<const uint4*>(
            a.quants + (((tile * sbs + sb) * 2 + h) * 32 + lane) * 32);
        const uint4 l0 = __ldg(qp), l1 = __ldg(qp + 1);
        const uint8_t* mp = a.meta + ((tile * sbs + sb) * 8 + g) * 32;
        const uint4 m0 = __ldg(reinterpret_cast<const uint4*>(mp));
        const uint4 m1 = __ldg(reinterpret_cast<const uint4*>(mp + 16));
        // Lane t decodes sub-block 4h+t for rows g and g+8: coefficients 16 d sc and
        // -(16 d sc + dmin m); the group's four lanes then exchange them.
        float cs[2], cx[2];
        {
          const uint4 mm[2] = {m0, m1};
#pragma unroll
          for (int r = 0; r < 2; r++) {
            const uint32_t w0 = mm[r].x, w1 = mm[r].y, w2 = mm[r].z, w3 = mm[r].w;
            const float d = __half2float(__ushort_as_half((uint16_t)(w0 & 0xFFFF)));
            const float dmin = __half2float(__ushort_as_half((uint16_t)(w0 >> 16)));
            // scale bytes q[0..11] are w1 (q0..3), w2 (q4..7), w3 (q8..11)
            const int j = 4 * h + t;
            int sc, mn;
            if (j < 4) {
              sc = (w1 >> (8 * j)) & 63;
              mn = (w2 >> (8 * j)) & 63;
            } else {
              const int jj = j - 4;
              const uint32_t qj4 = (w3 >> (8 * jj)) & 0xFF;  // q[j+4]
              sc = (qj4 & 0xF) | (((w1 >> (8 * jj + 6)) & 3) << 4);
              mn = (qj4 >> 4) | (((w2 >> (8 * jj + 6)) & 3) << 4);
            }
            const float ds = d * (float)sc;
            cs[r] = 16.f * ds;
            cx[r] = -fmaf(16.f, ds, dmin * (float)mn);
          }
        }
        const uint32_t wv[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
          float tmp[NT][4];
#pragma unroll
          for (int n = 0; n < NT; n++) tmp[n][0] = tmp[n][1] = tmp[n][2] = tmp[n][3] = 0.f;
#pragma unroll
          for (int ks = 0; ks < 2; ks++) {
            uint32_t av[4];
            q4_pairs(wv[2 * q + ks], av);
            const int j = 2 * q + ks;
#pragma unroll
            for (int n = 0; n < NT; n++) {
              mma16816(tmp[n], av[0], av[1], av[2], av[3], bh[n][j][0], bh[n][j][1]);
              mma16816(tmp[n], av[0], av[1], av[2], av[3], bl[n][j][0], bl[n][j][1]);
            }
          }
          const int src = (lane & ~3) | q;
          const float s0 = __shfl_sync(0xffffffffu, cs[0], src);
          const float s1 = __shfl_sync(0xffffffffu, cs[1], src);
          const float z0 = __shfl_sync(0xffffffffu, cx[0], src);
          const float z1 = __shfl_sync(0xffffffffu, cx[1], src);
#pragma unroll
          for (int n = 0; n < NT; n++) {
            acc[n][0] += fmaf(s0, tmp[n][0], z0 * xblk[n][q][0]);
            acc[n][1] += fmaf(s0, tmp[n][1], z0 * xblk[n][q][1]);
            acc[n][2] += fmaf(s1, tmp[n][2], z1 * xblk[n][q][0]);
            acc[n][3] += fmaf(s1, tmp[n][3], z1 * xblk[n][q][1]);
          }
        }
      }
    }

    // ---- sum the 8 warp partials of this row tile ----
#pragma unroll
    for (int n = 0; n < NT; n++)
#pragma unroll
      for (int c = 0; c < 4; c++) red[buf][warp][n * 4 + c][lane] = acc[n][c];
    __syncthreads();
    const int v = threadIdx.x;  // one (n, c, lane) value per thread
    float total = 0.f;
    int row = 0, bcol = 0;
    const bool owner = v < NT * 4 * 32;
    if (owner) {
      const int nc = v / 32, ln = v % 32, n = nc / 4, c = nc % 4;
#pragma unroll
      for (int w = 0; w < kWarps; w++) total += red[buf][w][nc][ln];
      row = (ln >> 2) + 8 * (c >> 1);
      bcol = 8 * n + 2 * (ln & 3) + (c & 1);
    }
    if (a.ksplit == 1) {
      if (owner) {
        const int64_t r = tile * 16 + row;
        if (r < a.rows && bcol < a.batch) {
          if (a.add) total += a.add[(int64_t)bcol * a.rows + r];
          a.y[(int64_t)bcol * a.rows + r] = total;
        }
      }
    } else {
      float* part = a.partials + ((int64_t)split * a.rt + tile) * 256;
      if (owner) part[v] = total;
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(a.arrivals + tile, 1u);
        last_flag = prev == (unsigned)(a.ksplit - 1);
      }
      __syncthreads();
      if (last_flag) {
        __threadfence();
        if (owner) {
          float s = 0.f;
          for (int sp = 0; sp < a.ksplit; sp++)
            s += __ldcg(a.partials + ((int64_t)sp * a.rt + tile) * 256 + v);
          const int64_t r = tile * 16 + row;
          if (r < a.rows && bcol < a.batch) {
            if (a.add) s += a.add[(int64_t)bcol * a.rows + r];
            a.y[(int64_t)bcol * a.rows + r] = s;
          }
        }
        if (threadIdx.x == 0) a.arrivals[tile] = 0u;
      }
    }
    buf ^= 1;
  }
}

// ---------------------------------------------------------------------------------------------
// device encoder: byte-identical to the published block encoders the oracle restates
// ---------------------------------------------------------------------------------------------
__device__ inline void wr16(uint8_t* p, uint16_t v) {
  p[0] = (uint8_t)(v & 0xff);
  p[1] = (uint8_t)(v >> 8);
}
__device__ inline uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

__global__ void quantize_kernel(int type, const float* __restrict__ w, int64_t rows, int64_t cols,
                                uint8_t* __restrict__ out) {
  const int be = block_elems(type), bb = block_bytes(type);
  const int64_t nblk = rows * (cols / be);
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= nblk) return;
  const float* src = w + idx * be;  // row-major: blocks of a row are consecutive
  uint8_t* blk = out + idx * bb;
  if (type == J4B_Q8_0) {
    float amax = 0.f;
    for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(src[i]));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
    wr16(blk, f2h(d));
    for (int i = 0; i < 32; i++) {
      int q = (int)roundf(__fmul_rn(src[i], id));
      q = max(-127, min(127, q));
      blk[2 + i] = (uint8_t)(int8_t)q;
    }
  } else if (type == J4B_Q4_0) {
    float amax = 0.f, m = 0.f;
    for (int i = 0; i < 32; i++)
      if (fabsf(src[i]) > amax) {
        amax = fabsf(src[i]);
        m = src[i];
      }
    const float d = __fdiv_rn(m, -8.0f);
    const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
    wr16(blk, f2h(d));
    for (int j = 0; j < 16; j++) {
      int q0 = (int)__fadd_rn(__fmul_rn(src[j], id), 8.5f);
      int q1 = (int)__fadd_rn(__fmul_rn(src[j + 16], id), 8.5f);
      q0 = max(0, min(15, q0));
      q1 = max(0, min(15, q1));
      blk[2 + j] = (uint8_t)(q0 | (q1 << 4));
    }
  } else if (type == J4B_Q2_0) {
    float amax = 0.f;
    for (int i = 0; i < 128; i++) amax = fmaxf(amax, fabsf(src[i]));
    const float id = amax != 0.f ? __fdiv_rn(1.0f, amax) : 0.f;
    wr16(blk, f2h(amax));
    for (int p = 0; p < 32; p++) {
      int byte = 0;
      for (int s = 0; s < 4; s++) {
        int q = (int)roundf(__fmul_rn(src[4 * p + s], id));
        q = max(-1, min(1, q));
        byte |= (q + 1) << (2 * s);
      }
      blk[2 + p] = (uint8_t)byte;
    }
  } else if (type == J4B_Q4_K) {
    float scale[8], mins[8], max_scale = 0.f, max_min = 0.f;
    for (int j = 0; j < 8; j++) {
      float lo = 0.f, hi = src[32 * j];
      for (int i = 0; i < 32; i++) {
        const float v = src[32 * j + i];
        if (v < lo) lo = v;
        if (v > hi) hi = v;
      }
      if (hi < 0.f) hi = 0.f;
      scale[j] = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
      mins[j] = -lo;
      if (scale[j] > max_scale) max_scale = scale[j];
      if (mins[j] > max_min) max_min = mins[j];
    }
    const uint16_t dh = f2h(__fdiv_rn(max_scale, 63.0f)), mh = f2h(__fdiv_rn(max_min, 63.0f));
    const float d = __half2float(__ushort_as_half(dh)), dmin = __half2float(__ushort_as_half(mh));
    int sc[8], m[8];
    for (int j = 0; j < 8; j++) {
      const int s = d > 0.f ? (int)roundf(__fdiv_rn(scale[j], d)) : 0;
      const int mm = dmin > 0.f ? (int)roundf(__fdiv_rn(mins[j], dmin)) : 0;
      sc[j] = max(0, min(63, s));
      m[j] = max(0, min(63, mm));
    }
    wr16(blk, dh);
    wr16(blk + 2, mh);
    uint8_t* sbp = blk + 4;
    for (int j = 0; j < 4; j++) {
      sbp[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
      sbp[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
      sbp[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
    }
    uint8_t* qs = blk + 16;
    for (int c = 0; c < 4; c++)
      for (int l = 0; l < 32; l++) {
        int q[2];
        for (int hh = 0; hh < 2; hh++) {
          const int j = 2 * c + hh;
          const float ds = __fmul_rn(d, (float)sc[j]);
          const float v = __fadd_rn(src[64 * c + 32 * hh + l], __fmul_rn(dmin, (float)m[j]));
          const int qq = ds > 0.f ? (int)roundf(__fdiv_rn(v, ds)) : 0;
          q[hh] = max(0, min(15, qq));
        }
        qs[32 * c + l] = (uint8_t)(q[0] | (q[1] << 4));
      }
  }
}

int qtype_ok(int t) { return block_elems(t) > 0; }

int upload_common(int dev, const uint8_t* dblob, int type, int64_t rows, int64_t cols,
                  cudaStream_t stream, j4b_qweight_t* out) {
  j4b_qweight* w = new j4b_qweight();
  memset(w, 0, sizeof(*w));
  w->dev = dev;
  w->type = type;
  w->rows = rows;
  w->cols = cols;
  w->rt = (rows + 15) / 16;
  w->kpad = (cols + kWarpCols - 1) / kWarpCols * kWarpCols;
  if (type == J4B_Q4_K) w->kpad = (cols + 255) / 256 * 256;
  w->ksplit = (int)((w->kpad + kCtaCols - 1) / kCtaCols);
  const int64_t groups = w->kpad / 32;
  w->quant_bytes = (size_t)(w->rt * groups * 32) * (type == J4B_Q8_0 ? 16 : (type == J4B_Q2_0 ? 4 : 8));
  const int be = block_elems(type);
  w->meta_bytes = (size_t)(w->rt * (w->kpad / be) * 16) * (type == J4B_Q4_K ? 16 : 2);
  cudaError_t e = cudaMalloc(&w->quants, w->quant_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&w->meta, w->meta_bytes);
  if (e == cudaSuccess && w->ksplit > 1) {
    e = cudaMalloc(&w->partials, (size_t)w->ksplit * w->rt * 256 * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&w->arrivals, (size_t)w->rt * sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemsetAsync(w->arrivals, 0, (size_t)w->rt * sizeof(unsigned), stream);
  }
  if (e != cudaSuccess) {
    cudaFree(w->quants);
    cudaFree(w->meta);
    cudaFree(w->partials);
    cudaFree(w->arrivals);
    delete w;
    return cuda_error(e, "quantized weight allocation");
  }
  counters().allocations += w->ksplit > 1 ? 4 : 2;
  {
    const int64_t n = w->rt * groups * 32;
    repack_quants_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(type, dblob, rows, cols, w->rt, w->kpad, w->quants);
    cudaError_t le = cudaGetLastError();
    if (le != cudaSuccess) {
      j4b_quant_free(w);
      return cuda_error(le, "repack_quants_kernel");
    }
    count_launch();
  }
  {
    const int64_t n = w->rt * (w->kpad / be) * 16;
    repack_meta_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(type, dblob, rows, cols, w->rt, w->kpad, w->meta);
    cudaError_t le = cudaGetLastError();
    if (le != cudaSuccess) {
      j4b_quant_free(w);
      return cuda_error(le, "repack_meta_kernel");
    }
    count_launch();
  }
  *out = w;
  return J4B_OK;
}

int check_geometry(int type, int64_t rows, int64_t cols, size_t bytes) {
  if (!qtype_ok(type)) return set_error(J4B_EUNSUPPORTED, "unsupported quant type id %d", type);
  const int be = block_elems(type);
  if (rows <= 0 || cols <= 0 || cols % be)
    return set_error(J4B_EINVAL, "invalid quant dimensions: rows=%lld columns=%lld (block %d)",
                     (long long)rows, (long long)cols, be);
  const int64_t need = rows * (cols / be) * block_bytes(type);
  if ((int64_t)bytes != need)
    return set_error(J4B_EINVAL, "quant blob is %zu bytes, shape needs %lld", bytes, (long long)need);
  return J4B_OK;
}

template <int QT, int NT>
cudaError_t launch_gemv(const j4b_qweight* w, const float* x, const float* add, float* y,
                        int batch, int sms, cudaStream_t stream) {
  GemvArgs a;
  a.quants = w->quants;
  a.meta = w->meta;
  a.rows = w->rows;
  a.cols = w->cols;
  a.kpad = w->kpad;
  a.rt = w->rt;
  a.x = x;
  a.add = add;
  a.y = y;
  a.batch = batch;
  a.ksplit = w->ksplit;
  a.partials = w->partials;
  a.arrivals = w->arrivals;
  // Aim at two resident CTAs per SM in a single wave.
  const int64_t slots = 2ll * sms;
  int64_t tiles = (w->rt * w->ksplit + slots - 1) / slots;
  if (tiles < 1) tiles = 1;
  a.tiles_per_cta = (int)tiles;
  const int64_t grid = (w->rt + tiles - 1) / tiles * w->ksplit;
  qgemv_kernel<QT, NT><<<(unsigned)grid, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

template <int QT>
cudaError_t gemv_dispatch(const j4b_qweight* w, const float* x, const float* add, float* y,
                          int batch, int sms, cudaStream_t stream) {
  if (batch <= 8) return launch_gemv<QT, 1>(w, x, add, y, batch, sms, stream);
  return launch_gemv<QT, 2>(w, x, add, y, batch, sms, stream);
}

}  // namespace
}  // namespace j4b

using namespace j4b;

extern "C" int j4b_quant_supported(int* ids, int cap, int* n) {
  static const int kIds[] = {J4B_Q4_0, J4B_Q8_0, J4B_Q4_K, J4B_Q2_0};
  if (!n) return set_error(J4B_EINVAL, "n is null");
  *n = 4;
  for (int i = 0; i < 4 && i < cap && ids; i++) ids[i] = kIds[i];
  return J4B_OK;
}

extern "C" int j4b_quant_bytes(int type, int64_t rows, int64_t cols, int64_t* bytes) {
  if (!qtype_ok(type)) return set_error(J4B_EUNSUPPORTED, "unsupported quant type id %d", type);
  const int be = block_elems(type);
  if (rows <= 0 || cols <= 0 || cols % be)
    return set_error(J4B_EINVAL, "quant tensor is not block-aligned: %lld columns, block=%d",
                     (long long)cols, be);
  *bytes = rows * (cols / be) * block_bytes(type);
  return J4B_OK;
}

extern "C" int j4b_quant_upload(int dev, const void* blocks, size_t bytes, int type, int64_t rows,
                                int64_t cols, j4b_qweight_t* out) {
  if (!out || !blocks) return set_error(J4B_EINVAL, "null argument to quant upload");
  int st = check_geometry(type, rows, cols, bytes);
  if (st) return st;
  st = ensure_device(dev);
  if (st) return st;
  DeviceGuard guard(dev);
  cudaStream_t stream = device_ctx(dev)->stream;
  void* staging = nullptr;
  J4B_CUDA(cudaMallocAsync(&staging, bytes, stream), "cudaMallocAsync(quant staging)");
  J4B_CUDA(cudaMemcpyAsync(staging, blocks, bytes, cudaMemcpyHostToDevice, stream), "cudaMemcpyAsync(quant)");
  counters().h2d += bytes;
  st = upload_common(dev, (const uint8_t*)staging, type, rows, cols, stream, out);
  cudaFreeAsync(staging, stream);
  if (st) return st;
  J4B_CUDA(cudaStreamSynchronize(stream), "cudaStreamSynchronize(quant upload)");
  return J4B_OK;
}

extern "C" int j4b_quant_upload_device(int dev, j4b_buf blocks, size_t bytes, int type,
                                       int64_t rows, int64_t cols, j4b_qweight_t* out) {
  if (!out || !blocks) return set_error(J4B_EINVAL, "null argument to quant upload");
  int st = check_geometry(type, rows, cols, bytes);
  if (st) return st;
  st = ensure_device(dev);
  if (st) return st;
  DeviceGuard guard(dev);
  cudaStream_t stream = device_ctx(dev)->stream;
  // Order after any work the caller queued on its own streams that produced the blob.
  J4B_CUDA(cudaDeviceSynchronize(), "cudaDeviceSynchronize(quant upload)");
  st = upload_common(dev, (const uint8_t*)(uintptr_t)blocks, type, rows, cols, stream, out);
  if (st) return st;
  J4B_CUDA(cudaStreamSynchronize(stream), "cudaStreamSynchronize(quant upload)");
  return J4B_OK;
}

extern "C" int j4b_quant_free(j4b_qweight_t w) {
  if (!w) return J4B_OK;
  DeviceGuard guard(w->dev);
  cudaFree(w->quants);
  cudaFree(w->meta);
  cudaFree(w->partials);
  cudaFree(w->arrivals);
  counters().releases += w->partials ? 4 : 2;
  delete w;
  return J4B_OK;
}

extern "C" int j4b_quant_shape(j4b_qweight_t w, int* type, int64_t* rows, int64_t* cols) {
  if (!w) return set_error(J4B_EINVAL, "null quantized weight");
  if (type) *type = w->type;
  if (rows) *rows = w->rows;
  if (cols) *cols = w->cols;
  return J4B_OK;
}

extern "C" int j4b_quant_matvec(j4b_qweight_t w, j4b_buf x, j4b_buf add, j4b_buf y,
                                int64_t batch, j4b_stream s) {
  if (!w) return set_error(J4B_EINVAL, "null quantized weight");
  J4B_REQUIRE(batch >= 1, "quantMatvec batch must be positive, got %lld", (long long)batch);
  J4B_REQUIRE(x && y, "quantMatvec needs x and y buffers");
  J4B_REQUIRE(((x | y | add) & 7) == 0, "quantMatvec buffers must be 8-byte aligned");
  DeviceGuard guard(w->dev);
  cudaStream_t stream = resolve_stream(w->dev, s);
  const int sms = device_ctx(w->dev)->sm_count;
  for (int64_t b0 = 0; b0 < batch; b0 += 16) {
    const int nb = (int)std::min<int64_t>(16, batch - b0);
    const float* xp = (const float*)(uintptr_t)x + b0 * w->cols;
    const float* ap = add ? (const float*)(uintptr_t)add + b0 * w->rows : nullptr;
    float* yp = (float*)(uintptr_t)y + b0 * w->rows;
    cudaError_t e = cudaErrorInvalidValue;
    switch (w->type) {
      case J4B_Q8_0: e = gemv_dispatch<J4B_Q8_0>(w, xp, ap, yp, nb, sms, stream); break;
      case J4B_Q4_0: e = gemv_dispatch<J4B_Q4_0>(w, xp, ap, yp, nb, sms, stream); break;
      case J4B_Q4_K: e = gemv_dispatch<J4B_Q4_K>(w, xp, ap, yp, nb, sms, stream); break;
      case J4B_Q2_0: e = gemv_dispatch<J4B_Q2_0>(w, xp, ap, yp, nb, sms, stream); break;
    }
    if (e != cudaSuccess) return cuda_error(e, "qgemv_kernel");
    count_launch();
  }
  return J4B_OK;
}

extern "C" int j4b_quant_gather_row(j4b_qweight_t w, int64_t row, j4b_buf out, j4b_stream s) {
  if (!w) return set_error(J4B_EINVAL, "null quantized weight");
  J4B_REQUIRE(row >= 0 && row < w->rows, "quantGatherRow row %lld out of range [0, %lld)",
              (long long)row, (long long)w->rows);
  J4B_REQUIRE(out, "quantGatherRow needs an output buffer");
  DeviceGuard guard(w->dev);
  cudaStream_t stream = resolve_stream(w->dev, s);
  gather_row_kernel<<<(unsigned)((w->cols + 255) / 256), 256, 0, stream>>>(*w, row, (float*)(uintptr_t)out);
  J4B_CHECK_LAUNCH("gather_row_kernel");
  return J4B_OK;
}

extern "C" int j4b_quantize(int type, j4b_buf w, int64_t rows, int64_t cols, j4b_buf out,
                            j4b_stream s) {
  if (!qtype_ok(type)) return set_error(J4B_EUNSUPPORTED, "unsupported quant type id %d", type);
  const int be = block_elems(type);
  J4B_REQUIRE(rows > 0 && cols > 0 && cols % be == 0, "invalid quantize dimensions");
  J4B_REQUIRE(w && out, "quantize needs input and output buffers");
  int dev = 0;
  int st = device_of((const void*)(uintptr_t)w, &dev);
  if (st) return st;
  DeviceGuard guard(dev);
  const int64_t nblk = rows * (cols / be);
  quantize_kernel<<<(unsigned)((nblk + 127) / 128), 128, 0, resolve_stream(dev, s)>>>(
      type, (const float*)(uintptr_t)w, rows, cols, (uint8_t*)(uintptr_t)out);
  J4B_CHECK_LAUNCH("quantize_kernel");
  return J4B_OK;
}
