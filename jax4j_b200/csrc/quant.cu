// GGUF block-quantised matrices: upload + repack, batched dequant-GEMV, bit-exact row gather and
// a device-side encoder.
//
// Reference interface: core/tensor/spi/QuantizedOps.java:19-34, CPU semantics in
// core/backend/cpu/CpuBackend.java:690-755, CpuQ4Gemm.java:17-77, CpuQ2Gemm.java:17-83. The
// reference has no GPU quantised path; Q8_0, Q4_K and Q6_K have no implementation at all there
// (core/tensor/QuantType.java:8-10 only) and follow the public GGUF block layouts.
//
// Device layout ("fragment-major repack", same byte count as the GGUF blob):
//   A weight of R rows x K columns is cut into row tiles of 16 rows. Inside a row tile, every
//   group of 32 columns (one Q8_0/Q4_0 block, one Q4_K sub-block, an eighth of a Q6_K
//   super-block, a quarter Q2_0 block) holds
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
// Work split (qgemv_stream.cuh): one CTA per SM owns one K range of 1024 columns and a run of row
// tiles, streamed into shared memory by a producer warp; each compute warp owns whole tiles, so
// a tile's partial over the K range stays in one warp's registers. K ranges are combined by the
// warp whose arrival completes the tile's counter (partials in per-weight scratch, added in K
// order), which also applies `add`.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>

#include <cuda_bf16.h>

#include "j4b_internal.h"
#include "j4b_wait.cuh"
#include "tc_common.cuh"

struct j4b_qweight {
  int dev;
  int type;
  int64_t rows, cols;
  int64_t rt;     // row tiles of 16
  int64_t kpad;   // K rounded up to the 128-column warp chunk
  int ksplit;     // K ranges of 1024 columns
  uint8_t* data;       // repacked plane (split-major, see Layout)
  size_t data_bytes;   // equal to the GGUF blob size when rows % 16 == 0 and cols % 128 == 0
  float* partials;     // [ksplit][rt][256] split-K scratch
  unsigned* arrivals;  // [rt] arrival counters (one per tile group), zero between launches
  int* status;         // set to nonzero by a kernel whose bounded wait gave up
  // Set by the upload: the repack kernels that wrote `data` may be the kernels right before the
  // next GEMV in the stream, and a GEMV launched with programmatic dependent launch reads its
  // weights before it waits on the kernel before it; the first GEMV after an upload therefore
  // launches without it (host-side flag, cleared at that launch).
  bool fresh;
  // Device staging of x and y for the host-buffer calls (16 rows of x, then y), allocated by the
  // first one; like the split-K scratch, it serialises the calls made on one weight.
  float* io;
  int64_t io_floats;
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
    case J4B_Q6_K: return 256;
    case J4B_Q2_0: return 128;
  }
  return -1;
}
__host__ __device__ inline int block_bytes(int t) {
  switch (t) {
    case J4B_Q4_0: return 18;
    case J4B_Q8_0: return 34;
    case J4B_Q4_K: return 144;
    case J4B_Q6_K: return 210;
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
    case J4B_Q6_K: {  // 6-bit code 0..63: ql nibble | qh crumb << 4
      const int n = w / 128, s = (w % 128) / 32, l = w % 32;
      const int b = blk[64 * n + l + 32 * (s & 1)];
      const int nib = s >= 2 ? (b >> 4) : (b & 0xF);
      return nib | (((blk[128 + 32 * n + l] >> (2 * s)) & 3) << 4);
    }
  }
  return 0;
}

// ---------------------------------------------------------------------------------------------
// repacked layout ("split-major"): one plane holding, for each 1024-column K range ("split") s
// and each 16-row tile t, one contiguous chunk [quant bytes of the split's 32-column groups |
// scale bytes of those groups]. A CTA that owns split s of tiles t0..t1 therefore streams one
// contiguous byte range. Within a chunk, group gl (0..groups_here) occupies, per type:
//   Q8_0: quants gl*512 + lane*16 (k-step ks, element e at byte 8ks+e, code ^ 0x80);
//         scales gl*32 + g*4 + which*2 (f16 d of row g / row g+8 of the tile)
//   Q4_0: quants (gl/2)*512 + lane*16 + (gl%2)*8 (two words, k-steps 0/1, nibbles at nib_pos);
//         scales as Q8_0
//   Q4_K: quants (gl/4)*1024 + lane*32 + (gl%4)*8; scales (gl/8)*256 + (g*2+which)*16, the
//         row's 16 GGUF bytes (d, dmin, 12 packed 6-bit scales/mins) per super-block
//   Q2_0: quants (gl/4)*512 + lane*16 + (gl%4)*4 (one word, crumbs at crumb_pos);
//         scales (gl/4)*32 + g*4 + which*2
//   Q6_K: quants (gl/4)*1536 + lane*48: the lane's low-nibble words at + (gl%4)*8 (two words,
//         k-steps 0/1, nibbles at nib_pos) and its high-crumb word at + 32 + (gl%4)*4 (bits 4-5
//         of each code at crumb_pos); scales (gl/8)*288: the row's 16 int8 sub-block scales at
//         + (g*2+which)*16, its f16 d at + 256 + (g*2+which)*2
// ---------------------------------------------------------------------------------------------
__host__ __device__ inline int group_quant_bytes(int t) {
  return t == J4B_Q8_0 ? 512 : (t == J4B_Q2_0 ? 128 : (t == J4B_Q6_K ? 384 : 256));
}
__host__ __device__ inline int group_meta_bytes(int t) { return t == J4B_Q2_0 ? 8 : (t == J4B_Q6_K ? 36 : 32); }

struct Layout {
  int type;
  int64_t rt, kpad;
  __host__ __device__ int groups_in_split(int64_t s) const {
    const int64_t rem = (kpad - s * 1024) / 32;
    return (int)(rem < 32 ? rem : 32);
  }
  __host__ __device__ int64_t chunk_bytes(int64_t s) const {
    return (int64_t)groups_in_split(s) * (group_quant_bytes(type) + group_meta_bytes(type));
  }
  __host__ __device__ int64_t chunk_offset(int64_t s, int64_t tile) const {
    return s * rt * 32 * (group_quant_bytes(type) + group_meta_bytes(type)) + tile * chunk_bytes(s);
  }
  __host__ __device__ int64_t total_bytes() const {
    const int64_t splits = (kpad + 1023) / 1024;
    return chunk_offset(splits - 1, rt);
  }
  // byte offset of lane `lane`'s quant data for global 32-column group G of `tile`
  __host__ __device__ int64_t quant_offset(int64_t tile, int64_t G, int lane) const {
    const int64_t s = G / 32;
    const int gl = (int)(G % 32);
    const int64_t base = chunk_offset(s, tile);
    switch (type) {
      case J4B_Q8_0: return base + gl * 512 + lane * 16;
      case J4B_Q4_0: return base + (gl / 2) * 512 + lane * 16 + (gl % 2) * 8;
      case J4B_Q4_K: return base + (gl / 4) * 1024 + lane * 32 + (gl % 4) * 8;
      case J4B_Q6_K: return base + (gl / 4) * 1536 + lane * 48 + (gl % 4) * 8;
      default: return base + (gl / 4) * 512 + lane * 16 + (gl % 4) * 4;
    }
  }
  // Q6_K: byte offset of lane `lane`'s high-crumb word for global group G of `tile`
  __host__ __device__ int64_t crumb_offset(int64_t tile, int64_t G, int lane) const {
    const int gl = (int)(G % 32);
    return chunk_offset(G / 32, tile) + (gl / 4) * 1536 + lane * 48 + 32 + (gl % 4) * 4;
  }
  // byte offset of the scale data of row (g, which) of `tile` for global group G
  __host__ __device__ int64_t meta_offset(int64_t tile, int64_t G, int g, int which) const {
    const int64_t s = G / 32;
    const int gl = (int)(G % 32);
    const int64_t base = chunk_offset(s, tile) + (int64_t)groups_in_split(s) * group_quant_bytes(type);
    switch (type) {
      case J4B_Q4_K: return base + (gl / 8) * 256 + (g * 2 + which) * 16;
      case J4B_Q6_K: return base + (gl / 8) * 288 + (g * 2 + which) * 16;
      case J4B_Q2_0: return base + (gl / 4) * 32 + g * 4 + which * 2;
      default: return base + gl * 32 + g * 4 + which * 2;
    }
  }
  // Q6_K: byte offset of the f16 d of row (g, which) of `tile` for global group G
  __host__ __device__ int64_t d_offset(int64_t tile, int64_t G, int g, int which) const {
    const int64_t s = G / 32;
    const int gl = (int)(G % 32);
    return chunk_offset(s, tile) + (int64_t)groups_in_split(s) * group_quant_bytes(type) + (gl / 8) * 288 + 256 +
           (g * 2 + which) * 2;
  }
};

// One thread per (row tile, 32-column group, lane): writes that lane's quant bytes.
__global__ void repack_quants_kernel(Layout L, const uint8_t* __restrict__ blob, int64_t rows,
                                     int64_t cols, uint8_t* __restrict__ out) {
  const int type = L.type;
  const int64_t groups = L.kpad / 32;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= L.rt * groups * 32) return;
  const int lane = (int)(idx % 32);
  const int64_t grp = (idx / 32) % groups;
  const int64_t tile = idx / 32 / groups;
  const int64_t r0 = tile * 16, k0 = grp * 32;
  uint8_t* dst = out + L.quant_offset(tile, grp, lane);
  bool in;
  if (type == J4B_Q8_0) {
    for (int ks = 0; ks < 2; ks++)
      for (int e = 0; e < 8; e++) {
        const int q = raw_code(type, blob, rows, cols, r0 + frag_row(lane, e), k0 + 16 * ks + frag_col(lane, e), &in);
        dst[8 * ks + e] = (uint8_t)((q & 0xFF) ^ 0x80);
      }
  } else if (type == J4B_Q4_0 || type == J4B_Q4_K) {
    uint32_t words[2] = {0, 0};
    for (int ks = 0; ks < 2; ks++)
      for (int e = 0; e < 8; e++) {
        const int q = raw_code(type, blob, rows, cols, r0 + frag_row(lane, e), k0 + 16 * ks + frag_col(lane, e), &in);
        words[ks] |= rotl32((uint32_t)(q & 0xF), nib_pos(e));
      }
    reinterpret_cast<uint32_t*>(dst)[0] = words[0];
    reinterpret_cast<uint32_t*>(dst)[1] = words[1];
  } else if (type == J4B_Q2_0) {
    uint32_t word = 0;
    for (int ks = 0; ks < 2; ks++)
      for (int e = 0; e < 8; e++) {
        int c = raw_code(type, blob, rows, cols, r0 + frag_row(lane, e), k0 + 16 * ks + frag_col(lane, e), &in);
        if (!in) c = 1;  // padding decodes to 0
        word |= rotl32((uint32_t)(c & 3), crumb_pos(4 * ks + (e >> 1), e & 1));
      }
    reinterpret_cast<uint32_t*>(dst)[0] = word;
  } else if (type == J4B_Q6_K) {
    uint32_t words[2] = {0, 0}, crumbs = 0;
    for (int ks = 0; ks < 2; ks++)
      for (int e = 0; e < 8; e++) {
        const int q = raw_code(type, blob, rows, cols, r0 + frag_row(lane, e), k0 + 16 * ks + frag_col(lane, e), &in);
        words[ks] |= rotl32((uint32_t)(q & 0xF), nib_pos(e));
        crumbs |= rotl32((uint32_t)((q >> 4) & 3), crumb_pos(4 * ks + (e >> 1), e & 1));
      }
    reinterpret_cast<uint32_t*>(dst)[0] = words[0];
    reinterpret_cast<uint32_t*>(dst)[1] = words[1];
    *reinterpret_cast<uint32_t*>(out + L.crumb_offset(tile, grp, lane)) = crumbs;
  }
}

// One thread per (row tile, GGUF block, row in tile): copies the row's scale bytes.
__global__ void repack_meta_kernel(Layout L, const uint8_t* __restrict__ blob, int64_t rows,
                                   int64_t cols, uint8_t* __restrict__ out) {
  const int type = L.type;
  const int be = block_elems(type), bb = block_bytes(type);
  const int64_t blocks = L.kpad / be;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= L.rt * blocks * 16) return;
  const int rr = (int)(idx % 16);
  const int64_t blk = (idx / 16) % blocks;
  const int64_t tile = idx / 16 / blocks;
  const int64_t r = tile * 16 + rr;
  const bool in = r < rows && blk * be < cols;
  const uint8_t* src = in ? blob + (r * (cols / be) + blk) * bb : nullptr;
  const int g = rr & 7, which = rr >> 3;
  const int64_t G = blk * be / 32;  // first 32-column group of the block
  uint8_t* dst = out + L.meta_offset(tile, G, g, which);
  if (type == J4B_Q6_K) {  // 16 scales from byte 192, d from byte 208
    for (int i = 0; i < 16; i++) dst[i] = in ? src[192 + i] : 0;
    uint8_t* dd = out + L.d_offset(tile, G, g, which);
    dd[0] = in ? src[208] : 0;
    dd[1] = in ? src[209] : 0;
    return;
  }
  const int n = type == J4B_Q4_K ? 16 : 2;
  for (int i = 0; i < n; i++) dst[i] = in ? src[i] : 0;
}

// ---------------------------------------------------------------------------------------------
// bit-exact gather (quantGatherRow) from the repacked layout
// ---------------------------------------------------------------------------------------------
__device__ inline int repacked_code(const Layout& L, const uint8_t* data, int64_t r, int64_t k) {
  const int64_t tile = r / 16;
  const int rr = (int)(r % 16);
  const int64_t grp = k / 32;
  const int kk = (int)(k % 32), ks = kk / 16, k16 = kk % 16;
  const int g = rr & 7, hi8 = rr >> 3;
  const int t = (k16 & 7) >> 1;
  const int lane = 4 * g + t;
  const int e = (k16 & 1) + 2 * hi8 + 4 * (k16 >> 3);
  const uint8_t* p = data + L.quant_offset(tile, grp, lane);
  if (L.type == J4B_Q8_0) return (int)(int8_t)(p[8 * ks + e] ^ 0x80);
  if (L.type == J4B_Q4_0 || L.type == J4B_Q4_K)
    return rotr32(reinterpret_cast<const uint32_t*>(p)[ks], nib_pos(e)) & 0xF;
  if (L.type == J4B_Q6_K) {
    const uint32_t cw = *reinterpret_cast<const uint32_t*>(data + L.crumb_offset(tile, grp, lane));
    return (int)((rotr32(reinterpret_cast<const uint32_t*>(p)[ks], nib_pos(e)) & 0xF) |
                 ((rotr32(cw, crumb_pos(4 * ks + (e >> 1), e & 1)) & 3) << 4));
  }
  return rotr32(reinterpret_cast<const uint32_t*>(p)[0], crumb_pos(4 * ks + (e >> 1), e & 1)) & 3;
}

__global__ void gather_row_kernel(Layout L, const uint8_t* __restrict__ data, int64_t cols,
                                  int64_t row, float* __restrict__ out) {
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= cols) return;
  const int64_t tile = row / 16;
  const int rr = (int)(row % 16), g = rr & 7, which = rr >> 3;
  const int q = repacked_code(L, data, row, k);
  const uint8_t* m = data + L.meta_offset(tile, k / 32, g, which);
  float v;
  if (L.type == J4B_Q4_K) {
    const float d = __half2float(__ushort_as_half(rd16(m)));
    const float dmin = __half2float(__ushort_as_half(rd16(m + 2)));
    const int j = (int)((k % 256) / 32);
    int sc, mn;
    q4k_scale_min(j, m + 4, &sc, &mn);
    const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)mn);
    v = __fsub_rn(__fmul_rn(d1, (float)q), m1);  // d1*q is exact; one rounding, as the oracle
  } else if (L.type == J4B_Q6_K) {
    const float d = __half2float(__ushort_as_half(rd16(data + L.d_offset(tile, k / 32, g, which))));
    const int sc = (int)(int8_t)m[(k % 256) / 16];
    v = __fmul_rn(__fmul_rn(d, (float)sc), (float)(q - 32));  // (d * sc) * (q - 32), as the oracle
  } else {
    const float d = __half2float(__ushort_as_half(rd16(m)));
    const int code = L.type == J4B_Q8_0 ? q : (L.type == J4B_Q4_0 ? q - 8 : q - 1);
    v = __fmul_rn(d, (float)code);
  }
  out[k] = v;
}

// Prefill operands: W decoded to bf16 hi (and lo = residual, for the 3-term mode) K-major [rows, kp];
// each value is first decoded bit-exactly as by gather_row_kernel. One thread per (row, 32-column
// group): the group's scale once, its 32 codes from the fragment words of lanes 4g .. 4g+3 (row
// rr of a tile lives in lanes 4 (rr & 7) + t, half rr >> 3 of their elements) at positions fixed at
// compile time, four 16-byte stores. Columns past `cols` are zeros.
template <int QT>
__device__ __forceinline__ void group_codes(const Layout& L, const uint8_t* __restrict__ data, int64_t tile,
                                            int64_t G, int g, int hi8, int (&q)[32]) {
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const uint8_t* p = data + L.quant_offset(tile, G, 4 * g + t);
    uint32_t w[4];
    if constexpr (QT == J4B_Q8_0) {
      const uint4 v = *reinterpret_cast<const uint4*>(p);
      w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    } else if constexpr (QT == J4B_Q2_0) {
      w[0] = *reinterpret_cast<const uint32_t*>(p);
    } else {
      const uint2 v = *reinterpret_cast<const uint2*>(p);
      w[0] = v.x; w[1] = v.y;
      if constexpr (QT == J4B_Q6_K) w[2] = *reinterpret_cast<const uint32_t*>(data + L.crumb_offset(tile, G, 4 * g + t));
    }
#pragma unroll
    for (int ks = 0; ks < 2; ++ks)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          const int e = b + 2 * hi8 + 4 * h;  // hi8 is 0 or 1: both cases unroll below
          const int col = 16 * ks + 8 * h + 2 * t + b;
          int code;
          if constexpr (QT == J4B_Q8_0) {
            const int byte = 8 * ks + e;
            code = (int)(int8_t)(((w[byte >> 2] >> (8 * (byte & 3))) & 0xFF) ^ 0x80);
          } else if constexpr (QT == J4B_Q2_0) {
            code = (int)(rotr32(w[0], crumb_pos(4 * ks + (e >> 1), e & 1)) & 3);
          } else if constexpr (QT == J4B_Q6_K) {
            code = (int)((rotr32(w[ks], nib_pos(e)) & 0xF) | ((rotr32(w[2], crumb_pos(4 * ks + (e >> 1), e & 1)) & 3) << 4));
          } else {
            code = (int)(rotr32(w[ks], nib_pos(e)) & 0xF);
          }
          q[col] = code;
        }
  }
}

template <int QT>
__global__ void dequant_bf16_kernel(Layout L, const uint8_t* __restrict__ data, int64_t rows, int64_t cols,
                                    int64_t kp, __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
  const int64_t groups = kp / 32;
  const int64_t total = rows * groups;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / groups, G = i % groups, k0 = G * 32;
    const int64_t tile = row / 16;
    const int rr = (int)(row % 16), g = rr & 7, which = rr >> 3;
    float d1 = 0.f, m1 = 0.f, d = 0.f;  // Q6_K: d1, m1 = d * sc of the group's two sub-blocks
    const bool live = k0 < cols;
    int q[32];
    if (live) {
      const uint8_t* m = data + L.meta_offset(tile, G, g, which);
      d = __half2float(__ushort_as_half(rd16(m)));
      if constexpr (QT == J4B_Q4_K) {
        const float dmin = __half2float(__ushort_as_half(rd16(m + 2)));
        int sc, mn;
        q4k_scale_min((int)((k0 % 256) / 32), m + 4, &sc, &mn);
        d1 = __fmul_rn(d, (float)sc);
        m1 = __fmul_rn(dmin, (float)mn);
      } else if constexpr (QT == J4B_Q6_K) {
        d = __half2float(__ushort_as_half(rd16(data + L.d_offset(tile, G, g, which))));
        const int j = (int)((k0 % 256) / 16);
        d1 = __fmul_rn(d, (float)(int8_t)m[j]);
        m1 = __fmul_rn(d, (float)(int8_t)m[j + 1]);
      }
      if (which) group_codes<QT>(L, data, tile, G, g, 1, q);
      else group_codes<QT>(L, data, tile, G, g, 0, q);
    }
    __nv_bfloat16* hrow = hi + row * kp + k0;
    __nv_bfloat16* lrow = lo ? lo + row * kp + k0 : nullptr;
#pragma unroll
    for (int c = 0; c < 32; c += 8) {
      alignas(16) __nv_bfloat16 h8[8], l8[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t k = k0 + c + u;
        float v = 0.0f;
        if (live && k < cols) {
          if constexpr (QT == J4B_Q4_K) v = __fsub_rn(__fmul_rn(d1, (float)q[c + u]), m1);
          else if constexpr (QT == J4B_Q6_K) v = __fmul_rn(c < 16 ? d1 : m1, (float)(q[c + u] - 32));
          else v = __fmul_rn(d, (float)(QT == J4B_Q8_0 ? q[c + u] : (QT == J4B_Q4_0 ? q[c + u] - 8 : q[c + u] - 1)));
        }
        h8[u] = __float2bfloat16_rn(v);
        l8[u] = __float2bfloat16_rn(v - __bfloat162float(h8[u]));
      }
      *reinterpret_cast<uint4*>(hrow + c) = *reinterpret_cast<const uint4*>(h8);
      if (lrow) *reinterpret_cast<uint4*>(lrow + c) = *reinterpret_cast<const uint4*>(l8);
    }
  }
}

Layout layout_of(const j4b_qweight* w) {
  Layout L;
  L.type = w->type;
  L.rt = w->rt;
  L.kpad = w->kpad;
  return L;
}

#include "qgemv.cuh"
#include "qgemm_fused.cuh"

// ---------------------------------------------------------------------------------------------
// device encoder: byte-identical to the published block encoders the oracle restates
// ---------------------------------------------------------------------------------------------
__device__ inline uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// A block is assembled in a register array of 32-bit words, then written out byte by byte.
struct BlockBytes {
  uint32_t w[53] = {};
  __device__ void put(int i, uint32_t v) { w[i >> 2] |= (v & 0xffu) << (8 * (i & 3)); }
  __device__ void put16(int i, uint16_t v) {
    put(i, v & 0xffu);
    put(i + 1, v >> 8);
  }
  __device__ uint8_t get(int i) const { return (uint8_t)(w[i >> 2] >> (8 * (i & 3))); }
};

__global__ void quantize_kernel(int type, const float* __restrict__ w, int64_t rows, int64_t cols,
                                uint8_t* __restrict__ out) {
  const int be = block_elems(type), bb = block_bytes(type);
  const int64_t nblk = rows * (cols / be);
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= nblk) return;
  const float* src = w + idx * be;  // row-major: blocks of a row are consecutive
  BlockBytes blk;
  if (type == J4B_Q8_0) {
    float amax = 0.f;
    for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(src[i]));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
    blk.put16(0, f2h(d));
    for (int i = 0; i < 32; i++) {
      int q = (int)roundf(__fmul_rn(src[i], id));
      q = max(-127, min(127, q));
      blk.put(2 + i, (uint32_t)(q & 0xff));
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
    blk.put16(0, f2h(d));
    for (int j = 0; j < 16; j++) {
      int q0 = (int)__fadd_rn(__fmul_rn(src[j], id), 8.5f);
      int q1 = (int)__fadd_rn(__fmul_rn(src[j + 16], id), 8.5f);
      q0 = max(0, min(15, q0));
      q1 = max(0, min(15, q1));
      blk.put(2 + j, (uint32_t)(q0 | (q1 << 4)));
    }
  } else if (type == J4B_Q2_0) {
    float amax = 0.f;
    for (int i = 0; i < 128; i++) amax = fmaxf(amax, fabsf(src[i]));
    const float id = amax != 0.f ? __fdiv_rn(1.0f, amax) : 0.f;
    blk.put16(0, f2h(amax));
    for (int p = 0; p < 32; p++) {
      int byte = 0;
      for (int s = 0; s < 4; s++) {
        int q = (int)roundf(__fmul_rn(src[4 * p + s], id));
        q = max(-1, min(1, q));
        byte |= (q + 1) << (2 * s);
      }
      blk.put(2 + p, (uint32_t)byte);
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
    blk.put16(0, dh);
    blk.put16(2, mh);
    for (int j = 0; j < 4; j++) {
      blk.put(4 + j, (uint32_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6)));
      blk.put(8 + j, (uint32_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6)));
      blk.put(12 + j, (uint32_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4)));
    }
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
        blk.put(16 + 32 * c + l, (uint32_t)(q[0] | (q[1] << 4)));
      }
  } else if (type == J4B_Q6_K) {
    // per 16 elements s_j = (the largest-magnitude value) / 31; d = max |s_j| / 127 (f16);
    // sc_j = round(s_j / d) in [-127, 127]; codes round(w / (d sc_j)) in [-32, 31], stored + 32
    float sub[16], max_abs = 0.f;
    for (int j = 0; j < 16; j++) {
      float best = 0.f;
      for (int i = 0; i < 16; i++)
        if (fabsf(src[16 * j + i]) > fabsf(best)) best = src[16 * j + i];
      sub[j] = __fdiv_rn(best, 31.0f);
      if (fabsf(sub[j]) > max_abs) max_abs = fabsf(sub[j]);
    }
    const uint16_t dh = f2h(__fdiv_rn(max_abs, 127.0f));
    const float d = __half2float(__ushort_as_half(dh));
    int sc[16];
    for (int j = 0; j < 16; j++) {
      const int v = d > 0.f ? (int)roundf(__fdiv_rn(sub[j], d)) : 0;
      sc[j] = max(-127, min(127, v));
      blk.put(192 + j, (uint32_t)(sc[j] & 0xff));
    }
    blk.put16(208, dh);
    for (int e = 0; e < 256; e++) {
      const int n = e / 128, s = (e % 128) / 32, l = e % 32;
      const float ds = __fmul_rn(d, (float)sc[e / 16]);
      int q = ds != 0.f ? (int)roundf(__fdiv_rn(src[e], ds)) : 0;
      q = max(-32, min(31, q)) + 32;
      blk.put(64 * n + l + 32 * (s & 1), (uint32_t)((q & 0xF) << (s >= 2 ? 4 : 0)));
      blk.put(128 + 32 * n + l, (uint32_t)(((q >> 4) & 3) << (2 * s)));
    }
  }
  uint8_t* dst = out + idx * bb;
  for (int i = 0; i < bb; i++) dst[i] = blk.get(i);
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
  if (type == J4B_Q4_K || type == J4B_Q6_K) w->kpad = (cols + 255) / 256 * 256;
  w->ksplit = (int)((w->kpad + kCtaCols - 1) / kCtaCols);
  const Layout L = layout_of(w);
  w->data_bytes = (size_t)L.total_bytes();
  cudaError_t e = cudaMalloc(&w->data, w->data_bytes);
  if (e == cudaSuccess && w->ksplit > 1)
    e = cudaMalloc(&w->partials, (size_t)w->ksplit * w->rt * 256 * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&w->arrivals, (size_t)(w->rt + 1) * sizeof(unsigned));
  if (e == cudaSuccess)
    e = cudaMemsetAsync(w->arrivals, 0, (size_t)(w->rt + 1) * sizeof(unsigned), stream);
  if (e == cudaSuccess) w->status = (int*)(w->arrivals + w->rt);
  if (e != cudaSuccess) {
    cudaFree(w->data);
    cudaFree(w->partials);
    cudaFree(w->arrivals);
    delete w;
    return cuda_error(e, "quantized weight allocation");
  }
  counters().allocations += w->ksplit > 1 ? 3 : 2;
  {
    const int64_t n = w->rt * (w->kpad / 32) * 32;
    repack_quants_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(L, dblob, rows, cols, w->data);
    cudaError_t le = cudaGetLastError();
    if (le != cudaSuccess) {
      j4b_quant_free(w);
      return cuda_error(le, "repack_quants_kernel");
    }
    count_launch();
  }
  {
    const int64_t n = w->rt * (w->kpad / block_elems(type)) * 16;
    repack_meta_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(L, dblob, rows, cols, w->data);
    cudaError_t le = cudaGetLastError();
    if (le != cudaSuccess) {
      j4b_quant_free(w);
      return cuda_error(le, "repack_meta_kernel");
    }
    count_launch();
  }
  w->fresh = true;
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

}  // namespace
}  // namespace j4b

using namespace j4b;

extern "C" int j4b_quant_supported(int* ids, int cap, int* n) {
  static const int kIds[] = {J4B_Q4_0, J4B_Q8_0, J4B_Q4_K, J4B_Q6_K, J4B_Q2_0};
  if (!n) return set_error(J4B_EINVAL, "n is null");
  *n = 5;
  for (int i = 0; i < 5 && i < cap && ids; i++) ids[i] = kIds[i];
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
  cudaFree(w->data);
  cudaFree(w->partials);
  cudaFree(w->arrivals);
  counters().releases += w->partials ? 3 : 2;
  if (w->io) {
    cudaFree(w->io);
    counters().releases += 1;
  }
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

namespace j4b {
namespace {
int quant_gemm_fused(const j4b_qweight* w, const float* x, float* y, const float* add, int64_t m, int64_t kp, int terms,
                     int sms, cudaStream_t stream);
}  // namespace
}  // namespace j4b

extern "C" int j4b_quant_matvec(j4b_qweight_t w, j4b_buf x, j4b_buf add, j4b_buf y,
                                int64_t batch, j4b_stream s) {
  if (!w) return set_error(J4B_EINVAL, "null quantized weight");
  J4B_REQUIRE(batch >= 1, "quantMatvec batch must be positive, got %lld", (long long)batch);
  J4B_REQUIRE(x && y, "quantMatvec needs x and y buffers");
  J4B_REQUIRE((x & 15) == 0 && ((y | add) & 3) == 0,
              "quantMatvec needs x 16-byte aligned and y/add 4-byte aligned");
  DeviceGuard guard(w->dev);
  cudaStream_t stream = resolve_stream(w->dev, s);
  const int sms = device_ctx(w->dev)->sm_count;
  // Larger batches: one pass over the weight on the tensor cores (the fused dequant-GEMM in its
  // fp32-accurate 3-term mode) instead of a GEMV pass per 16 rows. Its cost is nearly flat in the
  // batch up to 64 rows (decode-bound), so it wins only past two or three GEMV passes. Measured
  // per call (one B200): Q4_K 14336 x 4096 GEMV 23.5 us per 16 rows, fused 81-87 us at 17-64
  // rows; Q4_0 of that shape 21.2 against 70-75 us; Q8_0 4096 x 4096 9.9 against 22-25 us.
  const int64_t fused_from = w->type == J4B_Q8_0 ? 33 : 49;
  if (batch >= fused_from && (w->type == J4B_Q8_0 || w->type == J4B_Q4_0 || w->type == J4B_Q4_K) &&
      batch <= INT32_MAX) {
    w->fresh = false;
    return quant_gemm_fused(w, (const float*)(uintptr_t)x, (float*)(uintptr_t)y,
                            add ? (const float*)(uintptr_t)add : nullptr, batch, (w->cols + 63) / 64 * 64, 3, sms,
                            stream);
  }
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
      case J4B_Q6_K: e = gemv_dispatch<J4B_Q6_K>(w, xp, ap, yp, nb, sms, stream); break;
      case J4B_Q2_0: e = gemv_dispatch<J4B_Q2_0>(w, xp, ap, yp, nb, sms, stream); break;
    }
    if (e != cudaSuccess) return cuda_error(e, "qgemv_kernel");
    count_launch();
  }
  return J4B_OK;
}

namespace j4b {
namespace {
// Device address of page-locked host memory (cudaHostAlloc / cudaMallocHost, or registered as
// mapped), or null for pageable memory.
const void* mapped_host(const void* p) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return at.type == cudaMemoryTypeHost ? at.devicePointer : nullptr;
}

// Copies n4 float4s between mapped host memory and the device staging through the SMs (one
// float4 per thread, every read in flight at once): no copy-engine round trip. Stage-in (x, host
// to device) issues its PCIe reads before it waits on the kernel before it (the previous step's
// GEMV may still read the staging); stage-out (y, device to host) waits first, since the GEMV
// before it writes what it reads, and stores whole 128-byte lines.
template <bool kIn>
__global__ void __launch_bounds__(256) host_stage_kernel(const float4* __restrict__ src, float4* __restrict__ dst,
                                                         int64_t n4) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (!kIn) asm volatile("griddepcontrol.wait;" ::: "memory");
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  if (i < n4) v = src[i];
  if (kIn) asm volatile("griddepcontrol.wait;" ::: "memory");
  if (i < n4) dst[i] = v;
}

template <bool kIn>
int launch_host_stage(const void* src, void* dst, int64_t n4, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((n4 + 255) / 256));
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  J4B_CUDA(cudaLaunchKernelEx(&cfg, host_stage_kernel<kIn>, (const float4*)src, (float4*)dst, n4),
           "host_stage_kernel");
  count_launch();
  return J4B_OK;
}
}  // namespace
}  // namespace j4b

extern "C" int j4b_quant_matvec_allgather(j4b_qweight_t w, j4b_buf x, j4b_buf add, j4b_buf y_all,
                                          int64_t batch, j4b_peer_group* g, int channel, j4b_stream s) {
  if (!w) return set_error(J4B_EINVAL, "null quantized weight");
  J4B_REQUIRE(g != nullptr, "null peer group");
  J4B_REQUIRE(batch >= 1 && batch <= 16, "all-gathered quantMatvec takes batch 1..16, got %lld", (long long)batch);
  J4B_REQUIRE(x && y_all, "quantMatvec needs x and y buffers");
  J4B_REQUIRE((x & 15) == 0 && ((y_all | add) & 3) == 0, "quantMatvec needs x 16-byte aligned");
  DeviceGuard guard(w->dev);
  cudaStream_t stream = resolve_stream(w->dev, s);
  const int nranks = peer_group_ranks(g);
  const int64_t gathered = batch * w->rows * nranks;
  GemvPeers t;
  int st = peer_gemv_targets(g, channel, (float*)(uintptr_t)y_all, gathered, &t);
  if (st) return st;
  const float* xp = (const float*)(uintptr_t)x;
  const float* ap = add ? (const float*)(uintptr_t)add : nullptr;
  const int sms = device_ctx(w->dev)->sm_count;
  cudaError_t e = cudaErrorInvalidValue;
  switch (w->type) {
    case J4B_Q8_0: e = gemv_dispatch<J4B_Q8_0>(w, xp, ap, nullptr, (int)batch, sms, stream, &t); break;
    case J4B_Q4_0: e = gemv_dispatch<J4B_Q4_0>(w, xp, ap, nullptr, (int)batch, sms, stream, &t); break;
    case J4B_Q4_K: e = gemv_dispatch<J4B_Q4_K>(w, xp, ap, nullptr, (int)batch, sms, stream, &t); break;
    case J4B_Q6_K: e = gemv_dispatch<J4B_Q6_K>(w, xp, ap, nullptr, (int)batch, sms, stream, &t); break;
    case J4B_Q2_0: e = gemv_dispatch<J4B_Q2_0>(w, xp, ap, nullptr, (int)batch, sms, stream, &t); break;
  }
  if (e != cudaSuccess) return cuda_error(e, "qgemv_kernel");
  count_launch();
  return J4B_OK;
}

// quantMatvec with host buffers: x [batch, cols] in, y [batch, rows] out, queued on the stream; the
// caller synchronises the stream before it reads y. One call per decode step from a host loop.
// Page-locked buffers are used in place: the SMs read x over PCIe into the weight's staging and
// the GEMV stores y straight into host memory (copy-engine transfers of this size cost ~14 us
// each, twice the GEMV). Pageable buffers go through stream-ordered copies.
namespace j4b {
namespace {
// Device staging of the host-buffer calls: 16 rows of x, then y (`y_floats`); allocated on first
// use, or grown (after the work still using it) for a larger gathered y.
int ensure_io(j4b_qweight* w, int64_t y_floats) {
  const int64_t xs = (w->cols + 3) / 4 * 4;  // keeps the y staging 16-byte aligned
  if (w->io_floats >= 16 * xs + y_floats) return J4B_OK;
  if (w->io) {
    cudaFree(w->io);  // synchronises with the work still using it
    counters().releases += 1;
    w->io = nullptr;
    w->io_floats = 0;
  }
  J4B_CUDA(cudaMalloc(&w->io, (size_t)(16 * xs + y_floats) * sizeof(float)), "cudaMalloc(quantMatvec staging)");
  w->io_floats = 16 * xs + y_floats;
  counters().allocations += 1;
  return J4B_OK;
}

// Where the host buffers of one host-buffer call live: page-locked ones (both, 16-byte aligned,
// whole float4s) are moved by the SMs, others by stream-ordered copies.
struct HostIo {
  const void* xd = nullptr;  // device address of x, or null
  void* yd = nullptr;        // device address of y, or null
  bool direct = false;
};
HostIo host_io(const j4b_qweight* w, const float* x, const float* y, int64_t batch, int64_t y_floats) {
  HostIo h;
  h.xd = mapped_host(x);
  h.yd = const_cast<void*>(mapped_host(y));
  h.direct = h.xd && h.yd && ((uintptr_t)h.xd & 15) == 0 && ((uintptr_t)h.yd & 15) == 0 &&
             (batch * w->cols) % 4 == 0 && y_floats % 4 == 0;
  return h;
}

// One host-buffer quantMatvec (g == null) or all-gathered quantMatvec on `stream`: x into the
// staging, the GEMV into the staging, y out. The staging must already hold y_floats.
int host_call(j4b_qweight* w, const float* x, int64_t batch, float* y, int64_t y_floats, j4b_peer_group* g,
              int channel, const HostIo& h, cudaStream_t stream) {
  const int64_t xs = (w->cols + 3) / 4 * 4;
  float* dx = w->io;
  float* dy = w->io + 16 * xs;
  const size_t xb = (size_t)(batch * w->cols) * sizeof(float), yb = (size_t)y_floats * sizeof(float);
  int st = h.direct ? launch_host_stage<true>(h.xd, dx, batch * w->cols / 4, stream)
                    : (cudaMemcpyAsync(dx, x, xb, cudaMemcpyHostToDevice, stream) == cudaSuccess
                           ? J4B_OK
                           : cuda_error(cudaGetLastError(), "cudaMemcpyAsync(HtoD)"));
  if (st) return st;
  counters().h2d += xb;
  st = g ? j4b_quant_matvec_allgather(w, (j4b_buf)(uintptr_t)dx, 0, (j4b_buf)(uintptr_t)dy, batch, g, channel,
                                      (j4b_stream)stream)
         : j4b_quant_matvec(w, (j4b_buf)(uintptr_t)dx, 0, (j4b_buf)(uintptr_t)dy, batch, (j4b_stream)stream);
  if (st) return st;
  st = h.direct ? launch_host_stage<false>(dy, h.yd, y_floats / 4, stream)
                : (cudaMemcpyAsync(y, dy, yb, cudaMemcpyDeviceToHost, stream) == cudaSuccess
                       ? J4B_OK
                       : cuda_error(cudaGetLastError(), "cudaMemcpyAsync(DtoH)"));
  if (st) return st;
  counters().d2h += yb;
  return J4B_OK;
}
}  // namespace
}  // namespace j4b

// quantMatvec with host buffers: x [batch, cols] in, y [batch, rows] out, queued on the stream; the
// caller synchronises the stream before it reads y. Page-locked buffers are moved by the SMs (a
// kernel reads x over PCIe into the weight's staging, another writes y back in whole lines):
// copy-engine transfers of this size cost ~14 us each, twice the GEMV.
extern "C" int j4b_quant_matvec_host(j4b_qweight_t w, const float* x, int64_t batch, float* y, j4b_stream s) {
  if (!w) return set_error(J4B_EINVAL, "null quantized weight");
  J4B_REQUIRE(batch >= 1 && batch <= 16, "host-buffer quantMatvec takes batch 1..16, got %lld", (long long)batch);
  J4B_REQUIRE(x && y, "quantMatvec needs x and y host buffers");
  DeviceGuard guard(w->dev);
  const int64_t n = batch * w->rows;
  int st = ensure_io(w, 16 * w->rows);
  if (st) return st;
  return host_call(w, x, batch, y, n, nullptr, 0, host_io(w, x, y, batch, n), resolve_stream(w->dev, s));
}

// The all-gathered quantMatvec with host buffers: x [batch, cols] from host memory, the gathered
// y [batch, rows * nranks] into host memory.
extern "C" int j4b_quant_matvec_allgather_host(j4b_qweight_t w, const float* x, int64_t batch, float* y_all,
                                               j4b_peer_group* g, int channel, j4b_stream s) {
  if (!w) return set_error(J4B_EINVAL, "null quantized weight");
  J4B_REQUIRE(g != nullptr, "null peer group");
  J4B_REQUIRE(batch >= 1 && batch <= 16, "all-gathered quantMatvec takes batch 1..16, got %lld", (long long)batch);
  J4B_REQUIRE(x && y_all, "quantMatvec needs x and y host buffers");
  DeviceGuard guard(w->dev);
  const int64_t n = batch * w->rows * peer_group_ranks(g);
  int st = ensure_io(w, 16 * w->rows * peer_group_ranks(g));
  if (st) return st;
  return host_call(w, x, batch, y_all, n, g, channel, host_io(w, x, y_all, batch, n), resolve_stream(w->dev, s));
}

// A host-buffer call recorded once as a CUDA graph (stage-in, GEMV, stage-out, and for a peer
// group the gathering copy) and replayed with one launch: a decode loop's per-step host cost is
// then one graph launch. The buffers, the weight and the group are captured by address and must
// outlive the plan.
struct j4b_qplan {
  int dev = 0;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  uint64_t launches = 0, h2d = 0, d2h = 0;
};

extern "C" int j4b_quant_matvec_host_plan(j4b_qweight_t w, const float* x, int64_t batch, float* y,
                                          j4b_peer_group* g, int channel, j4b_qplan_t* out) {
  if (!w) return set_error(J4B_EINVAL, "null quantized weight");
  J4B_REQUIRE(out != nullptr, "null plan pointer");
  J4B_REQUIRE(batch >= 1 && batch <= 16, "host-buffer quantMatvec takes batch 1..16, got %lld", (long long)batch);
  J4B_REQUIRE(x && y, "quantMatvec needs x and y host buffers");
  DeviceGuard guard(w->dev);
  const int nr = g ? peer_group_ranks(g) : 1;
  const int64_t n = batch * w->rows * nr;
  int st = ensure_io(w, 16 * w->rows * nr);
  if (st) return st;
  const HostIo h = host_io(w, x, y, batch, n);
  cudaStream_t cs = nullptr;
  J4B_CUDA(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking), "cudaStreamCreate(plan capture)");
  const uint64_t l0 = counters().dispatches.load(), h0 = counters().h2d.load(), d0 = counters().d2h.load();
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
  if (e == cudaSuccess) {
    st = host_call(w, x, batch, y, n, g, channel, h, cs);
    e = cudaStreamEndCapture(cs, &graph);
  }
  cudaStreamDestroy(cs);
  if (st || e != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    return st ? st : cuda_error(e, "plan capture");
  }
  j4b_qplan* p = new j4b_qplan();
  p->dev = w->dev;
  p->graph = graph;
  e = cudaGraphInstantiate(&p->exec, graph, 0);
  if (e != cudaSuccess) {
    cudaGraphDestroy(graph);
    delete p;
    return cuda_error(e, "cudaGraphInstantiate(plan)");
  }
  p->launches = counters().dispatches.load() - l0;
  p->h2d = counters().h2d.load() - h0;
  p->d2h = counters().d2h.load() - d0;
  *out = p;
  return J4B_OK;
}

extern "C" int j4b_quant_matvec_host_run(j4b_qplan_t p, j4b_stream s) {
  J4B_REQUIRE(p != nullptr, "null plan");
  J4B_CUDA(cudaGraphLaunch(p->exec, resolve_stream(p->dev, s)), "cudaGraphLaunch(plan)");
  counters().dispatches += p->launches;
  counters().h2d += p->h2d;
  counters().d2h += p->d2h;
  return J4B_OK;
}

extern "C" int j4b_quant_matvec_host_plan_free(j4b_qplan_t p) {
  if (!p) return J4B_OK;
  DeviceGuard guard(p->dev);
  cudaGraphExecDestroy(p->exec);
  cudaGraphDestroy(p->graph);
  delete p;
  return J4B_OK;
}

extern "C" int j4b_quant_gather_row(j4b_qweight_t w, int64_t row, j4b_buf out, j4b_stream s) {
  if (!w) return set_error(J4B_EINVAL, "null quantized weight");
  J4B_REQUIRE(row >= 0 && row < w->rows, "quantGatherRow row %lld out of range [0, %lld)",
              (long long)row, (long long)w->rows);
  J4B_REQUIRE(out, "quantGatherRow needs an output buffer");
  DeviceGuard guard(w->dev);
  cudaStream_t stream = resolve_stream(w->dev, s);
  gather_row_kernel<<<(unsigned)((w->cols + 255) / 256), 256, 0, stream>>>(
      layout_of(w), w->data, w->cols, row, (float*)(uintptr_t)out);
  J4B_CHECK_LAUNCH("gather_row_kernel");
  return J4B_OK;
}

// Prefill projection: y[m, rows] = x[m, cols] . W^T on the tcgen05 tensor cores. The weight is
// decoded (bit-exact) to bf16 K-major operands in stream-ordered scratch, then multiplied.
namespace j4b {
namespace {
// x -> bf16 hi (and lo) [m, kp] in stream-ordered scratch, then the fused dequant-GEMM (+ add).
// Tile shape by token count: two 256-token accumulators per CTA for long inputs (prefill), one
// for up to 256 tokens, 64-token tiles for decode-time batches; the K range is split over CTAs
// (partials in stream-ordered scratch, summed in split order by qgemm_fold_kernel) when the
// output tiles alone would leave SMs idle.
int quant_gemm_fused(const j4b_qweight* w, const float* x, float* y, const float* add, int64_t m, int64_t kp, int terms,
                     int sms, cudaStream_t stream) {
  const int nk = (int)(kp / 64);
  const int n_tiles = (int)((w->rows + kQgBM - 1) / kQgBM);
  // tokens per MMA: 64 for decode-time batches; bf16 mode 256 (one accumulator and two CTAs per
  // SM, or two accumulators for long inputs); fp32-accurate mode 128 or 2 x 128
  const int NH = m > 256 ? 2 : 1;
  const int N = m <= 64 ? 64 : (terms == 1 ? 256 : 128);
  const int64_t t_tiles = (m + (int64_t)N * NH - 1) / ((int64_t)N * NH);
  // K splits: the count (at most 9, each split at least 8 k-blocks, partials at most 24 MB) whose
  // CTAs fill the SMs' slots best over whole waves, the fewest among near-equals
  const int64_t slots = (int64_t)sms * ((terms == 1 && N * NH <= 256) ? 2 : 1);
  int splits = 1;
  double best = 0.0;
  for (int sp = 1; sp <= std::min(9, std::max(1, nk / 8)); ++sp) {
    if (sp > 1 && m * w->rows * 4 * sp > ((int64_t)24 << 20)) break;  // partials stay small next to W
    const int64_t ctas = (int64_t)n_tiles * t_tiles * sp;
    const double eff = (double)ctas / (double)(((ctas + slots - 1) / slots) * slots);
    if (eff > best + 0.02) {
      best = eff;
      splits = sp;
    }
  }
  const int kb_per = (nk + splits - 1) / splits;
  splits = (nk + kb_per - 1) / kb_per;
  const size_t xbytes = (size_t)(m * kp) * 2;
  const size_t xspan = (xbytes + 255) & ~size_t(255);
  const size_t pbytes = splits > 1 ? (size_t)splits * (size_t)(m * w->rows) * 4 : 0;
  void* scratch = nullptr;
  J4B_CUDA(cudaMallocAsync(&scratch, 2 * xspan + pbytes + 256, stream), "cudaMallocAsync(x operand)");
  __nv_bfloat16* xh = (__nv_bfloat16*)scratch;
  __nv_bfloat16* xl = terms == 3 ? (__nv_bfloat16*)((uint8_t*)scratch + xspan) : nullptr;
  float* part = splits > 1 ? (float*)((uint8_t*)scratch + 2 * xspan) : nullptr;
  int rc = tc_split_rows(x, m, w->cols, w->cols, kp, xh, xl, stream);
  CUtensorMap mh, ml;
  if (rc == J4B_OK) {
    if (!make_map(&mh, xh, m, kp, N) || (terms == 3 && !make_map(&ml, xl, m, kp, N)))
      rc = set_error(J4B_ECUDA, "cuTensorMapEncodeTiled failed for the activations");
    if (terms != 3) ml = mh;
  }
  if (rc == J4B_OK) {
    cudaError_t e = cudaErrorInvalidValue;
    const int mi = (int)m, kpi = (int)kp;
    float* out = splits > 1 ? part : y;
    const int shape = N == 64 ? 0 : (NH == 1 ? 1 : 2);
    switch ((w->type * 4 + terms) * 3 + shape) {
#define J4B_QG_CASE(QT, T, NW, NW2)                                                                                \
  case (QT * 4 + T) * 3 + 0: e = launch_qgemm_fused<QT, T, 64, 1>(w, mh, ml, mi, kpi, splits, kb_per, out, add, stream); break; \
  case (QT * 4 + T) * 3 + 1: e = launch_qgemm_fused<QT, T, NW, 1>(w, mh, ml, mi, kpi, splits, kb_per, out, add, stream); break; \
  case (QT * 4 + T) * 3 + 2: e = launch_qgemm_fused<QT, T, NW2, 2>(w, mh, ml, mi, kpi, splits, kb_per, out, add, stream); break;
      J4B_QG_CASE(J4B_Q8_0, 1, 256, 256)
      J4B_QG_CASE(J4B_Q8_0, 3, 128, 128)
      J4B_QG_CASE(J4B_Q4_0, 1, 256, 256)
      J4B_QG_CASE(J4B_Q4_0, 3, 128, 128)
      J4B_QG_CASE(J4B_Q4_K, 1, 256, 256)
      J4B_QG_CASE(J4B_Q4_K, 3, 128, 128)
#undef J4B_QG_CASE
    }
    if (e != cudaSuccess) rc = cuda_error(e, "qgemm_fused_kernel");
    else count_launch();
    if (rc == J4B_OK && splits > 1) {
      const int64_t n = m * w->rows;
      qgemm_fold_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)sms * 8), 256, 0, stream>>>(
          part, splits, n, add, y);
      cudaError_t fe = cudaGetLastError();
      if (fe != cudaSuccess) rc = cuda_error(fe, "qgemm_fold_kernel");
      else count_launch();
    }
  }
  cudaFreeAsync(scratch, stream);
  return rc;
}
}  // namespace
}  // namespace j4b

extern "C" int j4b_quant_gemm(j4b_qweight_t w, j4b_buf x, j4b_buf y, int64_t m, int precision,
                              j4b_stream s) {
  J4B_REQUIRE(w != nullptr, "null quantized matrix");
  J4B_REQUIRE(m >= 0, "negative row count");
  J4B_REQUIRE(precision >= 0 && precision <= 2, "precision must be 0, 1 or 2");
  if (m == 0) return J4B_OK;
  J4B_REQUIRE(x && y, "quant_gemm needs x and y");
  DeviceGuard guard(w->dev);
  cudaStream_t stream = resolve_stream(w->dev, s);
  const int terms = precision == 1 ? 1 : 3;
  const int64_t kp = (w->cols + 63) / 64 * 64;
  if ((w->type == J4B_Q8_0 || w->type == J4B_Q4_0 || w->type == J4B_Q4_K) && m <= INT32_MAX &&
      w->rows <= INT32_MAX)
    return quant_gemm_fused(w, (const float*)(uintptr_t)x, (float*)(uintptr_t)y, nullptr, m, kp, terms,
                            device_ctx(w->dev)->sm_count, stream);
  const size_t bytes = (size_t)(w->rows * kp) * 2;
  void* scratch = nullptr;
  J4B_CUDA(cudaMallocAsync(&scratch, 2 * bytes + 512, stream), "cudaMallocAsync(dequantised weight)");
  __nv_bfloat16* hi = (__nv_bfloat16*)scratch;
  __nv_bfloat16* lo = terms == 3 ? (__nv_bfloat16*)((uint8_t*)scratch + ((bytes + 255) & ~size_t(255))) : nullptr;
  const int64_t total = w->rows * (kp / 32);
  const unsigned grid = (unsigned)std::min<int64_t>((total + 255) / 256, 148 * 32);
  const Layout L = layout_of(w);
  switch (w->type) {
    case J4B_Q8_0: dequant_bf16_kernel<J4B_Q8_0><<<grid, 256, 0, stream>>>(L, w->data, w->rows, w->cols, kp, hi, lo); break;
    case J4B_Q4_0: dequant_bf16_kernel<J4B_Q4_0><<<grid, 256, 0, stream>>>(L, w->data, w->rows, w->cols, kp, hi, lo); break;
    case J4B_Q4_K: dequant_bf16_kernel<J4B_Q4_K><<<grid, 256, 0, stream>>>(L, w->data, w->rows, w->cols, kp, hi, lo); break;
    case J4B_Q6_K: dequant_bf16_kernel<J4B_Q6_K><<<grid, 256, 0, stream>>>(L, w->data, w->rows, w->cols, kp, hi, lo); break;
    default: dequant_bf16_kernel<J4B_Q2_0><<<grid, 256, 0, stream>>>(L, w->data, w->rows, w->cols, kp, hi, lo); break;
  }
  cudaError_t e = cudaGetLastError();
  int rc = e == cudaSuccess ? J4B_OK : cuda_error(e, "dequant_bf16_kernel");
  count_launch();
  if (rc == J4B_OK)
    rc = tc_gemm_bt((const float*)(uintptr_t)x, m, w->cols, hi, lo, w->rows, terms, (float*)(uintptr_t)y, w->dev, stream);
  cudaFreeAsync(scratch, stream);
  return rc;
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
