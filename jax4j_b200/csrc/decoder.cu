// Decoder-block kernels (the Llama-style block with Q4_0 projections): row RMSNorm, RoPE with the
// f16 KV-cache append, attention over the f16 KV cache for decode (one new token per sequence) and
// causal prefill, and the SwiGLU gate. The projections themselves are the quantised GEMV / GEMM
// of quant.cu.
//
// The reference has no attention op, RoPE or KV cache (a sequence is just a tensor axis there); a
// block written with its Tensor API composes matmul, mul/add, exp, sumAxis/maxAxis and rsqrt.
// These kernels compute the same functions:
//   rmsnorm(x)[r, c] = x[r, c] / sqrt(mean_c x[r, :]^2 + eps) * g[c]
//   rope: adjacent pairs (2i, 2i+1) of each head rotated by pos * theta^(-2i / head_dim)
//   attention: softmax(q . k^T / sqrt(head_dim)) . v, causal in prefill
//   swiglu(gate, up) = gate * sigmoid(gate) * up
//
// Layouts: activations are token-major f32 [tokens, width]; the fused QKV projection output is
// [tokens, 3 * heads * head_dim] (q | k | v); the KV cache is f16 [batch, heads, capacity,
// head_dim]; rotated queries are f32 [batch, heads, seq, head_dim]; attention output is
// token-major f32 [tokens, heads * head_dim]. head_dim is 128.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>

#include "j4b_internal.h"

namespace j4b {
namespace {

constexpr int kHeadDim = 128;

// ---------------------------------------------------------------------------------------------
// RMSNorm: one CTA of 256 threads per row, float4 loads; per-thread float partial sums are
// combined in double.
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ g,
                                                      float eps, int64_t cols, float* __restrict__ out) {
  const int64_t row = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + row * cols);
  const int64_t n4 = cols / 4;
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < n4; i += 256) {
    const float4 v = xr[i];
    s = fmaf(v.x, v.x, s);
    s = fmaf(v.y, v.y, s);
    s = fmaf(v.z, v.z, s);
    s = fmaf(v.w, v.w, s);
  }
  double d = s;
  for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
  __shared__ double part[8];
  __shared__ float scale;
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = d;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < 8; ++w) t += part[w];
    scale = (float)(1.0 / sqrt(t / (double)cols + (double)eps));
  }
  __syncthreads();
  const float r = scale;
  const float4* gr = reinterpret_cast<const float4*>(g);
  float4* o = reinterpret_cast<float4*>(out + row * cols);
  for (int64_t i = threadIdx.x; i < n4; i += 256) {
    const float4 v = xr[i], w = gr[i];
    o[i] = make_float4(v.x * r * w.x, v.y * r * w.y, v.z * r * w.z, v.w * r * w.w);
  }
}

// ---------------------------------------------------------------------------------------------
// RoPE + KV append: one CTA per token (b, t) at position pos0 + t. The token's 64 rotation angles
// are formed once, in double (positions reach thousands of radians), into shared memory; the
// CTA's threads then rotate every head's (q, k) pairs and copy v.
__global__ void __launch_bounds__(256) rope_kv_kernel(const float* __restrict__ qkv, int64_t stride, int64_t seq,
                                                      int heads, int64_t pos0, double theta,
                                                      float* __restrict__ q_out, __half* __restrict__ k_cache,
                                                      __half* __restrict__ v_cache, int64_t capacity) {
  constexpr int kPairs = kHeadDim / 2;
  __shared__ float2 cs[kPairs];
  const int64_t tok = blockIdx.x;
  const int64_t b = tok / seq, t = tok % seq;
  const int64_t pos = pos0 + t;
  if (threadIdx.x < kPairs) {
    const double ang = (double)pos * pow(theta, -2.0 * threadIdx.x / kHeadDim);
    double sn, c;
    sincos(ang, &sn, &c);
    cs[threadIdx.x] = make_float2((float)c, (float)sn);
  }
  __syncthreads();
  const float* row = qkv + tok * stride;
  const int64_t width = (int64_t)heads * kHeadDim;
  for (int idx = threadIdx.x; idx < heads * kPairs; idx += blockDim.x) {
    const int h = idx / kPairs, i = idx % kPairs;
    const float c = cs[i].x, s = cs[i].y;
    const int col = h * kHeadDim + 2 * i;
    const float2 q = *reinterpret_cast<const float2*>(row + col);
    const float2 k = *reinterpret_cast<const float2*>(row + width + col);
    const float2 v = *reinterpret_cast<const float2*>(row + 2 * width + col);
    const int64_t qo = ((b * heads + h) * seq + t) * kHeadDim + 2 * i;
    *reinterpret_cast<float2*>(q_out + qo) = make_float2(q.x * c - q.y * s, q.x * s + q.y * c);
    const int64_t co = ((b * heads + h) * capacity + pos) * kHeadDim + 2 * i;
    *reinterpret_cast<__half2*>(k_cache + co) = __floats2half2_rn(k.x * c - k.y * s, k.x * s + k.y * c);
    *reinterpret_cast<__half2*>(v_cache + co) = __floats2half2_rn(v.x, v.y);
  }
}

// ---------------------------------------------------------------------------------------------
// Decode attention: one CTA of 4 warps per (sequence, head). A half-warp owns a token at a time
// (16 lanes x 8 dims = one 256-byte key row), so a warp's loads cover 512 contiguous bytes; each
// half-warp keeps its own online-softmax state (max, sum, 8 output dims per lane) over the tokens
// it visits, four at a time, and the 8 half-warps are merged at the end.
constexpr int kDecWarps = 4;
constexpr int kDecUnroll = 4;  // tokens per half-warp per step

__device__ __forceinline__ void h8_to_f(const uint4& u, float (&f)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 p = __half22float2(h[i]);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}

// With gridDim.y > 1 the token range is split: CTA (bh, s) covers tokens [s chunk, (s+1) chunk)
// and writes its unnormalised state (max, sum, 128 output dims) to part[(bh * splits + s) * 130]
// for attn_combine_kernel; with one split it writes the normalised output.
__global__ void __launch_bounds__(kDecWarps * 32) attn_decode_kernel(const float* __restrict__ q, const __half* __restrict__ kc,
                                                                    const __half* __restrict__ vc, int heads,
                                                                    int64_t capacity, int64_t len, int64_t chunk,
                                                                    float scale_log2, float* __restrict__ out,
                                                                    float* __restrict__ part) {
  const int bh = blockIdx.x;  // b * heads + h
  const int64_t t_begin = (int64_t)blockIdx.y * chunk;
  const int64_t t_end = min(len, t_begin + chunk);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int half = lane >> 4, sub = lane & 15;
  const float* qp = q + (int64_t)bh * kHeadDim + sub * 8;
  float qv[8];
  {
    const float4 a = *reinterpret_cast<const float4*>(qp), b = *reinterpret_cast<const float4*>(qp + 4);
    qv[0] = a.x * scale_log2; qv[1] = a.y * scale_log2; qv[2] = a.z * scale_log2; qv[3] = a.w * scale_log2;
    qv[4] = b.x * scale_log2; qv[5] = b.y * scale_log2; qv[6] = b.z * scale_log2; qv[7] = b.w * scale_log2;
  }
  const __half* kb = kc + ((int64_t)bh * capacity + t_begin) * kHeadDim + sub * 8;
  const __half* vb = vc + ((int64_t)bh * capacity + t_begin) * kHeadDim + sub * 8;
  const int64_t n_tok = t_end - t_begin;
  float m = -INFINITY, l = 0.f, acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  // token of (step, u) for this half-warp: ((step * kDecUnroll + u) * kDecWarps + warp) * 2 + half
  const int64_t per_step = (int64_t)kDecUnroll * kDecWarps * 2;
  for (int64_t base = 0; base < n_tok; base += per_step) {
    uint4 kr[kDecUnroll], vr[kDecUnroll];
    bool ok[kDecUnroll];
#pragma unroll
    for (int u = 0; u < kDecUnroll; ++u) {
      const int64_t tk = base + ((int64_t)u * kDecWarps + warp) * 2 + half;
      ok[u] = tk < n_tok;
      const int64_t off = (ok[u] ? tk : 0) * kHeadDim;
      kr[u] = __ldg(reinterpret_cast<const uint4*>(kb + off));
      vr[u] = __ldg(reinterpret_cast<const uint4*>(vb + off));
    }
    float sc[kDecUnroll];
#pragma unroll
    for (int u = 0; u < kDecUnroll; ++u) {
      float kf[8];
      h8_to_f(kr[u], kf);
      float d = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) d = fmaf(qv[i], kf[i], d);
      d += __shfl_xor_sync(0xffffffffu, d, 8);
      d += __shfl_xor_sync(0xffffffffu, d, 4);
      d += __shfl_xor_sync(0xffffffffu, d, 2);
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      sc[u] = ok[u] ? d : -INFINITY;
    }
    float mn = m;
#pragma unroll
    for (int u = 0; u < kDecUnroll; ++u) mn = fmaxf(mn, sc[u]);
    const bool any = mn != -INFINITY;  // false only before this half-warp's first valid token
    const float corr = any ? exp2f(m - mn) : 1.f;
    l *= corr;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] *= corr;
#pragma unroll
    for (int u = 0; u < kDecUnroll; ++u) {
      const float p = any ? exp2f(sc[u] - mn) : 0.f;
      l += p;
      float vf[8];
      h8_to_f(vr[u], vf);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(p, vf[i], acc[i]);
    }
    if (any) m = mn;
  }
  // merge the 8 half-warps: (m, l) per half-warp, acc per half-warp and dim
  __shared__ float sm_m[kDecWarps * 2], sm_l[kDecWarps * 2];
  __shared__ float sm_acc[kDecWarps * 2][kHeadDim];
  const int hw = warp * 2 + half;
  if (sub == 0) {
    sm_m[hw] = m;
    sm_l[hw] = l;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) sm_acc[hw][sub * 8 + i] = acc[i];
  __syncthreads();
  const int d = threadIdx.x;  // 128 threads = 128 dims
  float mt = -INFINITY;
  for (int w = 0; w < kDecWarps * 2; ++w) mt = fmaxf(mt, sm_m[w]);
  float lt = 0.f, ot = 0.f;
  for (int w = 0; w < kDecWarps * 2; ++w) {
    if (sm_m[w] == -INFINITY) continue;
    const float f = exp2f(sm_m[w] - mt);
    lt = fmaf(sm_l[w], f, lt);
    ot = fmaf(sm_acc[w][d], f, ot);
  }
  if (gridDim.y == 1) {
    // out is token-major [batch, heads * head_dim]: (b, h) maps to row b, column block h
    out[(int64_t)bh * kHeadDim + d] = ot / lt;
  } else {
    float* p = part + ((int64_t)bh * gridDim.y + blockIdx.y) * (kHeadDim + 2);
    p[2 + d] = ot;
    if (d == 0) {
      p[0] = mt;
      p[1] = lt;
    }
  }
}

// Merges the split states of one (sequence, head) in split order.
__global__ void __launch_bounds__(kHeadDim) attn_combine_kernel(const float* __restrict__ part, int splits,
                                                              float* __restrict__ out) {
  const int bh = blockIdx.x, d = threadIdx.x;
  const float* p = part + (int64_t)bh * splits * (kHeadDim + 2);
  float mt = -INFINITY;
  for (int s = 0; s < splits; ++s) mt = fmaxf(mt, p[s * (kHeadDim + 2)]);
  float lt = 0.f, ot = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float* ps = p + s * (kHeadDim + 2);
    const float f = exp2f(ps[0] - mt);
    lt = fmaf(ps[1], f, lt);
    ot = fmaf(ps[2 + d], f, ot);
  }
  out[(int64_t)bh * kHeadDim + d] = ot / lt;
}

// ---------------------------------------------------------------------------------------------
// Causal prefill attention, flash-attention style on mma.sync m16n8k16 (f16 operands, f32
// accumulation): a CTA of 4 warps owns 64 queries of one (sequence, head); each warp 16 of them.
// Keys and values stream through double-buffered 64-token shared-memory tiles (cp.async 16-byte
// copies); S = Q K^T stays in registers, the online softmax runs on the accumulators, and P is
// re-packed from the accumulator layout straight into A fragments for O += P V. Rows of 128 f16
// (256 bytes) are stored with their 16-byte chunks XOR-swizzled by (row & 7), so the 8-row
// ldmatrix reads hit distinct banks.
constexpr int kBr = 64, kBc = 64;
constexpr int kRowBytes = kHeadDim * 2;
constexpr int kTileBytes = kBr * kRowBytes;  // 16 KB

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint32_t swz(int row, int chunk) {  // byte offset of (row, 16-byte chunk)
  return (uint32_t)(row * kRowBytes + ((chunk ^ (row & 7)) << 4));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__global__ void __launch_bounds__(128) attn_prefill_kernel(const float* __restrict__ q, const __half* __restrict__ kc,
                                                         const __half* __restrict__ vc, int heads, int64_t capacity,
                                                         int64_t seq, float scale_log2, float* __restrict__ out) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sq = smem;                    // Q tile
  uint8_t* skv = smem + kTileBytes;      // [2 stages][K tile | V tile]
  const int nq = (int)(seq / kBr);
  const int qi = nq - 1 - (int)blockIdx.x;  // heaviest (longest causal range) tiles first
  const int bh = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const float* qg = q + ((int64_t)bh * seq + (int64_t)qi * kBr) * kHeadDim;
  const __half* kg = kc + (int64_t)bh * capacity * kHeadDim;
  const __half* vg = vc + (int64_t)bh * capacity * kHeadDim;

  auto load_kv = [&](int j, int stage) {
    uint8_t* sk = skv + stage * 2 * kTileBytes;
    uint8_t* sv = sk + kTileBytes;
    const __half* ks = kg + (int64_t)j * kBc * kHeadDim;
    const __half* vs = vg + (int64_t)j * kBc * kHeadDim;
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int c = tid + it * 128, row = c >> 4, ch = c & 15;
      cp_async16(smem_addr(sk) + swz(row, ch), ks + row * kHeadDim + ch * 8);
      cp_async16(smem_addr(sv) + swz(row, ch), vs + row * kHeadDim + ch * 8);
    }
    cp_commit();
  };
  load_kv(0, 0);
  // Q tile: f32 -> f16, swizzled
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int c = tid + it * 128, row = c >> 4, ch = c & 15;
    const float4 a = *reinterpret_cast<const float4*>(qg + row * kHeadDim + ch * 8);
    const float4 b = *reinterpret_cast<const float4*>(qg + row * kHeadDim + ch * 8 + 4);
    uint4 h;
    h.x = pack_h2(a.x, a.y);
    h.y = pack_h2(a.z, a.w);
    h.z = pack_h2(b.x, b.y);
    h.w = pack_h2(b.z, b.w);
    *reinterpret_cast<uint4*>(sq + swz(row, ch)) = h;
  }
  __syncthreads();
  // Q fragments of this warp's 16 rows, all 8 k-steps
  uint32_t qa[8][4];
  {
    const int row = warp * 16 + (lane & 15);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) ldsm_x4(smem_addr(sq) + swz(row, 2 * ks + (lane >> 4)), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
  }
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const int q0 = qi * kBr + warp * 16 + g;  // query of accumulator rows g (and g + 8)

  for (int j = 0; j <= qi; ++j) {
    const int stage = j & 1;
    if (j < qi) {
      load_kv(j + 1, stage ^ 1);
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const uint8_t* sk = skv + stage * 2 * kTileBytes;
    const uint8_t* sv = sk + kTileBytes;
    // S = Q K^T for 16 queries x 64 keys
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int n = 0; n < 8; n += 2) {
        uint32_t b0, b1, b2, b3;
        const int krow = n * 8 + (lane & 7) + ((lane >> 4) << 3);
        ldsm_x4(smem_addr(sk) + swz(krow, 2 * ks + ((lane >> 3) & 1)), b0, b1, b2, b3);
        mma_f16(s[n], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
        mma_f16(s[n + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
      }
    }
    // scale, causal mask on the diagonal tile, online softmax
    float mx[2] = {mrow[0], mrow[1]};
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = s[n][e] * scale_log2;
        if (j == qi) {
          const int key = j * kBc + n * 8 + 2 * t + (e & 1);
          const int qq = q0 + ((e >> 1) << 3);
          if (key > qq) v = -INFINITY;
        }
        s[n][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      corr[r] = exp2f(mrow[r] - mx[r]);  // mrow = -inf on the first tile: corr = 0
      mrow[r] = mx[r];
      lrow[r] *= corr[r];
    }
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= corr[0];
      o[n][1] *= corr[0];
      o[n][2] *= corr[1];
      o[n][3] *= corr[1];
    }
    uint32_t pa[4][4];  // P as A fragments, one per 16-key step
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float p0 = exp2f(s[n][0] - mx[0]), p1 = exp2f(s[n][1] - mx[0]);
      const float p2 = exp2f(s[n][2] - mx[1]), p3 = exp2f(s[n][3] - mx[1]);
      lrow[0] += p0 + p1;
      lrow[1] += p2 + p3;
      pa[n >> 1][(n & 1) * 2 + 0] = pack_h2(p0, p1);
      pa[n >> 1][(n & 1) * 2 + 1] = pack_h2(p2, p3);
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int n = 0; n < 16; n += 2) {
        uint32_t b0, b1, b2, b3;
        const int vrow = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        ldsm_x4_t(smem_addr(sv) + swz(vrow, n + (lane >> 4)), b0, b1, b2, b3);
        mma_f16(o[n], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b0, b1);
        mma_f16(o[n + 1], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b2, b3);
      }
    }
    __syncthreads();  // the stage is refilled in the next iteration
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
  }
  const float inv0 = 1.f / lrow[0], inv1 = 1.f / lrow[1];
  const int b = bh / heads, h = bh % heads;
  const int64_t width = (int64_t)heads * kHeadDim;
  float* o0 = out + ((int64_t)b * seq + q0) * width + h * kHeadDim + 2 * t;
  float* o1 = o0 + 8 * width;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    *reinterpret_cast<float2*>(o0 + n * 8) = make_float2(o[n][0] * inv0, o[n][1] * inv0);
    *reinterpret_cast<float2*>(o1 + n * 8) = make_float2(o[n][2] * inv1, o[n][3] * inv1);
  }
}

// ---------------------------------------------------------------------------------------------
// SwiGLU over a fused [rows, 2 * width] gate|up buffer -> [rows, width]: blockIdx.y strides the
// rows, threads take float4s of a row (width % 4 == 0 and 16-byte aligned rows) or single floats.
__global__ void swiglu_kernel(const float* __restrict__ gu, int64_t rows, int64_t width, bool vec,
                              float* __restrict__ out) {
  const int64_t n = vec ? width / 4 : width;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const float* g = gu + r * 2 * width;
    const float* u = g + width;
    float* o = out + r * width;
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < n; c += (int64_t)gridDim.x * blockDim.x) {
      if (vec) {
        const float4 a = reinterpret_cast<const float4*>(g)[c], b = reinterpret_cast<const float4*>(u)[c];
        reinterpret_cast<float4*>(o)[c] =
            make_float4(a.x / (1.0f + expf(-a.x)) * b.x, a.y / (1.0f + expf(-a.y)) * b.y,
                        a.z / (1.0f + expf(-a.z)) * b.z, a.w / (1.0f + expf(-a.w)) * b.w);
      } else {
        o[c] = g[c] / (1.0f + expf(-g[c])) * u[c];
      }
    }
  }
}

}  // namespace
}  // namespace j4b

using namespace j4b;

#define J4B_DEV_OF(ptr)                                             \
  int dev = 0;                                                      \
  {                                                                 \
    int st_ = device_of((const void*)(uintptr_t)(ptr), &dev);       \
    if (st_) return st_;                                            \
  }                                                                 \
  DeviceGuard guard_(dev);                                          \
  cudaStream_t stream = resolve_stream(dev, s)

extern "C" int j4b_rmsnorm(j4b_buf x, j4b_buf g, float eps, int64_t rows, int64_t cols, j4b_buf out, j4b_stream s) {
  J4B_REQUIRE(rows >= 0 && cols > 0 && cols % 4 == 0, "rmsnorm needs cols a positive multiple of 4, got %lld",
              (long long)cols);
  J4B_REQUIRE(x && g && out && ((x | g | out) & 15) == 0, "rmsnorm needs 16-byte aligned buffers");
  J4B_REQUIRE(eps >= 0.f, "rmsnorm eps must be non-negative");
  if (rows == 0) return J4B_OK;
  J4B_REQUIRE(rows <= 0x7fffffffLL, "rmsnorm: too many rows");
  J4B_DEV_OF(out);
  rmsnorm_kernel<<<(unsigned)rows, 256, 0, stream>>>((const float*)(uintptr_t)x, (const float*)(uintptr_t)g, eps,
                                                       cols, (float*)(uintptr_t)out);
  J4B_CHECK_LAUNCH("rmsnorm_kernel");
  return J4B_OK;
}

extern "C" int j4b_rope_kv(j4b_buf qkv, int64_t batch, int64_t seq, int64_t heads, int64_t head_dim, int64_t pos0,
                           double theta, j4b_buf q_out, j4b_buf k_cache, j4b_buf v_cache, int64_t capacity,
                           j4b_stream s) {
  J4B_REQUIRE(head_dim == kHeadDim, "rope/attention kernels take head_dim 128, got %lld", (long long)head_dim);
  J4B_REQUIRE(batch > 0 && seq > 0 && heads > 0 && heads <= 4096, "rope: bad batch/seq/heads");
  J4B_REQUIRE(pos0 >= 0 && pos0 + seq <= capacity, "rope: positions [%lld, %lld) exceed the cache capacity %lld",
              (long long)pos0, (long long)(pos0 + seq), (long long)capacity);
  J4B_REQUIRE(theta > 0.0, "rope theta must be positive");
  J4B_REQUIRE(qkv && q_out && k_cache && v_cache && ((qkv | q_out) & 7) == 0 && ((k_cache | v_cache) & 3) == 0,
              "rope: misaligned buffers");
  J4B_DEV_OF(q_out);
  J4B_REQUIRE(batch * seq <= 0x7fffffffLL, "rope: too many tokens");
  rope_kv_kernel<<<(unsigned)(batch * seq), 256, 0, stream>>>(
      (const float*)(uintptr_t)qkv, 3 * heads * kHeadDim, seq, (int)heads, pos0, theta, (float*)(uintptr_t)q_out,
      (__half*)(uintptr_t)k_cache, (__half*)(uintptr_t)v_cache, capacity);
  J4B_CHECK_LAUNCH("rope_kv_kernel");
  return J4B_OK;
}

extern "C" int j4b_attention_decode(j4b_buf q, j4b_buf k_cache, j4b_buf v_cache, int64_t batch, int64_t heads,
                                    int64_t head_dim, int64_t capacity, int64_t length, j4b_buf out, j4b_stream s) {
  J4B_REQUIRE(head_dim == kHeadDim, "attention kernels take head_dim 128, got %lld", (long long)head_dim);
  J4B_REQUIRE(batch > 0 && heads > 0 && batch * heads <= 0x7fffffffLL, "attention: bad batch/heads");
  J4B_REQUIRE(length >= 1 && length <= capacity, "attention: length %lld outside [1, capacity %lld]", (long long)length,
              (long long)capacity);
  J4B_REQUIRE(q && k_cache && v_cache && out && ((q | k_cache | v_cache | out) & 15) == 0,
              "attention needs 16-byte aligned buffers");
  J4B_DEV_OF(out);
  const float scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)kHeadDim));
  // One CTA per (sequence, head) streams the cache at full bandwidth once there are enough of
  // them (batch 64 x 32 heads: ~14 per SM); fewer are split along the tokens (at least 256 per
  // split) to about 16 CTAs per SM, and their states merged by a second kernel.
  const int64_t pairs = batch * heads;
  const int sms = device_ctx(dev) ? device_ctx(dev)->sm_count : 148;
  int64_t splits = 1;
  if (pairs < 8LL * sms) {
    splits = std::min<int64_t>((16LL * sms + pairs - 1) / pairs, (length + 255) / 256);
    splits = std::max<int64_t>(1, std::min<int64_t>(splits, 64));
  }
  const int64_t chunk = (length + splits - 1) / splits;
  splits = (length + chunk - 1) / chunk;  // every split holds at least one token
  float* part = nullptr;
  if (splits > 1)
    J4B_CUDA(cudaMallocAsync((void**)&part, (size_t)(pairs * splits * (kHeadDim + 2)) * sizeof(float), stream),
             "cudaMallocAsync(attention split state)");
  attn_decode_kernel<<<dim3((unsigned)pairs, (unsigned)splits), kDecWarps * 32, 0, stream>>>(
      (const float*)(uintptr_t)q, (const __half*)(uintptr_t)k_cache, (const __half*)(uintptr_t)v_cache, (int)heads,
      capacity, length, chunk, scale_log2, (float*)(uintptr_t)out, part);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess && splits > 1) {
    count_launch();
    attn_combine_kernel<<<(unsigned)pairs, kHeadDim, 0, stream>>>(part, (int)splits, (float*)(uintptr_t)out);
    e = cudaGetLastError();
  }
  if (part) cudaFreeAsync(part, stream);
  if (e != cudaSuccess) return cuda_error(e, "attn_decode_kernel");
  count_launch();
  return J4B_OK;
}

extern "C" int j4b_attention_prefill(j4b_buf q, j4b_buf k_cache, j4b_buf v_cache, int64_t batch, int64_t heads,
                                     int64_t head_dim, int64_t capacity, int64_t seq, j4b_buf out, j4b_stream s) {
  J4B_REQUIRE(head_dim == kHeadDim, "attention kernels take head_dim 128, got %lld", (long long)head_dim);
  J4B_REQUIRE(batch > 0 && heads > 0 && batch * heads <= 65535, "attention prefill: batch * heads must be <= 65535");
  J4B_REQUIRE(seq > 0 && seq % kBr == 0 && seq <= capacity, "attention prefill: seq must be a multiple of 64 and <= capacity");
  J4B_REQUIRE(q && k_cache && v_cache && out && ((q | k_cache | v_cache | out) & 15) == 0,
              "attention needs 16-byte aligned buffers");
  J4B_DEV_OF(out);
  const int smem = 5 * kTileBytes;  // Q + 2 stages of K and V
  static bool attr_set[kMaxDevices] = {};
  if (!attr_set[dev]) {
    J4B_CUDA(cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
             "cudaFuncSetAttribute");
    attr_set[dev] = true;
  }
  const float scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)kHeadDim));
  attn_prefill_kernel<<<dim3((unsigned)(seq / kBr), (unsigned)(batch * heads)), 128, smem, stream>>>(
      (const float*)(uintptr_t)q, (const __half*)(uintptr_t)k_cache, (const __half*)(uintptr_t)v_cache, (int)heads,
      capacity, seq, scale_log2, (float*)(uintptr_t)out);
  J4B_CHECK_LAUNCH("attn_prefill_kernel");
  return J4B_OK;
}

extern "C" int j4b_swiglu(j4b_buf gate_up, int64_t rows, int64_t width, j4b_buf out, j4b_stream s) {
  J4B_REQUIRE(rows >= 0 && width > 0, "swiglu: bad shape");
  J4B_REQUIRE(gate_up && out && ((gate_up | out) & 3) == 0, "swiglu: misaligned buffers");
  if (rows == 0) return J4B_OK;
  J4B_DEV_OF(out);
  const bool vec = width % 4 == 0 && ((gate_up | out) & 15) == 0;
  const int64_t per_row = vec ? width / 4 : width;
  const unsigned gx = (unsigned)std::min<int64_t>((per_row + 255) / 256, 64);
  const unsigned gy = (unsigned)std::min<int64_t>(rows, 65535);
  swiglu_kernel<<<dim3(gx, gy), 256, 0, stream>>>((const float*)(uintptr_t)gate_up, rows, width, vec,
                                                  (float*)(uintptr_t)out);
  J4B_CHECK_LAUNCH("swiglu_kernel");
  return J4B_OK;
}
