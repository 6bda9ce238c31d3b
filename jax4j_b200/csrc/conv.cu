// 2-D convolution: ComputeBackend.conv2d / conv2dGradInput / conv2dGradWeight
// (core/tensor/spi/ComputeBackend.java:191-200; CPU semantics core/backend/cpu/CpuBackend.java:
// 479-609). Images are NCHW flattened per row: x [batch, inC*inH*inW], weights
// [outC, inC*k*k], output [batch, outC*outH*outW]; stride and zero padding on both axes.
//
// Each call is one large GEMM on the engine's matmul (the tcgen05 tensor cores with the
// fp32-accurate 3-term bf16 split, or bf16 operands, or the SIMT kernel for small shapes) over
// patch matrices built by gather kernels, with P = outH*outW positions and K = inC*k*k taps:
//   conv2d           Y' [outC, B*P]  = W [outC, K] . Xcol [K, B*P],   then out[b][oc][p] = Y'
//   conv2dGradInput  dXcol [K, B*P]  = W^T [K, outC] . dY' [outC, B*P], then a gather over the
//                    taps that touch each input pixel (no atomics, deterministic)
//   conv2dGradWeight dW [outC, K]    = dY' [outC, B*P] . XcolT [B*P, K]
// On the tensor cores the forward runs the other way round: the patches are written straight
// into the GEMM's bf16 operand (hi and lo halves for the fp32-accurate split), K-major
// [B*P, Kp], the weights are the second operand, and C' [B*P, outC] is transposed per image.
// Scratch (patches, transposes) is stream-ordered (cudaMallocAsync) and freed after the call.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "j4b_internal.h"

namespace j4b {
namespace {

struct ConvGeom {
  int64_t B, C, H, W, O, k, s, pad, OH, OW, P, K;
};

// Xcol [K, B*P] (transposed = false) or XcolT [B*P, K]: element (tap, position) is the input
// pixel under tap (ic, kh, kw) of output position (b, oh, ow), or 0 in the padding.
__global__ void im2col_kernel(const float* __restrict__ x, ConvGeom g, bool transposed, float* __restrict__ col) {
  const int64_t total = g.K * g.B * g.P;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    int64_t tap, pos;
    if (transposed) {
      pos = idx / g.K;
      tap = idx % g.K;
    } else {
      tap = idx / (g.B * g.P);
      pos = idx % (g.B * g.P);
    }
    const int64_t b = pos / g.P, p = pos % g.P, oh = p / g.OW, ow = p % g.OW;
    const int64_t ic = tap / (g.k * g.k), kh = (tap / g.k) % g.k, kw = tap % g.k;
    const int64_t ih = oh * g.s - g.pad + kh, iw = ow * g.s - g.pad + kw;
    float v = 0.0f;
    if (ih >= 0 && ih < g.H && iw >= 0 && iw < g.W) v = __ldg(x + ((b * g.C + ic) * g.H + ih) * g.W + iw);
    col[idx] = v;
  }
}

// Patches as the bf16 GEMM operand: row = output position (b, oh, ow), 8 taps per thread, columns
// past K zero; hi = bf16(v), lo = bf16(v - hi) when lo is given.
__global__ void im2col_bf16_kernel(const float* __restrict__ x, ConvGeom g, int64_t kp, __nv_bfloat16* __restrict__ hi,
                                   __nv_bfloat16* __restrict__ lo) {
  // 32-bit index arithmetic (the host keeps B*P and K below 2^30); one division per coordinate
  // per thread, then the tap (ic, kh, kw) steps along
  const int groups = (int)(kp / 8), P = (int)g.P, OW = (int)g.OW, k = (int)g.k, kk = k * k, K = (int)g.K;
  const int H = (int)g.H, W = (int)g.W, s = (int)g.s, pad = (int)g.pad;
  const int64_t total = g.B * g.P * groups;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    const int pos = (int)(idx / groups), c0 = (int)(idx - (int64_t)pos * groups) * 8;
    const int b = pos / P, p = pos - b * P, oh = p / OW, ow = p - oh * OW;
    const float* img = x + (int64_t)b * g.C * H * W;
    int ic = c0 / kk, r = c0 - ic * kk, kh = r / k, kw = r - kh * k;
    alignas(16) __nv_bfloat16 h8[8], l8[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      float v = 0.0f;
      const int ih = oh * s - pad + kh, iw = ow * s - pad + kw;
      if (c0 + u < K && ih >= 0 && ih < H && iw >= 0 && iw < W) v = __ldg(img + ((int64_t)ic * H + ih) * W + iw);
      h8[u] = __float2bfloat16_rn(v);
      l8[u] = __float2bfloat16_rn(v - __bfloat162float(h8[u]));
      if (++kw == k) {
        kw = 0;
        if (++kh == k) {
          kh = 0;
          ++ic;
        }
      }
    }
    *reinterpret_cast<uint4*>(hi + (int64_t)pos * kp + c0) = *reinterpret_cast<const uint4*>(h8);
    if (lo) *reinterpret_cast<uint4*>(lo + (int64_t)pos * kp + c0) = *reinterpret_cast<const uint4*>(l8);
  }
}

// The same operand, one CTA per output row (b, oh). The k input rows of every channel that the
// row's windows cover are staged in shared memory with coalesced loads (zeros in the padding),
// with a table of each tap's offset into the stage (taps past K point at a zero slot); then each
// warp takes an output position and its lanes consecutive 8-tap groups, so a warp writes 512
// contiguous bytes per pass (no integer division in either phase). Shared
// memory: (C * k * Wn + 1) floats + kp ints, Wn = (OW - 1) * stride + k.
__global__ void im2col_rows_bf16_kernel(const float* __restrict__ x, ConvGeom g, int64_t kp,
                                        __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
  extern __shared__ __align__(16) float rows[];
  const int C = (int)g.C, H = (int)g.H, W = (int)g.W, k = (int)g.k, s = (int)g.s, pad = (int)g.pad;
  const int OW = (int)g.OW, OH = (int)g.OH, K = (int)g.K, kk = k * k, kpi = (int)kp;
  const int Wn = (OW - 1) * s + k, zero = C * k * Wn;
  int* tapoff = reinterpret_cast<int*>(rows + (zero + 4) / 4 * 4);  // 16-byte aligned (int4 reads)
  const int b = blockIdx.x / OH, oh = blockIdx.x - b * OH;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const float* img = x + (int64_t)b * C * H * W;
  for (int c = warp; c < C; c += nwarps)
    for (int kh = 0; kh < k; ++kh) {
      const int ih = oh * s - pad + kh;
      const bool row_in = ih >= 0 && ih < H;
      const float* src = img + ((int64_t)c * H + ih) * W;
      float* dst = rows + (c * k + kh) * Wn;
      for (int j = lane; j < Wn; j += 32) {
        const int iw = j - pad;
        dst[j] = (row_in && iw >= 0 && iw < W) ? __ldg(src + iw) : 0.0f;
      }
    }
  for (int t = threadIdx.x; t < kpi; t += blockDim.x) {
    int off = zero;
    if (t < K) {
      const int ic = t / kk, r = t - ic * kk, kh = r / k, kw = r - kh * k;
      off = (ic * k + kh) * Wn + kw;
    }
    tapoff[t] = off;
  }
  if (threadIdx.x == 0) rows[zero] = 0.0f;
  __syncthreads();
  const int groups = kpi / 8;
  const int64_t row0 = ((int64_t)b * OH + oh) * OW;
  for (int ow = warp; ow < OW; ow += nwarps) {
    const int base = ow * s;
    __nv_bfloat16* hrow = hi + (row0 + ow) * kp;
    __nv_bfloat16* lrow = lo ? lo + (row0 + ow) * kp : nullptr;
    for (int gi = lane; gi < groups; gi += 32) {
      const int c0 = gi * 8;
      const int4 o0 = *reinterpret_cast<const int4*>(tapoff + c0);
      const int4 o1 = *reinterpret_cast<const int4*>(tapoff + c0 + 4);
      const int off[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
      alignas(16) __nv_bfloat162 h4[4], l4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float v0 = rows[off[2 * u] + (off[2 * u] == zero ? 0 : base)];
        const float v1 = rows[off[2 * u + 1] + (off[2 * u + 1] == zero ? 0 : base)];
        h4[u] = __float22bfloat162_rn(make_float2(v0, v1));
        const float2 hf = __bfloat1622float2(h4[u]);
        l4[u] = __float22bfloat162_rn(make_float2(v0 - hf.x, v1 - hf.y));
      }
      *reinterpret_cast<uint4*>(hrow + c0) = *reinterpret_cast<const uint4*>(h4);
      if (lrow) *reinterpret_cast<uint4*>(lrow + c0) = *reinterpret_cast<const uint4*>(l4);
    }
  }
}

// out[b][o][p] = c[b*P + p][o]: 32 x 32 tiles through shared memory, one image per blockIdx.z.
__global__ void positions_to_channels_kernel(const float* __restrict__ c, int64_t P, int64_t O, float* __restrict__ out) {
  __shared__ float tile[32][33];
  const int64_t b = blockIdx.z, p0 = (int64_t)blockIdx.x * 32, o0 = (int64_t)blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int64_t p = p0 + r, o = o0 + threadIdx.x;
    if (p < P && o < O) tile[r][threadIdx.x] = __ldg(c + (b * P + p) * O + o);
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int64_t o = o0 + r, p = p0 + threadIdx.x;
    if (p < P && o < O) out[(b * O + o) * P + p] = tile[threadIdx.x][r];
  }
}

// [rows_a, B, P] <-> [B, rows_a, P]: out[b][r][p] = in[r][b][p] (forward) or the inverse.
__global__ void swap_outer_kernel(const float* __restrict__ in, int64_t R, int64_t B, int64_t P, bool to_batch_major,
                                  float* __restrict__ out) {
  const int64_t total = R * B * P;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    const int64_t p = idx % P;
    if (to_batch_major) {  // idx over out [B, R, P]
      const int64_t r = (idx / P) % R, b = idx / (P * R);
      out[idx] = __ldg(in + (r * B + b) * P + p);
    } else {  // idx over out [R, B, P]
      const int64_t b = (idx / P) % B, r = idx / (P * B);
      out[idx] = __ldg(in + (b * R + r) * P + p);
    }
  }
}

// dx[b][ic][ih][iw] = sum over taps (kh, kw) whose output position (oh, ow) exists of
// dXcol[(ic, kh, kw)][b*P + oh*OW + ow].
__global__ void col2im_kernel(const float* __restrict__ dcol, ConvGeom g, float* __restrict__ dx) {
  const int64_t total = g.B * g.C * g.H * g.W;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
    const int64_t iw = idx % g.W, ih = (idx / g.W) % g.H, ic = (idx / (g.W * g.H)) % g.C, b = idx / (g.W * g.H * g.C);
    float acc = 0.0f;
    for (int64_t kh = 0; kh < g.k; ++kh) {
      const int64_t hn = ih + g.pad - kh;
      if (hn < 0 || hn % g.s) continue;
      const int64_t oh = hn / g.s;
      if (oh >= g.OH) continue;
      for (int64_t kw = 0; kw < g.k; ++kw) {
        const int64_t wn = iw + g.pad - kw;
        if (wn < 0 || wn % g.s) continue;
        const int64_t ow = wn / g.s;
        if (ow >= g.OW) continue;
        acc += __ldg(dcol + ((ic * g.k + kh) * g.k + kw) * (g.B * g.P) + b * g.P + oh * g.OW + ow);
      }
    }
    dx[idx] = acc;
  }
}

// Largest per-row input stage for the shared-memory im2col (two CTAs per SM fit).
constexpr int64_t kRowStageBytes = 96 * 1024;

// Sub-buffers of one scratch allocation start on 256-byte boundaries (the GEMM stores its output
// with 16-byte vector stores).
int64_t aligned(int64_t floats) { return (floats + 63) / 64 * 64; }

unsigned grid_for(int64_t n, int dev) {
  const int sms = device_ctx(dev)->sm_count;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)sms * 16));
}

int geometry(int64_t batch, int in_c, int in_h, int in_w, int out_c, int kernel, int stride, int pad, ConvGeom* g) {
  J4B_REQUIRE(batch >= 1, "conv2d batch must be positive");
  // ConvSpec's checks (core/tensor/ConvSpec.java)
  J4B_REQUIRE(in_c >= 1 && in_h >= 1 && in_w >= 1 && out_c >= 1, "channels and spatial dims must be positive");
  J4B_REQUIRE(kernel >= 1 && stride >= 1 && pad >= 0, "kernel/stride must be positive, pad non-negative");
  J4B_REQUIRE(in_h + 2 * pad >= kernel && in_w + 2 * pad >= kernel, "kernel %d does not fit %dx%d with pad %d", kernel,
              in_h, in_w, pad);
  g->B = batch;
  g->C = in_c;
  g->H = in_h;
  g->W = in_w;
  g->O = out_c;
  g->k = kernel;
  g->s = stride;
  g->pad = pad;
  g->OH = (in_h + 2 * pad - kernel) / stride + 1;
  g->OW = (in_w + 2 * pad - kernel) / stride + 1;
  g->P = g->OH * g->OW;
  g->K = (int64_t)in_c * kernel * kernel;
  return J4B_OK;
}

// Stream-ordered scratch for one call.
struct Scratch {
  cudaStream_t st;
  void* p = nullptr;
  explicit Scratch(cudaStream_t s) : st(s) {}
  ~Scratch() {
    if (p) cudaFreeAsync(p, st);
  }
};

}  // namespace
}  // namespace j4b

using namespace j4b;

#define J4B_CONV_ARGS int64_t batch, int in_c, int in_h, int in_w, int out_c, int kernel, int stride, int pad

extern "C" int j4b_conv2d(j4b_buf x, j4b_buf w, j4b_buf out, J4B_CONV_ARGS, int precision, j4b_stream s) {
  ConvGeom g;
  int st = geometry(batch, in_c, in_h, in_w, out_c, kernel, stride, pad, &g);
  if (st) return st;
  J4B_REQUIRE(x && w && out, "conv2d needs input, weight and output buffers");
  J4B_REQUIRE(precision >= 0 && precision <= 2, "precision must be 0, 1 or 2");
  int dev = 0;
  st = device_of((const void*)(uintptr_t)out, &dev);
  if (st) return st;
  DeviceGuard guard(dev);
  cudaStream_t stream = resolve_stream(dev, s);
  const int64_t M = g.B * g.P;
  if ((precision != 0 || M * g.O * g.K >= (int64_t(1) << 24)) && M >= 128 && M < (int64_t(1) << 30) &&
      g.K < (int64_t(1) << 30)) {
    // tensor cores: bf16 patches [M, Kp] . W^T -> C' [M, O] -> out [B, O, P]
    const int terms = precision == 1 ? 1 : 3;
    const int64_t kp = (g.K + 63) / 64 * 64;
    const int64_t a_n = aligned(M * kp / 2), b_n = aligned(g.O * kp / 2);  // in floats (2 bf16 each)
    Scratch sc(stream);
    J4B_CUDA(cudaMallocAsync(&sc.p, (size_t)(2 * a_n + 2 * b_n + M * g.O) * sizeof(float), stream),
             "cudaMallocAsync(conv2d operands)");
    float* base = (float*)sc.p;
    __nv_bfloat16* ahi = (__nv_bfloat16*)base;
    __nv_bfloat16* alo = terms == 3 ? (__nv_bfloat16*)(base + a_n) : nullptr;
    __nv_bfloat16* bhi = (__nv_bfloat16*)(base + 2 * a_n);
    __nv_bfloat16* blo = terms == 3 ? (__nv_bfloat16*)(base + 2 * a_n + b_n) : nullptr;
    float* cbuf = base + 2 * a_n + 2 * b_n;
    const int64_t row_smem = (g.C * g.k * ((g.OW - 1) * g.s + g.k) + 1) * (int64_t)sizeof(float) + 16 + kp * 4;
    if (row_smem <= kRowStageBytes && g.B * g.OH <= INT32_MAX) {
      J4B_CUDA(cudaFuncSetAttribute(im2col_rows_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)kRowStageBytes),
               "cudaFuncSetAttribute(im2col_rows_bf16_kernel)");
      im2col_rows_bf16_kernel<<<(unsigned)(g.B * g.OH), 256, (size_t)row_smem, stream>>>((const float*)(uintptr_t)x, g,
                                                                                          kp, ahi, alo);
      J4B_CHECK_LAUNCH("im2col_rows_bf16_kernel");
    } else {
      im2col_bf16_kernel<<<grid_for(M * (kp / 8), dev), 256, 0, stream>>>((const float*)(uintptr_t)x, g, kp, ahi, alo);
      J4B_CHECK_LAUNCH("im2col_bf16_kernel");
    }
    st = tc_split_rows((const float*)(uintptr_t)w, g.O, g.K, g.K, kp, bhi, blo, stream);
    if (st) return st;
    st = tc_gemm_bf16(ahi, alo, M, kp, bhi, blo, g.O, terms, cbuf, dev, stream);
    if (st) return st;
    dim3 tg((unsigned)((g.P + 31) / 32), (unsigned)((g.O + 31) / 32), (unsigned)g.B);
    positions_to_channels_kernel<<<tg, dim3(32, 8), 0, stream>>>(cbuf, g.P, g.O, (float*)(uintptr_t)out);
    J4B_CHECK_LAUNCH("positions_to_channels_kernel");
    return J4B_OK;
  }
  const int64_t col_n = g.K * g.B * g.P, y_n = g.O * g.B * g.P;
  Scratch sc(stream);
  J4B_CUDA(cudaMallocAsync(&sc.p, (size_t)(aligned(col_n) + y_n) * sizeof(float), stream),
           "cudaMallocAsync(conv2d patches)");
  float* col = (float*)sc.p;
  float* y = col + aligned(col_n);
  im2col_kernel<<<grid_for(col_n, dev), 256, 0, stream>>>((const float*)(uintptr_t)x, g, false, col);
  J4B_CHECK_LAUNCH("im2col_kernel");
  st = j4b_matmul(w, (j4b_buf)(uintptr_t)col, (j4b_buf)(uintptr_t)y, 1, g.O, g.K, g.B * g.P, precision, stream);
  if (st) return st;
  swap_outer_kernel<<<grid_for(y_n, dev), 256, 0, stream>>>(y, g.O, g.B, g.P, true, (float*)(uintptr_t)out);
  J4B_CHECK_LAUNCH("swap_outer_kernel");
  return J4B_OK;
}

extern "C" int j4b_conv2d_grad_input(j4b_buf upstream, j4b_buf w, j4b_buf out, J4B_CONV_ARGS, int precision,
                                     j4b_stream s) {
  ConvGeom g;
  int st = geometry(batch, in_c, in_h, in_w, out_c, kernel, stride, pad, &g);
  if (st) return st;
  J4B_REQUIRE(upstream && w && out, "conv2dGradInput needs upstream, weight and output buffers");
  J4B_REQUIRE(precision >= 0 && precision <= 2, "precision must be 0, 1 or 2");
  int dev = 0;
  st = device_of((const void*)(uintptr_t)out, &dev);
  if (st) return st;
  DeviceGuard guard(dev);
  cudaStream_t stream = resolve_stream(dev, s);
  const int64_t dy_n = g.O * g.B * g.P, wt_n = g.K * g.O, col_n = g.K * g.B * g.P;
  Scratch sc(stream);
  J4B_CUDA(cudaMallocAsync(&sc.p, (size_t)(aligned(dy_n) + aligned(wt_n) + col_n) * sizeof(float), stream),
           "cudaMallocAsync(conv2dGradInput scratch)");
  float* dy = (float*)sc.p;
  float* wt = dy + aligned(dy_n);
  float* dcol = wt + aligned(wt_n);
  swap_outer_kernel<<<grid_for(dy_n, dev), 256, 0, stream>>>((const float*)(uintptr_t)upstream, g.O, g.B, g.P, false,
                                                               dy);
  J4B_CHECK_LAUNCH("swap_outer_kernel");
  st = j4b_transpose(w, (j4b_buf)(uintptr_t)wt, g.O, g.K, stream);
  if (st) return st;
  st = j4b_matmul((j4b_buf)(uintptr_t)wt, (j4b_buf)(uintptr_t)dy, (j4b_buf)(uintptr_t)dcol, 1, g.K, g.O, g.B * g.P,
                  precision, stream);
  if (st) return st;
  col2im_kernel<<<grid_for(g.B * g.C * g.H * g.W, dev), 256, 0, stream>>>(dcol, g, (float*)(uintptr_t)out);
  J4B_CHECK_LAUNCH("col2im_kernel");
  return J4B_OK;
}

extern "C" int j4b_conv2d_grad_weight(j4b_buf x, j4b_buf upstream, j4b_buf out, J4B_CONV_ARGS, int precision,
                                      j4b_stream s) {
  ConvGeom g;
  int st = geometry(batch, in_c, in_h, in_w, out_c, kernel, stride, pad, &g);
  if (st) return st;
  J4B_REQUIRE(x && upstream && out, "conv2dGradWeight needs input, upstream and output buffers");
  J4B_REQUIRE(precision >= 0 && precision <= 2, "precision must be 0, 1 or 2");
  int dev = 0;
  st = device_of((const void*)(uintptr_t)out, &dev);
  if (st) return st;
  DeviceGuard guard(dev);
  cudaStream_t stream = resolve_stream(dev, s);
  const int64_t dy_n = g.O * g.B * g.P, col_n = g.B * g.P * g.K;
  Scratch sc(stream);
  J4B_CUDA(cudaMallocAsync(&sc.p, (size_t)(aligned(dy_n) + col_n) * sizeof(float), stream),
           "cudaMallocAsync(conv2dGradWeight scratch)");
  float* dy = (float*)sc.p;
  float* colt = dy + aligned(dy_n);
  swap_outer_kernel<<<grid_for(dy_n, dev), 256, 0, stream>>>((const float*)(uintptr_t)upstream, g.O, g.B, g.P, false,
                                                               dy);
  J4B_CHECK_LAUNCH("swap_outer_kernel");
  im2col_kernel<<<grid_for(col_n, dev), 256, 0, stream>>>((const float*)(uintptr_t)x, g, true, colt);
  J4B_CHECK_LAUNCH("im2col_kernel");
  return j4b_matmul((j4b_buf)(uintptr_t)dy, (j4b_buf)(uintptr_t)colt, out, 1, g.O, g.B * g.P, g.K, precision, stream);
}
