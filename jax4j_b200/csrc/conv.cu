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
// Scratch (patches, transposes) is stream-ordered (cudaMallocAsync) and freed after the call.
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
