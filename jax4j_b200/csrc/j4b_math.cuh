// Scalar semantics shared by the eager SPI kernels and the fused-tape code generator.
//
// Binary/unary ops follow the reference's CPU backend (core/backend/cpu/CpuBackend.java:61-167,
// 657-682): java.lang.Math.max/min (NaN propagates, +0.0 > -0.0), sign() returning -1/0/1, relu as
// Math.max(0f, x). Transcendentals use CUDA's single-precision library functions (expf, logf,
// tanhf: a few ulp) where the reference evaluates in double and rounds to float; results agree
// within the engine's fp32 tolerance, not bit-for-bit.
#pragma once

#include <cuda_runtime.h>
#include <math.h>

namespace j4b {

__device__ __forceinline__ float java_max(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == 0.0f && b == 0.0f) return signbit(a) ? b : a;
  return a >= b ? a : b;
}

__device__ __forceinline__ float java_min(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == 0.0f && b == 0.0f) return signbit(a) ? a : b;
  return a <= b ? a : b;
}

__device__ __forceinline__ float apply_binary(int op, float x, float y) {
  switch (op) {
    case J4B_ADD: return __fadd_rn(x, y);
    case J4B_SUB: return __fsub_rn(x, y);
    case J4B_MUL: return __fmul_rn(x, y);
    case J4B_DIV: return __fdiv_rn(x, y);
    case J4B_MAX: return java_max(x, y);
    case J4B_MIN: return java_min(x, y);
  }
  return __int_as_float(0x7fc00000);
}

__device__ __forceinline__ float apply_unary(int op, float x) {
  switch (op) {
    case J4B_NEG: return -x;
    case J4B_EXP: return expf(x);
    case J4B_LOG: return logf(x);
    case J4B_SQRT: return __fsqrt_rn(x);
    case J4B_RSQRT: return __fdiv_rn(1.0f, __fsqrt_rn(x));
    case J4B_TANH: return tanhf(x);
    case J4B_SIGMOID: return __fdiv_rn(1.0f, 1.0f + expf(-x));
    case J4B_RELU: return java_max(0.0f, x);
    case J4B_ABS: return fabsf(x);
    case J4B_SIGN: return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f);
  }
  return __int_as_float(0x7fc00000);
}

}  // namespace j4b
