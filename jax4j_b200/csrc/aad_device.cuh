// Device helpers of the scalar-AAD replay engines. This file is compiled into the library (the
// fixed interpreter and eager kernels) and, as text, into every generated per-tape kernel
// (NVRTC), so the three engines draw identical random numbers and reduce in the same order.
// It uses no headers and only built-in types, as NVRTC requires.

#define J4B_AAD_BLOCK 256
#define J4B_AAD_WARPS (J4B_AAD_BLOCK / 32)

// AadOp ordinals (core/engine/AadOp.java:22-37).
#define J4B_AAD_CONST 0
#define J4B_AAD_INPUT 1
#define J4B_AAD_RANDN 2
#define J4B_AAD_RANDU 3
#define J4B_AAD_ADD 4
#define J4B_AAD_SUB 5
#define J4B_AAD_MUL 6
#define J4B_AAD_DIV 7
#define J4B_AAD_NEG 8
#define J4B_AAD_EXP 9
#define J4B_AAD_LOG 10
#define J4B_AAD_SQRT 11
#define J4B_AAD_MAX 12
#define J4B_AAD_MIN 13
#define J4B_AAD_ABS 14

// Philox2x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3",
// SC'11): ten rounds of (c0, c1) <- (mulhi(M, c0) ^ key ^ c1, mullo(M, c0)), key += 0x9E3779B9,
// with M = 0xD256D193, starting from key 0x1BD11BDA (core/engine/cpu/Philox.java:56-64).
__device__ __forceinline__ void j4b_philox10(unsigned int& c0, unsigned int& c1) {
  unsigned int key = 0x1BD11BDAu;
#pragma unroll
  for (int i = 0; i < 10; i++) {
    const unsigned int hi = __umulhi(0xD256D193u, c0);
    const unsigned int lo = 0xD256D193u * c0;
    c0 = hi ^ key ^ c1;
    c1 = lo;
    key += 0x9E3779B9u;
  }
}

// Two independent Philox blocks with their rounds interleaved (two dependency chains in flight
// per thread).
__device__ __forceinline__ void j4b_philox10x2(unsigned int& a0, unsigned int& a1, unsigned int& b0,
                                               unsigned int& b1) {
  unsigned int key = 0x1BD11BDAu;
#pragma unroll
  for (int i = 0; i < 10; i++) {
    const unsigned int ha = __umulhi(0xD256D193u, a0), la = 0xD256D193u * a0;
    const unsigned int hb = __umulhi(0xD256D193u, b0), lb = 0xD256D193u * b0;
    a0 = ha ^ key ^ a1;
    a1 = la;
    b0 = hb ^ key ^ b1;
    b1 = lb;
    key += 0x9E3779B9u;
  }
}

// Scenario key: lo = low word of path ^ low word of seed, hi = the high words
// (Philox.java:36-38).
__device__ __forceinline__ void j4b_scenario_key(unsigned long long path, unsigned long long seed,
                                                 unsigned int& lo, unsigned int& hi) {
  lo = (unsigned int)(path & 0xffffffffull) ^ (unsigned int)(seed & 0xffffffffull);
  hi = (unsigned int)(path >> 32) ^ (unsigned int)(seed >> 32);
}

// Standard-normal draws 2m (cosine leg) and 2m + 1 (sine leg) of a scenario: Box-Muller on the
// Philox block of counter (lo, hi ^ m), u = (c + 1/2) 2^-32, r = sqrt(-2 ln u1), angle 2 pi u2
// (Philox.java:47-63).
// FLOAT32: u1 keeps full relative precision (one rounding of c0 to 24 bits), so the radius is
// accurate however close u1 is to 0 or 1; the angle is taken as 2 pi t + pi with t = u2 - 1/2
// to 2^-24 (the top 23 bits of c1, centred), so sin and cos are evaluated on [-pi, pi], where
// the hardware approximations are accurate to 2^-21.4 absolute.
template <typename real>
__device__ __forceinline__ void j4b_box_muller(unsigned int c0, unsigned int c1, real& zc, real& zs);

template <>
__device__ __forceinline__ void j4b_box_muller<float>(unsigned int c0, unsigned int c1, float& zc, float& zs) {
  const float u1 = fmaf(__uint2float_rn(c0), 2.3283064365386963e-10f, 1.16415321826934814e-10f);
  const float t = (__uint_as_float(0x3F800000u | (c1 >> 9)) - 1.5f) + 5.9604644775390625e-8f;
  const float r = sqrtf(-2.0f * logf(u1));
  float s, c;
  __sincosf(6.283185307179586f * t, &s, &c);
  zc = -r * c;
  zs = -r * s;
}

// FLOAT64: exactly the CPU engine's formulation.
template <>
__device__ __forceinline__ void j4b_box_muller<double>(unsigned int c0, unsigned int c1, double& zc, double& zs) {
  const double u1 = ((double)c0 + 0.5) * 2.3283064365386963e-10;
  const double u2 = ((double)c1 + 0.5) * 2.3283064365386963e-10;
  const double r = sqrt(-2.0 * log(u1));
  double s, c;
  sincos(6.283185307179586 * u2, &s, &c);
  zc = r * c;
  zs = r * s;
}

template <typename real>
__device__ __forceinline__ void j4b_normal_pair(unsigned int lo, unsigned int hi, unsigned int m, real& zc, real& zs) {
  unsigned int c0 = lo, c1 = hi ^ m;
  j4b_philox10(c0, c1);
  j4b_box_muller<real>(c0, c1, zc, zs);
}

// Pairs m and m + 1 (draws 2m .. 2m + 3) from interleaved Philox blocks.
template <typename real>
__device__ __forceinline__ void j4b_normal_pair2(unsigned int lo, unsigned int hi, unsigned int m, real& zc0,
                                                 real& zs0, real& zc1, real& zs1) {
  unsigned int a0 = lo, a1 = hi ^ m, b0 = lo, b1 = hi ^ (m + 1u);
  j4b_philox10x2(a0, a1, b0, b1);
  j4b_box_muller<real>(a0, a1, zc0, zs0);
  j4b_box_muller<real>(b0, b1, zc1, zs1);
}

// Sums C per-thread double accumulators over the grid: warp shuffles, then the block's warps in
// order into partials[block][C]; the last block to arrive (ticket) sums the partials in block
// order -- a fixed order, so replays are deterministic -- and stores (or, with `accumulate`,
// adds) the totals into sums[0 .. C). The ticket is left at zero for the next launch. Called by
// every thread of the block, once.
template <int C>
__device__ __forceinline__ void j4b_aad_finish(const double (&acc)[C], int live, double* partials,
                                               unsigned int* ticket, double* sums, bool accumulate) {
  __shared__ double red[C][J4B_AAD_WARPS];
  __shared__ bool last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    double v = acc[c];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[c][warp] = v;
  }
  __syncthreads();
  const int warps = (int)(blockDim.x >> 5);  // blockDim.x is a multiple of 32, at most J4B_AAD_BLOCK
  for (int c = threadIdx.x; c < live; c += blockDim.x) {
    double s = 0.0;
    for (int w = 0; w < warps; ++w) s += red[c][w];
    partials[(unsigned long long)blockIdx.x * live + c] = s;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  if (last) {
    __threadfence();
    for (int c = threadIdx.x; c < live; c += blockDim.x) {
      double s = 0.0;
      for (unsigned int b = 0; b < gridDim.x; ++b) s += __ldcg(partials + (unsigned long long)b * live + c);
      sums[c] = accumulate ? sums[c] + s : s;
    }
    if (threadIdx.x == 0) *ticket = 0u;
  }
}
