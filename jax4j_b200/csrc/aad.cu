// Scalar-AAD Monte-Carlo replay engines (the AadEngine SPI, core/engine/AadEngine.java:29-75):
// a recorded scalar tape -- constants, inputs, standard-normal draws and the 11 arithmetic ops
// of core/engine/AadOp.java -- is replayed for many independent scenarios ("paths"), each a
// forward sweep and, with adjoints, a reverse sweep; the replay returns sums over the paths of
// the output, its square and the adjoint of every input.
//
// Three engines share the tape format, the random numbers and the reduction:
//   * generated (the reference's `cuda`, AadKernel.java / CudaAadCodegen.java:39-101): CUDA C
//     emitted per tape -- the whole forward and reverse sweep unrolled into registers, one
//     scenario per thread in a grid-stride loop -- compiled for sm_100a by NVRTC (multiply-adds
//     fused) and cached by source text. Both legs of each Box-Muller pair are used (one Philox
//     block per two draws).
//   * interpreter (`cuda-interp`, CudaInterpExecutable.java, CudaTapeKernels.java:110-250): one
//     fixed kernel, compiled with the library, walks the tape as data; node values and adjoints
//     live in [node][thread] scratch so a warp's accesses coalesce.
//   * eager (`cuda-eager`, CudaEagerExecutable.java): one launch per node over an array of
//     scenarios, chunked to a scratch budget -- the unfused bound.
// Every engine sums per-thread double accumulators with warp shuffles and a fixed-order
// last-block fold (aad_device.cuh), so one replay is one D2H of 2 + inputs doubles and is
// deterministic. Random draws: RANDN node with ordinal k uses Philox counter k / 2, cosine leg
// for even k (Philox.java:47-63). Uniform draws and named streams are declined, as by the
// reference's CUDA engines (AadEngine.requireBasicRandom).
#include <cuda.h>

#include <algorithm>
#include <chrono>
#include <queue>
#include <cmath>
#include <cstring>
#include <sstream>
#include <string>
#include <vector>

#include "j4b_internal.h"
#include "j4b_rtc.h"
#include "aad_device.cuh"

namespace j4b {
namespace {

// The same helpers as text, prepended to every generated kernel.
const char* kAadDeviceSource =
#include "aad_device.inc"
    ;

constexpr int kInterpMaxInputs = 32;  // CudaTapeKernels.MAX_INPUTS
constexpr int kInterpChannels = 2 + kInterpMaxInputs;
constexpr int64_t kEagerDefaultBytes = 700ll << 20;  // CudaEagerExecutable.BUDGET_BYTES
constexpr int64_t kInterpL2Budget = 96ll << 20;      // interpreter scratch kept within L2

__host__ __device__ inline bool is_unary(int op) {
  return op == J4B_AAD_NEG || op == J4B_AAD_EXP || op == J4B_AAD_LOG || op == J4B_AAD_SQRT || op == J4B_AAD_ABS;
}
__host__ __device__ inline bool is_binary(int op) {
  return (op >= J4B_AAD_ADD && op <= J4B_AAD_DIV) || op == J4B_AAD_MAX || op == J4B_AAD_MIN;
}

// ---------------------------------------------------------------------------------------------
// interpreter. The tape is planned on the host into slots: a value occupies a slot from its
// definition to its last use (forward operand, reverse-sweep operand, or the output read), an
// adjoint from its first contribution (an assignment, so no slot is ever cleared) to the node's
// own reverse step; slots are reused by linear scan. Per-thread state is (value + adjoint slots)
// x element size, which for most tapes fits shared memory ([slot][thread], conflict-free);
// larger tapes use the same layout in global memory. Two int4 per node:
//   r0 = {op | flags << 8, value slot (-1: never read), slot of a (leaf: aux), slot of b}
//   r1 = {adjoint slot of the node, adjoint slot of a (-1: none), of b, unused}
// flags: 1 = swept in the reverse pass, 2 = first contribution to a, 4 = first to b;
// aux: CONST constant index, INPUT input index, RANDN draw ordinal.
// ---------------------------------------------------------------------------------------------
template <typename real>
__device__ __forceinline__ real unary_fwd(int op, real x);
template <>
__device__ __forceinline__ float unary_fwd<float>(int op, float x) {
  switch (op) {
    case J4B_AAD_NEG: return -x;
    case J4B_AAD_EXP: return expf(x);
    case J4B_AAD_LOG: return logf(x);
    case J4B_AAD_SQRT: return sqrtf(x);
    default: return fabsf(x);
  }
}
template <>
__device__ __forceinline__ double unary_fwd<double>(int op, double x) {
  switch (op) {
    case J4B_AAD_NEG: return -x;
    case J4B_AAD_EXP: return exp(x);
    case J4B_AAD_LOG: return log(x);
    case J4B_AAD_SQRT: return sqrt(x);
    default: return fabs(x);
  }
}
template <typename real>
__device__ __forceinline__ real binary_fwd(int op, real x, real y) {
  switch (op) {
    case J4B_AAD_ADD: return x + y;
    case J4B_AAD_SUB: return x - y;
    case J4B_AAD_MUL: return x * y;
    case J4B_AAD_DIV: return x / y;
    case J4B_AAD_MAX: return fmax(x, y);
    default: return fmin(x, y);
  }
}

// Adjoint contributions of node i (value vi, adjoint adj) to its arguments (eager engine).
template <typename real>
__device__ __forceinline__ void node_adjoint(int op, real va, real vb, real vi, real adj, real& ga, real& gb) {
  ga = 0;
  gb = 0;
  switch (op) {
    case J4B_AAD_ADD: ga = adj; gb = adj; break;
    case J4B_AAD_SUB: ga = adj; gb = -adj; break;
    case J4B_AAD_MUL: ga = adj * vb; gb = adj * va; break;
    case J4B_AAD_DIV: ga = adj / vb; gb = -(adj * vi / vb); break;
    case J4B_AAD_NEG: ga = -adj; break;
    case J4B_AAD_EXP: ga = adj * vi; break;
    case J4B_AAD_LOG: ga = adj / va; break;
    case J4B_AAD_SQRT: ga = adj * (real)0.5 / vi; break;
    case J4B_AAD_ABS: ga = va < (real)0 ? -adj : adj; break;
    case J4B_AAD_MAX: if (va >= vb) ga = adj; else gb = adj; break;
    case J4B_AAD_MIN: if (va <= vb) ga = adj; else gb = adj; break;
    default: break;
  }
}

constexpr int kSwept = 0x100, kFirstA = 0x200, kFirstB = 0x400;
constexpr unsigned kNoSlot = 0xFFFFu;
constexpr int kInterpMaxNodes = 0xFFFE;  // node indices and slots are 16-bit in the records

// One interpreter step per node, packed in 16 bytes (16-bit slots, kNoSlot = none):
//   x = op | flags << 8 | value slot << 16       y = slot of a (leaf: aux) | slot of b << 16
//   z = adjoint slot of the node | of a << 16     w = adjoint slot of b
// flags: kSwept (reverse step), kFirstA / kFirstB (first contribution: assign, not add);
// aux: CONST constant index, INPUT input index, RANDN draw ordinal.
// SMEM: slots and records live in dynamic shared memory ([slot][thread], 32-bit addressing);
// otherwise slots are [slot][thread] in global scratch with T threads and records are read
// through the read-only cache.
template <typename real, bool SMEM>
__global__ void __launch_bounds__(J4B_AAD_BLOCK) aad_interp_kernel(
    const int4* __restrict__ rec, const double* __restrict__ consts, const double* __restrict__ inputs,
    const int* __restrict__ in_dslot, int n, int n_in, int out_vslot, int out_dslot, int nv, int nd, int adjoints,
    unsigned long long n_paths, unsigned long long offset, unsigned long long seed, real* __restrict__ gscratch,
    unsigned long long T, double* partials, unsigned int* ticket, double* sums) {
  extern __shared__ __align__(16) unsigned char j4b_interp_smem[];
  const unsigned long long tid = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x;
  real* sv = reinterpret_cast<real*>(j4b_interp_smem);
  const unsigned bd = blockDim.x, tx = threadIdx.x;
  const int4* R = rec;
  if constexpr (SMEM) {
    int4* srec = reinterpret_cast<int4*>(sv + (size_t)(nv + nd) * bd);
    for (int i = tx; i < n; i += bd) srec[i] = rec[i];
    __syncthreads();
    R = srec;
  }
  real* gv = gscratch + tid;
  auto VAL = [&](unsigned s) -> real& {
    if constexpr (SMEM) return sv[s * bd + tx];
    else return gv[(unsigned long long)s * T];
  };
  auto ADJ = [&](unsigned s) -> real& { return VAL((unsigned)nv + s); };
  double acc[kInterpChannels];
#pragma unroll
  for (int c = 0; c < kInterpChannels; ++c) acc[c] = 0.0;
  for (unsigned long long path = tid; path < n_paths; path += T) {
    unsigned int lo, hi;
    j4b_scenario_key(path + offset, seed, lo, hi);
    int pair = -1;
    real zc = 0, zs = 0;
    for (int i = 0; i < n; ++i) {
      const int4 r = SMEM ? R[i] : __ldg(R + i);
      const int op = r.x & 0xff;
      const unsigned a = (unsigned)r.y & 0xFFFFu, b = (unsigned)r.y >> 16, vs = (unsigned)r.x >> 16;
      real v;
      switch (op) {  // dense: one indirect branch
        case J4B_AAD_CONST: v = (real)__ldg(consts + a); break;
        case J4B_AAD_INPUT: v = (real)__ldg(inputs + a); break;
        case J4B_AAD_RANDN: {
          const int m = (int)(a >> 1);
          if (m != pair) {
            j4b_normal_pair<real>(lo, hi, (unsigned int)m, zc, zs);
            pair = m;
          }
          v = (a & 1) ? zs : zc;
          break;
        }
        case J4B_AAD_ADD: v = VAL(a) + VAL(b); break;
        case J4B_AAD_SUB: v = VAL(a) - VAL(b); break;
        case J4B_AAD_MUL: v = VAL(a) * VAL(b); break;
        case J4B_AAD_DIV: v = VAL(a) / VAL(b); break;
        case J4B_AAD_NEG: v = -VAL(a); break;
        case J4B_AAD_EXP: v = unary_fwd<real>(J4B_AAD_EXP, VAL(a)); break;
        case J4B_AAD_LOG: v = unary_fwd<real>(J4B_AAD_LOG, VAL(a)); break;
        case J4B_AAD_SQRT: v = unary_fwd<real>(J4B_AAD_SQRT, VAL(a)); break;
        case J4B_AAD_MAX: v = fmax(VAL(a), VAL(b)); break;
        case J4B_AAD_MIN: v = fmin(VAL(a), VAL(b)); break;
        default: v = unary_fwd<real>(J4B_AAD_ABS, VAL(a)); break;
      }
      if (vs != kNoSlot) VAL(vs) = v;
    }
    const double y = (double)VAL((unsigned)out_vslot);
    acc[0] += y;
    acc[1] += y * y;
    if (!adjoints) continue;
    if (out_dslot >= 0) ADJ((unsigned)out_dslot) = (real)1;
    for (int i = n - 1; i >= 0; --i) {
      const int4 r = SMEM ? R[i] : __ldg(R + i);
      if (!(r.x & kSwept)) continue;
      const int op = r.x & 0xff;
      const unsigned a = (unsigned)r.y & 0xFFFFu, b = (unsigned)r.y >> 16, vs = (unsigned)r.x >> 16;
      const unsigned di = (unsigned)r.z & 0xFFFFu, da = (unsigned)r.z >> 16, db = (unsigned)r.w;
      const real adj = ADJ(di);
      real ga = 0, gb = 0;
      switch (op) {
        case J4B_AAD_ADD: ga = adj; gb = adj; break;
        case J4B_AAD_SUB: ga = adj; gb = -adj; break;
        case J4B_AAD_MUL: ga = adj * VAL(b); gb = adj * VAL(a); break;
        case J4B_AAD_DIV: {
          const real vb = VAL(b);
          ga = adj / vb;
          if (db != kNoSlot) gb = -(adj * VAL(vs) / vb);
          break;
        }
        case J4B_AAD_NEG: ga = -adj; break;
        case J4B_AAD_EXP: ga = adj * VAL(vs); break;
        case J4B_AAD_LOG: ga = adj / VAL(a); break;
        case J4B_AAD_SQRT: ga = adj * (real)0.5 / VAL(vs); break;
        case J4B_AAD_ABS: ga = VAL(a) < (real)0 ? -adj : adj; break;
        case J4B_AAD_MAX:
        case J4B_AAD_MIN: {
          const real va = VAL(a), vb = VAL(b);
          const bool take_a = op == J4B_AAD_MAX ? va >= vb : va <= vb;
          ga = take_a ? adj : (real)0;
          gb = take_a ? (real)0 : adj;
          break;
        }
        default: break;
      }
      if (da != kNoSlot) {
        real& p = ADJ(da);
        p = (r.x & kFirstA) ? ga : p + ga;
      }
      if (db != kNoSlot) {
        real& p = ADJ(db);
        p = (r.x & kFirstB) ? gb : p + gb;
      }
    }
#pragma unroll
    for (int j = 0; j < kInterpMaxInputs; ++j)
      if (j < n_in) {
        const int sl = __ldg(in_dslot + j);
        if (sl >= 0) acc[2 + j] += (double)ADJ((unsigned)sl);
      }
  }
  j4b_aad_finish<kInterpChannels>(acc, 2 + (adjoints ? n_in : 0), partials, ticket, sums, false);
}

// ---------------------------------------------------------------------------------------------
// eager: one launch per node over `n` scenarios starting at path `base`
// ---------------------------------------------------------------------------------------------
template <typename real>
__global__ void aad_eager_forward(int op, double cst, int k, const double* __restrict__ inputs, int input,
                                  unsigned long long base, unsigned long long seed, const real* __restrict__ va,
                                  const real* __restrict__ vb, real* __restrict__ out, unsigned long long n) {
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  for (unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    real r;
    if (op == J4B_AAD_CONST) {
      r = (real)cst;
    } else if (op == J4B_AAD_INPUT) {
      r = (real)inputs[input];
    } else if (op == J4B_AAD_RANDN) {
      unsigned int lo, hi;
      j4b_scenario_key(base + i, seed, lo, hi);
      real zc, zs;
      j4b_normal_pair<real>(lo, hi, (unsigned int)(k >> 1), zc, zs);
      r = (k & 1) ? zs : zc;
    } else if (is_binary(op)) {
      r = binary_fwd<real>(op, va[i], vb[i]);
    } else {
      r = unary_fwd<real>(op, va[i]);
    }
    out[i] = r;
  }
}

template <typename real>
__global__ void aad_eager_reverse(int op, const real* __restrict__ va, const real* __restrict__ vb,
                                  const real* __restrict__ vi, const real* __restrict__ di, real* da, real* db,
                                  unsigned long long n) {
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  for (unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    real ga, gb;
    node_adjoint<real>(op, va[i], vb ? vb[i] : (real)0, vi[i], di[i], ga, gb);
    if (da) da[i] += ga;
    if (db) db[i] += gb;
  }
}

template <typename real>
__global__ void aad_eager_fill(real* __restrict__ x, real v, unsigned long long n) {
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  for (unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) x[i] = v;
}

// sums[slot] += sum over i < n of x[i] (or x[i]^2)
template <typename real>
__global__ void __launch_bounds__(J4B_AAD_BLOCK) aad_eager_reduce(const real* __restrict__ x, unsigned long long n,
                                                                  int square, double* partials, unsigned int* ticket,
                                                                  double* slot) {
  double acc[1] = {0.0};
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  for (unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const double v = (double)x[i];
    acc[0] += square ? v * v : v;
  }
  j4b_aad_finish<1>(acc, 1, partials, ticket, slot, true);
}

// ---------------------------------------------------------------------------------------------
// generated kernel
// ---------------------------------------------------------------------------------------------
std::string real_lit(double v, bool f32) {
  if (std::isnan(v)) return f32 ? "__int_as_float(0x7fc00000)" : "__longlong_as_double(0x7ff8000000000000ll)";
  if (std::isinf(v)) return std::string(v > 0 ? "" : "-") + (f32 ? "__int_as_float(0x7f800000)" : "__longlong_as_double(0x7ff0000000000000ll)");
  char b[64];
  snprintf(b, sizeof b, "(real)%a", v);  // exact hexadecimal double literal
  return b;
}

}  // namespace
}  // namespace j4b

struct j4b_aad {
  int dev = 0, engine = 0, adjoints = 1;
  bool f32 = true;
  int n = 0, n_in = 0, out = 0, channels = 2;
  std::vector<int32_t> op, a, b, in_nodes;
  std::vector<double> cst;
  std::vector<uint8_t> active;
  // generated
  std::string src;
  CUmodule mod = nullptr;
  CUfunction fn = nullptr;
  int gen_blocks_per_sm = 1;
  double compile_seconds = 0.0;
  // interpreter: slot-planned records, per-input adjoint slots, launch shape
  int4* d_nodes = nullptr;
  double* d_consts = nullptr;
  int* d_in_nodes = nullptr;  // adjoint slot per input (-1: gradient identically 0)
  int nv = 0, nd = 0, out_vslot = 0, out_dslot = -1;
  int interp_block = J4B_AAD_BLOCK;
  size_t interp_smem = 0;  // dynamic shared memory per CTA; 0 = slots in global scratch
  int64_t interp_threads = 0;
  // eager
  int64_t slot = 0;
  // scratch: interpreter [slot][thread] values then adjoints (global mode, in vs); eager
  // [node][scenario] values (vs) and adjoints (ds)
  void* vs = nullptr;
  void* ds = nullptr;
  // common
  double* d_inputs = nullptr;
  double* d_partials = nullptr;
  int64_t partial_slots = 0;
  unsigned int* d_ticket = nullptr;
  double* d_sums = nullptr;
};

namespace j4b {
namespace {

void aad_release(j4b_aad* h) {
  if (!h) return;
  DeviceGuard g(h->dev);
  if (h->mod && driver().ok) driver().ModuleUnload(h->mod);
  for (void* p : {(void*)h->d_nodes, (void*)h->d_consts, (void*)h->d_in_nodes, h->vs, h->ds, (void*)h->d_inputs,
                  (void*)h->d_partials, (void*)h->d_ticket, (void*)h->d_sums})
    if (p) cudaFree(p);
  delete h;
}

std::string generate(const j4b_aad& h) {
  const bool f32 = h.f32;
  const char* ex = f32 ? "expf" : "exp";
  const char* lg = f32 ? "logf" : "log";
  const char* sq = f32 ? "sqrtf" : "sqrt";
  const char* ab = f32 ? "fabsf" : "fabs";
  const char* mx = f32 ? "fmaxf" : "fmax";
  const char* mn = f32 ? "fminf" : "fmin";
  const int C = h.channels;
  std::ostringstream s;
  s << kAadDeviceSource << "\ntypedef " << (f32 ? "float" : "double") << " real;\n";
  s << "extern \"C\" __global__ void __launch_bounds__(J4B_AAD_BLOCK) aad_replay(\n"
       "    const double* __restrict__ inputs, unsigned long long n_paths, unsigned long long path_offset,\n"
       "    unsigned long long seed, double* partials, unsigned int* ticket, double* sums) {\n";
  for (int j = 0; j < h.n_in; ++j) s << "  const real in" << j << " = (real)inputs[" << j << "];\n";
  s << "  double acc[" << C << "];\n#pragma unroll\n  for (int c = 0; c < " << C << "; ++c) acc[c] = 0.0;\n";
  s << "  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;\n"
       "  for (unsigned long long path = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; path < n_paths;\n"
       "       path += stride) {\n"
       "    unsigned int lo, hi;\n"
       "    j4b_scenario_key(path + path_offset, seed, lo, hi);\n";
  // Box-Muller pairs in use; pairs 2g and 2g + 1 are drawn together (interleaved Philox) at the
  // first use of either.
  std::vector<char> pair_used, group_done;
  for (int i = 0; i < h.n; ++i)
    if (h.op[i] == J4B_AAD_RANDN) {
      const int m = h.a[i] >> 1;
      if ((int)pair_used.size() <= m) pair_used.resize(m + 1, 0);
      pair_used[m] = 1;
    }
  pair_used.push_back(0);
  group_done.assign(pair_used.size() / 2 + 1, 0);
  for (int i = 0; i < h.n; ++i) {
    const int o = h.op[i], a = h.a[i], b = h.b[i];
    if (o == J4B_AAD_RANDN && !group_done[(a >> 1) / 2]) {
      const int g = (a >> 1) / 2, m0 = 2 * g, m1 = 2 * g + 1;
      group_done[g] = 1;
      if (pair_used[m0] && pair_used[m1]) {
        s << "    real zc" << m0 << ", zs" << m0 << ", zc" << m1 << ", zs" << m1 << ";\n    j4b_normal_pair2<real>(lo, hi, "
          << m0 << "u, zc" << m0 << ", zs" << m0 << ", zc" << m1 << ", zs" << m1 << ");\n";
      } else {
        const int m = pair_used[m0] ? m0 : m1;
        s << "    real zc" << m << ", zs" << m << ";\n    j4b_normal_pair<real>(lo, hi, " << m << "u, zc" << m << ", zs" << m
          << ");\n";
      }
    }
    s << "    const real v" << i << " = ";
    switch (o) {
      case J4B_AAD_CONST: s << real_lit(h.cst[i], f32); break;
      case J4B_AAD_INPUT: s << "in" << a; break;
      case J4B_AAD_RANDN: s << ((a & 1) ? "zs" : "zc") << (a >> 1); break;
      case J4B_AAD_ADD: s << "v" << a << " + v" << b; break;
      case J4B_AAD_SUB: s << "v" << a << " - v" << b; break;
      case J4B_AAD_MUL: s << "v" << a << " * v" << b; break;
      case J4B_AAD_DIV: s << "v" << a << " / v" << b; break;
      case J4B_AAD_NEG: s << "-v" << a; break;
      case J4B_AAD_EXP: s << ex << "(v" << a << ")"; break;
      case J4B_AAD_LOG: s << lg << "(v" << a << ")"; break;
      case J4B_AAD_SQRT: s << sq << "(v" << a << ")"; break;
      case J4B_AAD_ABS: s << ab << "(v" << a << ")"; break;
      case J4B_AAD_MAX: s << mx << "(v" << a << ", v" << b << ")"; break;
      case J4B_AAD_MIN: s << mn << "(v" << a << ", v" << b << ")"; break;
    }
    s << ";\n";
  }
  s << "    acc[0] += (double)v" << h.out << ";\n    acc[1] += (double)v" << h.out << " * (double)v" << h.out << ";\n";
  if (h.adjoints) {
    for (int i = 0; i < h.n; ++i)
      if (h.active[i]) s << "    real d" << i << " = (real)0;\n";
    if (h.active[h.out]) s << "    d" << h.out << " = (real)1;\n";
    for (int i = h.n - 1; i >= 0; --i) {
      if (!h.active[i]) continue;
      const int o = h.op[i], a = h.a[i], b = h.b[i];
      const bool la = a >= 0 && (is_unary(o) || is_binary(o)) && h.active[a];
      const bool lb = b >= 0 && is_binary(o) && h.active[b];
      const std::string di = "d" + std::to_string(i), va = "v" + std::to_string(a), vb = "v" + std::to_string(b),
                        vi = "v" + std::to_string(i), da = "d" + std::to_string(a), db = "d" + std::to_string(b);
      switch (o) {
        case J4B_AAD_ADD:
          if (la) s << "    " << da << " += " << di << ";\n";
          if (lb) s << "    " << db << " += " << di << ";\n";
          break;
        case J4B_AAD_SUB:
          if (la) s << "    " << da << " += " << di << ";\n";
          if (lb) s << "    " << db << " -= " << di << ";\n";
          break;
        case J4B_AAD_MUL:
          if (la) s << "    " << da << " += " << di << " * " << vb << ";\n";
          if (lb) s << "    " << db << " += " << di << " * " << va << ";\n";
          break;
        case J4B_AAD_DIV:
          if (la) s << "    " << da << " += " << di << " / " << vb << ";\n";
          if (lb) s << "    " << db << " -= " << di << " * " << vi << " / " << vb << ";\n";
          break;
        case J4B_AAD_NEG:
          if (la) s << "    " << da << " -= " << di << ";\n";
          break;
        case J4B_AAD_EXP:
          if (la) s << "    " << da << " += " << di << " * " << vi << ";\n";
          break;
        case J4B_AAD_LOG:
          if (la) s << "    " << da << " += " << di << " / " << va << ";\n";
          break;
        case J4B_AAD_SQRT:
          if (la) s << "    " << da << " += " << di << " * (real)0.5 / " << vi << ";\n";
          break;
        case J4B_AAD_ABS:
          if (la) s << "    " << da << " += " << va << " < (real)0 ? -" << di << " : " << di << ";\n";
          break;
        case J4B_AAD_MAX:
        case J4B_AAD_MIN: {
          // the adjoint follows the branch this scenario took
          const std::string taken = "(" + va + (o == J4B_AAD_MAX ? " >= " : " <= ") + vb + ")";
          if (la) s << "    if " << taken << " " << da << " += " << di << ";\n";
          if (lb) s << "    if (!" << taken << ") " << db << " += " << di << ";\n";
          break;
        }
        default: break;
      }
    }
    for (int j = 0; j < h.n_in; ++j) s << "    acc[" << 2 + j << "] += (double)d" << h.in_nodes[j] << ";\n";
  }
  s << "  }\n  j4b_aad_finish<" << C << ">(acc, " << C << ", partials, ticket, sums, false);\n}\n";
  return s.str();
}

// Linear-scan slot assignment: interval k = [start, end] gets slot_of[k]; a slot whose interval
// ends at t may be taken by one that starts at t (a node reads its operands before it writes).
int assign_slots(const std::vector<std::pair<int64_t, int64_t>>& iv, std::vector<int>& slot_of) {
  std::vector<int> order(iv.size());
  for (size_t k = 0; k < iv.size(); ++k) order[k] = (int)k;
  std::sort(order.begin(), order.end(), [&](int x, int y) { return iv[x].first < iv[y].first; });
  using EndSlot = std::pair<int64_t, int>;
  std::priority_queue<EndSlot, std::vector<EndSlot>, std::greater<EndSlot>> busy;
  std::priority_queue<int, std::vector<int>, std::greater<int>> free_slots;
  int slots = 0;
  slot_of.assign(iv.size(), -1);
  for (int k : order) {
    while (!busy.empty() && busy.top().first <= iv[k].first) {
      free_slots.push(busy.top().second);
      busy.pop();
    }
    int sl;
    if (!free_slots.empty()) {
      sl = free_slots.top();
      free_slots.pop();
    } else {
      sl = slots++;
    }
    slot_of[k] = sl;
    busy.push({iv[k].second, sl});
  }
  return slots;
}

// Plans the interpreter's slots and records (see the kernel). Times: forward node i at i, the
// output read at n, reverse step of node j at n + (n - 1 - j), the input gradients read at 2n.
void plan_interp(j4b_aad& h, std::vector<int4>& rec, std::vector<int>& in_dslot) {
  const int n = h.n, out = h.out;
  auto R = [&](int j) { return (int64_t)n + (n - 1 - j); };
  auto args = [&](int j) { return is_unary(h.op[j]) || is_binary(h.op[j]); };
  // adjoint needed: the output, and every active operand of a swept node
  std::vector<char> need(n, 0), swept(n, 0);
  need[out] = 1;
  for (int j = n - 1; j >= 0; --j) {
    if (!(need[j] && h.active[j] && args(j) && h.adjoints)) continue;
    swept[j] = 1;
    if (h.active[h.a[j]]) need[h.a[j]] = 1;
    if (is_binary(h.op[j]) && h.active[h.b[j]]) need[h.b[j]] = 1;
  }
  // value intervals
  std::vector<int64_t> vend(n, -1);
  auto use = [&](int x, int64_t t) { vend[x] = std::max(vend[x], t); };
  for (int k = 0; k < n; ++k) {
    if (args(k)) use(h.a[k], k);
    if (is_binary(h.op[k])) use(h.b[k], k);
  }
  use(out, n);
  for (int j = 0; j < n; ++j) {
    if (!swept[j]) continue;
    const int o = h.op[j], a = h.a[j], b = h.b[j];
    const bool la = h.active[a], lb = is_binary(o) && h.active[b];
    switch (o) {
      case J4B_AAD_MUL: if (la) use(b, R(j)); if (lb) use(a, R(j)); break;
      case J4B_AAD_DIV: use(b, R(j)); if (lb) use(j, R(j)); break;
      case J4B_AAD_EXP: case J4B_AAD_SQRT: use(j, R(j)); break;
      case J4B_AAD_LOG: case J4B_AAD_ABS: use(a, R(j)); break;
      case J4B_AAD_MAX: case J4B_AAD_MIN: use(a, R(j)); use(b, R(j)); break;
      default: break;
    }
  }
  std::vector<std::pair<int64_t, int64_t>> iv;
  std::vector<int> owner;
  for (int i = 0; i < n; ++i)
    if (vend[i] >= 0) {
      iv.push_back({i, vend[i]});
      owner.push_back(i);
    }
  std::vector<int> sl;
  h.nv = assign_slots(iv, sl);
  std::vector<int> vslot(n, -1);
  for (size_t k = 0; k < owner.size(); ++k) vslot[owner[k]] = sl[k];
  // adjoint intervals and first-contribution flags
  std::vector<int64_t> dstart(n, -1);
  std::vector<int> flags(n, 0);
  if (h.adjoints) dstart[out] = n;
  for (int j = n - 1; j >= 0; --j) {
    if (!swept[j]) continue;
    const int o = h.op[j], a = h.a[j], b = h.b[j];
    if (h.active[a]) {
      if (dstart[a] < 0) {
        dstart[a] = R(j);
        flags[j] |= kFirstA;
      }
    }
    if (is_binary(o) && h.active[b]) {
      if (dstart[b] < 0) {
        dstart[b] = R(j);
        flags[j] |= kFirstB;
      }
    }
  }
  iv.clear();
  owner.clear();
  for (int x = 0; x < n; ++x)
    if (dstart[x] >= 0) {
      iv.push_back({dstart[x], h.op[x] == J4B_AAD_INPUT ? 2 * (int64_t)n : R(x)});
      owner.push_back(x);
    }
  h.nd = assign_slots(iv, sl);
  std::vector<int> dslot(n, -1);
  for (size_t k = 0; k < owner.size(); ++k) dslot[owner[k]] = sl[k];
  auto u16 = [](int v) { return (unsigned)(v < 0 ? kNoSlot : v); };
  rec.assign((size_t)n, make_int4(0, 0, 0, 0));
  for (int i = 0; i < n; ++i) {
    const int o = h.op[i];
    const int fl = (swept[i] ? kSwept : 0) | flags[i];
    unsigned a = 0, b = 0;
    if (o == J4B_AAD_CONST) a = (unsigned)i;
    else if (o == J4B_AAD_INPUT || o == J4B_AAD_RANDN) a = (unsigned)h.a[i];
    else {
      a = u16(vslot[h.a[i]]);
      b = is_binary(o) ? u16(vslot[h.b[i]]) : 0u;
    }
    unsigned di = kNoSlot, da = kNoSlot, db = kNoSlot;
    if (swept[i]) {
      di = u16(dslot[i]);
      if (h.active[h.a[i]]) da = u16(dslot[h.a[i]]);
      if (is_binary(o) && h.active[h.b[i]]) db = u16(dslot[h.b[i]]);
    }
    rec[i] = make_int4((int)((unsigned)o | (unsigned)fl | (u16(vslot[i]) << 16)), (int)(a | (b << 16)),
                       (int)(di | (da << 16)), (int)db);
  }
  in_dslot.assign(std::max(1, h.n_in), -1);
  for (int j = 0; j < h.n_in; ++j) in_dslot[j] = dslot[h.in_nodes[j]];
  h.out_vslot = vslot[out];
  h.out_dslot = h.adjoints ? dslot[out] : -1;
}

int ensure_partials(j4b_aad* h, int64_t slots) {
  if (slots <= h->partial_slots) return J4B_OK;
  if (h->d_partials) cudaFree(h->d_partials);
  h->d_partials = nullptr;
  h->partial_slots = 0;
  J4B_CUDA(cudaMalloc(&h->d_partials, (size_t)slots * sizeof(double)), "cudaMalloc(aad partials)");
  counters().allocations++;
  h->partial_slots = slots;
  return J4B_OK;
}

template <typename real>
int eager_replay(j4b_aad* h, uint64_t paths, uint64_t offset, uint64_t seed, cudaStream_t st) {
  const int sms = device_ctx(h->dev)->sm_count;
  const unsigned grid = (unsigned)(2 * sms);
  int rc = ensure_partials(h, grid);
  if (rc) return rc;
  real* V = (real*)h->vs;
  real* D = (real*)h->ds;
  const uint64_t slot = (uint64_t)h->slot;
  auto row = [&](real* base, int node) { return base + (uint64_t)node * slot; };
  J4B_CUDA(cudaMemsetAsync(h->d_sums, 0, (size_t)h->channels * sizeof(double), st), "cudaMemsetAsync(aad sums)");
  for (uint64_t done = 0; done < paths; done += slot) {
    const uint64_t count = std::min<uint64_t>(slot, paths - done);
    const uint64_t base = offset + done;
    for (int i = 0; i < h->n; ++i) {
      const int a = h->a[i], b = h->b[i], o = h->op[i];
      const bool args = is_unary(o) || is_binary(o);
      aad_eager_forward<real><<<grid, J4B_AAD_BLOCK, 0, st>>>(
          o, h->cst[i], o == J4B_AAD_RANDN ? a : 0, h->d_inputs, o == J4B_AAD_INPUT ? a : 0, base, seed,
          args ? row(V, a) : V, is_binary(o) ? row(V, b) : V, row(V, i), count);
      J4B_CHECK_LAUNCH("aad_eager_forward");
    }
    aad_eager_reduce<real><<<grid, J4B_AAD_BLOCK, 0, st>>>(row(V, h->out), count, 0, h->d_partials, h->d_ticket,
                                                           h->d_sums + 0);
    J4B_CHECK_LAUNCH("aad_eager_reduce");
    aad_eager_reduce<real><<<grid, J4B_AAD_BLOCK, 0, st>>>(row(V, h->out), count, 1, h->d_partials, h->d_ticket,
                                                           h->d_sums + 1);
    J4B_CHECK_LAUNCH("aad_eager_reduce");
    if (!h->adjoints) continue;
    // adjoint rows of the chunk: all zero, then 1 for the output
    J4B_CUDA(cudaMemsetAsync(D, 0, (size_t)h->n * slot * sizeof(real), st), "cudaMemsetAsync(aad adjoints)");
    if (h->active[h->out]) {
      aad_eager_fill<real><<<grid, J4B_AAD_BLOCK, 0, st>>>(row(D, h->out), (real)1, count);
      J4B_CHECK_LAUNCH("aad_eager_fill");
    }
    for (int i = h->n - 1; i >= 0; --i) {
      const int o = h->op[i], a = h->a[i], b = h->b[i];
      if (!h->active[i] || !(is_unary(o) || is_binary(o))) continue;
      const bool la = h->active[a], lb = is_binary(o) && h->active[b];
      aad_eager_reverse<real><<<grid, J4B_AAD_BLOCK, 0, st>>>(o, row(V, a), is_binary(o) ? row(V, b) : nullptr,
                                                              row(V, i), row(D, i), la ? row(D, a) : nullptr,
                                                              lb ? row(D, b) : nullptr, count);
      J4B_CHECK_LAUNCH("aad_eager_reverse");
    }
    for (int j = 0; j < h->n_in; ++j) {
      aad_eager_reduce<real><<<grid, J4B_AAD_BLOCK, 0, st>>>(row(D, h->in_nodes[j]), count, 0, h->d_partials,
                                                             h->d_ticket, h->d_sums + 2 + j);
      J4B_CHECK_LAUNCH("aad_eager_reduce");
    }
  }
  return J4B_OK;
}

template <typename real, bool SMEM>
void launch_interp(j4b_aad* h, unsigned grid, const double* d_inputs, uint64_t paths, uint64_t offset, uint64_t seed,
                   cudaStream_t st) {
  aad_interp_kernel<real, SMEM><<<grid, h->interp_block, h->interp_smem, st>>>(
      h->d_nodes, h->d_consts, d_inputs, h->d_in_nodes, h->n, h->n_in, h->out_vslot, h->out_dslot, h->nv, h->nd,
      h->adjoints, paths, offset, seed, (real*)h->vs, (unsigned long long)h->interp_threads, h->d_partials, h->d_ticket,
      h->d_sums);
}

const void* interp_fn(bool f32, bool smem) {
  if (f32) return smem ? (const void*)aad_interp_kernel<float, true> : (const void*)aad_interp_kernel<float, false>;
  return smem ? (const void*)aad_interp_kernel<double, true> : (const void*)aad_interp_kernel<double, false>;
}

int launch_replay(j4b_aad* h, const double* d_inputs, uint64_t paths, uint64_t offset, uint64_t seed,
                  cudaStream_t st) {
  const int sms = device_ctx(h->dev)->sm_count;
  if (h->engine == J4B_AAD_ENGINE_GENERATED) {
    const uint64_t need = (paths + J4B_AAD_BLOCK - 1) / J4B_AAD_BLOCK;
    const unsigned grid = (unsigned)std::max<uint64_t>(1, std::min<uint64_t>(need, (uint64_t)sms * h->gen_blocks_per_sm));
    int rc = ensure_partials(h, (int64_t)grid * h->channels);
    if (rc) return rc;
    unsigned long long np = paths, off = offset, sd = seed;
    void* args[] = {(void*)&d_inputs, &np, &off, &sd, &h->d_partials, &h->d_ticket, &h->d_sums};
    CUresult r = driver().LaunchKernel(h->fn, grid, 1, 1, J4B_AAD_BLOCK, 1, 1, 0, (CUstream)st, args, nullptr);
    if (r != CUDA_SUCCESS) return cu_error(r, "cuLaunchKernel(aad_replay)");
    count_launch();
    return J4B_OK;
  }
  if (h->engine == J4B_AAD_ENGINE_INTERP) {
    const unsigned grid = (unsigned)(h->interp_threads / h->interp_block);
    int rc = ensure_partials(h, (int64_t)grid * h->channels);
    if (rc) return rc;
    const bool sm = h->interp_smem > 0;
    if (h->f32) {
      if (sm) launch_interp<float, true>(h, grid, d_inputs, paths, offset, seed, st);
      else launch_interp<float, false>(h, grid, d_inputs, paths, offset, seed, st);
    } else {
      if (sm) launch_interp<double, true>(h, grid, d_inputs, paths, offset, seed, st);
      else launch_interp<double, false>(h, grid, d_inputs, paths, offset, seed, st);
    }
    J4B_CHECK_LAUNCH("aad_interp_kernel");
    return J4B_OK;
  }
  if (d_inputs != h->d_inputs)
    J4B_CUDA(cudaMemcpyAsync(h->d_inputs, d_inputs, (size_t)std::max(1, h->n_in) * sizeof(double),
                             cudaMemcpyDeviceToDevice, st),
             "cudaMemcpyAsync(aad inputs)");
  return h->f32 ? eager_replay<float>(h, paths, offset, seed, st) : eager_replay<double>(h, paths, offset, seed, st);
}

}  // namespace
}  // namespace j4b

using namespace j4b;

namespace {
// Validates a tape (the checks AadTape's recorder guarantees, plus the engines' limits) and
// fills the host fields of `h`.
int load_tape(j4b_aad* h, int engine, int n_nodes, const int32_t* ops, const int32_t* arg_a, const int32_t* arg_b,
              const double* constants, int n_inputs, const int32_t* input_nodes, int output_node, int precision,
              int adjoints) {
  J4B_REQUIRE(engine >= J4B_AAD_ENGINE_GENERATED && engine <= J4B_AAD_ENGINE_EAGER, "unknown AAD engine %d", engine);
  J4B_REQUIRE(precision == 4 || precision == 8, "precision must be 4 (FLOAT32) or 8 (FLOAT64), got %d", precision);
  J4B_REQUIRE(n_nodes >= 1 && ops && arg_a && arg_b && constants, "an AAD tape needs at least one node");
  J4B_REQUIRE(n_inputs >= 0 && (n_inputs == 0 || input_nodes), "invalid AAD input list");
  J4B_REQUIRE(output_node >= 0 && output_node < n_nodes, "output node %d out of range", output_node);
  static const char* kNames[] = {"cuda", "cuda-interp", "cuda-eager"};
  for (int i = 0; i < n_nodes; ++i) {
    const int o = ops[i], a = arg_a[i], b = arg_b[i];
    J4B_REQUIRE(o >= J4B_AAD_CONST && o <= J4B_AAD_ABS, "node %d: unknown op %d", i, o);
    if (o == J4B_AAD_RANDU || (o == J4B_AAD_RANDN && b != 0))
      return set_error(J4B_EUNSUPPORTED,
                       "engine '%s' does not yet support rec.randu() or named random streams; use cpu-jit or cpu "
                       "for this tape",
                       kNames[engine]);
    if (o == J4B_AAD_RANDN) J4B_REQUIRE(a >= 0, "node %d: negative draw ordinal", i);
    if (o == J4B_AAD_INPUT) J4B_REQUIRE(a >= 0 && a < n_inputs, "node %d: input index %d out of range", i, a);
    if (is_unary(o) || is_binary(o)) J4B_REQUIRE(a >= 0 && a < i, "node %d: argument %d is not an earlier node", i, a);
    if (is_binary(o)) J4B_REQUIRE(b >= 0 && b < i, "node %d: argument %d is not an earlier node", i, b);
  }
  for (int j = 0; j < n_inputs; ++j) {
    const int v = input_nodes[j];
    J4B_REQUIRE(v >= 0 && v < n_nodes && ops[v] == J4B_AAD_INPUT && arg_a[v] == j, "input %d does not name its INPUT node",
                j);
  }
  if (engine == J4B_AAD_ENGINE_INTERP) {
    J4B_REQUIRE(n_inputs <= kInterpMaxInputs, "the interpreting engine supports at most %d inputs", kInterpMaxInputs);
    J4B_REQUIRE(n_nodes <= kInterpMaxNodes, "the interpreting engine supports at most %d nodes", kInterpMaxNodes);
  }
  h->engine = engine;
  h->f32 = precision == 4;
  h->adjoints = adjoints ? 1 : 0;
  h->n = n_nodes;
  h->n_in = n_inputs;
  h->out = output_node;
  h->channels = 2 + (h->adjoints ? n_inputs : 0);
  h->op.assign(ops, ops + n_nodes);
  h->a.assign(arg_a, arg_a + n_nodes);
  h->b.assign(arg_b, arg_b + n_nodes);
  h->cst.assign(constants, constants + n_nodes);
  if (n_inputs) h->in_nodes.assign(input_nodes, input_nodes + n_inputs);
  // active: depends on a differentiable input (AadTape.java:61-74)
  h->active.assign(n_nodes, 0);
  for (int i = 0; i < n_nodes; ++i) {
    const int o = ops[i];
    h->active[i] = o == J4B_AAD_INPUT ? 1
                   : is_unary(o)      ? h->active[arg_a[i]]
                   : is_binary(o)     ? (h->active[arg_a[i]] || h->active[arg_b[i]])
                                      : 0;
  }
  return J4B_OK;
}
}  // namespace

extern "C" int j4b_aad_dryrun(int n_nodes, const int32_t* ops, const int32_t* arg_a, const int32_t* arg_b,
                              const double* constants, int n_inputs, const int32_t* input_nodes, int output_node,
                              int precision, int adjoints, char* buf, size_t cap, size_t* len) {
  j4b_aad h;
  int st = load_tape(&h, J4B_AAD_ENGINE_GENERATED, n_nodes, ops, arg_a, arg_b, constants, n_inputs, input_nodes,
                     output_node, precision, adjoints);
  if (st) return st;
  h.src = generate(h);
  std::vector<char> cubin;
  st = compile_source(h.src, "j4b_aad.cu", cubin, true);
  if (st) return st;
  if (len) *len = h.src.size();
  if (buf && cap) {
    const size_t n = std::min(cap - 1, h.src.size());
    memcpy(buf, h.src.data(), n);
    buf[n] = '\0';
  }
  return J4B_OK;
}

extern "C" int j4b_aad_compile(int dev, int engine, int n_nodes, const int32_t* ops, const int32_t* arg_a,
                               const int32_t* arg_b, const double* constants, int n_inputs,
                               const int32_t* input_nodes, int output_node, int precision, int adjoints,
                               int64_t scratch_option, j4b_aad_t* out) {
  J4B_REQUIRE(out != nullptr, "null output handle");
  *out = nullptr;
  J4B_REQUIRE(scratch_option >= 0, "negative scratch option");
  {
    j4b_aad probe;
    int st = load_tape(&probe, engine, n_nodes, ops, arg_a, arg_b, constants, n_inputs, input_nodes, output_node,
                       precision, adjoints);
    if (st) return st;
  }
  int st = ensure_device(dev);
  if (st) return st;
  DeviceGuard guard(dev);
  j4b_aad* h = new j4b_aad();
  h->dev = dev;
  load_tape(h, engine, n_nodes, ops, arg_a, arg_b, constants, n_inputs, input_nodes, output_node, precision, adjoints);
  auto fail = [&](int code) {
    aad_release(h);
    return code;
  };
  auto cuda_fail = [&](cudaError_t e, const char* what) { return fail(cuda_error(e, what)); };
  cudaError_t e;
  if ((e = cudaMalloc(&h->d_inputs, (size_t)std::max(1, n_inputs) * sizeof(double))) != cudaSuccess)
    return cuda_fail(e, "cudaMalloc(aad inputs)");
  if ((e = cudaMalloc(&h->d_ticket, sizeof(unsigned int))) != cudaSuccess) return cuda_fail(e, "cudaMalloc(aad ticket)");
  if ((e = cudaMemset(h->d_ticket, 0, sizeof(unsigned int))) != cudaSuccess) return cuda_fail(e, "cudaMemset(aad ticket)");
  if ((e = cudaMalloc(&h->d_sums, (size_t)kInterpChannels * sizeof(double) + (size_t)h->channels * sizeof(double))) !=
      cudaSuccess)
    return cuda_fail(e, "cudaMalloc(aad sums)");
  counters().allocations += 3;
  const int sms = device_ctx(dev)->sm_count;
  const size_t elt = h->f32 ? 4 : 8;
  if (engine == J4B_AAD_ENGINE_GENERATED) {
    if (!driver().ok) return fail(set_error(J4B_ECUDA, "CUDA driver entry points unavailable"));
    h->src = generate(*h);
    const auto t0 = std::chrono::steady_clock::now();
    std::vector<char> cubin;
    int rc = compile_source(h->src, "j4b_aad.cu", cubin, true);
    if (rc) return fail(rc);
    CUresult r = driver().ModuleLoadData(&h->mod, cubin.data());
    if (r != CUDA_SUCCESS) return fail(cu_error(r, "cuModuleLoadData(aad)"));
    r = driver().ModuleGetFunction(&h->fn, h->mod, "aad_replay");
    if (r != CUDA_SUCCESS) return fail(cu_error(r, "cuModuleGetFunction(aad_replay)"));
    h->compile_seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    int per_sm = 0;
    r = driver().Occupancy(&per_sm, h->fn, J4B_AAD_BLOCK, 0);
    if (r != CUDA_SUCCESS) return fail(cu_error(r, "cuOccupancyMaxActiveBlocksPerMultiprocessor(aad)"));
    h->gen_blocks_per_sm = std::max(1, per_sm);
  } else if (engine == J4B_AAD_ENGINE_INTERP) {
    std::vector<int4> rec;
    std::vector<int> in_dslot;
    plan_interp(*h, rec, in_dslot);
    if ((e = cudaMalloc(&h->d_nodes, rec.size() * sizeof(int4))) != cudaSuccess) return cuda_fail(e, "cudaMalloc(aad nodes)");
    if ((e = cudaMalloc(&h->d_consts, (size_t)n_nodes * sizeof(double))) != cudaSuccess)
      return cuda_fail(e, "cudaMalloc(aad constants)");
    if ((e = cudaMalloc(&h->d_in_nodes, in_dslot.size() * sizeof(int))) != cudaSuccess)
      return cuda_fail(e, "cudaMalloc(aad input slots)");
    counters().allocations += 3;
    cudaMemcpy(h->d_nodes, rec.data(), rec.size() * sizeof(int4), cudaMemcpyHostToDevice);
    cudaMemcpy(h->d_consts, constants, (size_t)n_nodes * sizeof(double), cudaMemcpyHostToDevice);
    cudaMemcpy(h->d_in_nodes, in_dslot.data(), in_dslot.size() * sizeof(int), cudaMemcpyHostToDevice);
    // Shared-memory slots (and records) when at least one warp's state fits a CTA (up to 256
    // threads per CTA, as many CTAs per SM as fit); otherwise [slot][thread] in global memory with
    // one CTA per SM, more while the scratch stays within L2. `scratch_option` > 0 forces the
    // global layout with that many threads.
    const int64_t per_thread = (int64_t)(h->nv + (h->adjoints ? h->nd : 0)) * (int64_t)elt;
    const int64_t rec_bytes = (int64_t)rec.size() * (int64_t)sizeof(int4);
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa;
    cudaFuncGetAttributes(&fa, interp_fn(h->f32, true));
    const int64_t smem_cap = (int64_t)optin - (int64_t)fa.sharedSizeBytes;
    const int64_t fit = smem_cap > rec_bytes ? (smem_cap - rec_bytes) / std::max<int64_t>(1, per_thread) / 32 * 32 : 0;
    if (scratch_option == 0 && fit >= 32) {
      const void* kfn = interp_fn(h->f32, true);
      h->interp_block = (int)std::min<int64_t>(J4B_AAD_BLOCK, fit);
      h->interp_smem = (size_t)(h->interp_block * per_thread + rec_bytes);
      if ((e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_cap)) != cudaSuccess)
        return cuda_fail(e, "cudaFuncSetAttribute(aad interpreter)");
      int per_sm = 1;
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, h->interp_block, h->interp_smem);
      h->interp_threads = (int64_t)sms * std::max(1, per_sm) * h->interp_block;
    } else {
      const void* kfn = interp_fn(h->f32, false);
      h->interp_block = J4B_AAD_BLOCK;
      h->interp_smem = 0;
      int per_sm = 1;
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, J4B_AAD_BLOCK, 0);
      int64_t threads = (int64_t)sms * std::max(1, per_sm) * J4B_AAD_BLOCK;
      threads = std::min(threads, std::max<int64_t>((int64_t)sms * J4B_AAD_BLOCK, kInterpL2Budget / std::max<int64_t>(1, per_thread)));
      if (scratch_option > 0) threads = scratch_option;
      h->interp_threads = std::max<int64_t>(J4B_AAD_BLOCK, threads / J4B_AAD_BLOCK * J4B_AAD_BLOCK);
      if ((e = cudaMalloc(&h->vs, (size_t)std::max<int64_t>(1, per_thread) * h->interp_threads)) != cudaSuccess)
        return cuda_fail(e, "cudaMalloc(aad interpreter slots)");
      counters().allocations++;
    }
  } else {
    // Scenarios per chunk bounded by the scratch budget (CudaEagerExecutable.java:81-85).
    const int64_t budget = scratch_option > 0 ? scratch_option : kEagerDefaultBytes;
    const int64_t per_scenario = (int64_t)n_nodes * (int64_t)elt * (h->adjoints ? 2 : 1);
    h->slot = std::max<int64_t>(J4B_AAD_BLOCK, std::min<int64_t>(1 << 20, budget / per_scenario));
    if ((e = cudaMalloc(&h->vs, (size_t)n_nodes * h->slot * elt)) != cudaSuccess)
      return cuda_fail(e, "cudaMalloc(aad eager values)");
    if (h->adjoints && (e = cudaMalloc(&h->ds, (size_t)n_nodes * h->slot * elt)) != cudaSuccess)
      return cuda_fail(e, "cudaMalloc(aad eager adjoints)");
    counters().allocations += h->adjoints ? 2 : 1;
  }
  *out = h;
  return J4B_OK;
}

extern "C" int j4b_aad_launch(j4b_aad_t h, j4b_buf inputs, uint64_t paths, uint64_t path_offset, uint64_t seed,
                              j4b_buf sums, j4b_stream s) {
  J4B_REQUIRE(h != nullptr, "null AAD executable");
  J4B_REQUIRE(paths > 0, "paths must be positive");
  J4B_REQUIRE(sums != 0 && (h->n_in == 0 || inputs != 0), "AAD launch needs device inputs and sums");
  DeviceGuard guard(h->dev);
  cudaStream_t st = resolve_stream(h->dev, s);
  double* saved = h->d_sums;
  h->d_sums = (double*)(uintptr_t)sums;
  int rc = launch_replay(h, h->n_in ? (const double*)(uintptr_t)inputs : h->d_inputs, paths, path_offset, seed, st);
  h->d_sums = saved;
  return rc;
}

extern "C" int j4b_aad_replay(j4b_aad_t h, const double* inputs, uint64_t paths, uint64_t path_offset,
                              uint64_t seed, double* sums, j4b_stream s) {
  J4B_REQUIRE(h != nullptr, "null AAD executable");
  J4B_REQUIRE(paths > 0, "paths must be positive");
  J4B_REQUIRE(sums != nullptr && (h->n_in == 0 || inputs != nullptr), "AAD replay needs inputs and a sums array");
  DeviceGuard guard(h->dev);
  cudaStream_t st = resolve_stream(h->dev, s);
  if (h->n_in) {
    J4B_CUDA(cudaMemcpyAsync(h->d_inputs, inputs, (size_t)h->n_in * sizeof(double), cudaMemcpyHostToDevice, st),
             "cudaMemcpyAsync(aad inputs)");
    counters().h2d += (uint64_t)h->n_in * sizeof(double);
  }
  int rc = launch_replay(h, h->d_inputs, paths, path_offset, seed, st);
  if (rc) return rc;
  J4B_CUDA(cudaMemcpyAsync(sums, h->d_sums, (size_t)h->channels * sizeof(double), cudaMemcpyDeviceToHost, st),
           "cudaMemcpyAsync(aad sums)");
  counters().d2h += (uint64_t)h->channels * sizeof(double);
  J4B_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize(aad replay)");
  return J4B_OK;
}

extern "C" int j4b_aad_info(j4b_aad_t h, int* channels, double* compile_seconds, int64_t* threads_or_slot) {
  J4B_REQUIRE(h != nullptr, "null AAD executable");
  if (channels) *channels = h->channels;
  if (compile_seconds) *compile_seconds = h->compile_seconds;
  if (threads_or_slot)
    *threads_or_slot = h->engine == J4B_AAD_ENGINE_INTERP ? h->interp_threads
                       : h->engine == J4B_AAD_ENGINE_EAGER ? h->slot
                                                           : (int64_t)device_ctx(h->dev)->sm_count * h->gen_blocks_per_sm *
                                                                 J4B_AAD_BLOCK;
  return J4B_OK;
}

extern "C" int j4b_aad_source(j4b_aad_t h, char* buf, size_t cap, size_t* len) {
  J4B_REQUIRE(h != nullptr, "null AAD executable");
  if (len) *len = h->src.size();
  if (buf && cap) {
    const size_t n = std::min(cap - 1, h->src.size());
    memcpy(buf, h->src.data(), n);
    buf[n] = '\0';
  }
  return J4B_OK;
}

extern "C" int j4b_aad_free(j4b_aad_t h) {
  if (!h) return J4B_OK;
  aad_release(h);
  return J4B_OK;
}
