// Fused tape executor: j4b_tape_compile / j4b_tape_launch / j4b_tape_free.
//
// Replaces ExecutionPlan.capture/execute (core/tensor/ExecutionPlan.java:49-132) and the
// reference CUDA backend's one-NVRTC-kernel-per-fused-call path (cuda/backend/cuda/
// CudaBackend.java:883-1006). A tape is the call list the front end recorded (the same calls the
// reference's recording proxy sees). The compiler walks it once and groups calls into *row
// programs*: one sm_100a kernel per group, generated as CUDA C++ and compiled with NVRTC, where
//   - ROW values are per-row tensors: a CTA owns row r of every [R, W] tensor of the group and
//     keeps it in registers (float4 slots: element j = (e*NT + t)*4 + q of thread t);
//   - SHARED values are row-invariant (broadcast gains, constants, small parameter tensors),
//     computed once per CTA before the row loop;
//   - POST values depend on reductions across rows (column sums such as a broadcast's
//     gradient, global sums such as a loss): each CTA accumulates its rows in double, writes a
//     partial, and a small fold kernel sums the partials in CTA order (deterministic) and
//     evaluates what follows.
// Elementwise chains (fused/binary/scalar/unary), row reductions (warp shuffles + shared
// memory), broadcasts and static gather/scatter maps that stay inside a row (the vmap slices
// and their transposes) are fused; reshape and slice are views. Calls that are real
// contractions or data movement (matmul, transpose, stack, random, irregular maps) run as the
// engine's own eager kernels between groups, with their operands materialised in an arena that
// is allocated once per compiled tape.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <nvrtc.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <unordered_map>
#include <vector>

#include "j4b_internal.h"
#include "j4b_rtc.h"

namespace j4b {
namespace {

enum : int {
  T_FULL = 1, T_FUSED, T_TRANSPOSE, T_MATMUL, T_BMM, T_SLICE0, T_STACK0, T_RSUM, T_RMAX, T_SUMAX,
  T_MAXAX, T_ARGMAX, T_MAXBWD, T_RESHAPE, T_BCAST, T_REINDEX, T_SCATTER, T_RELUBWD, T_RUNIF,
  T_RNORM, T_BINARY, T_SCALAR, T_UNARY, T_LAST
};

constexpr int64_t kTapeMagic = 0x314550415442344ALL;  // "J4BTAPE1"
// Row and fold kernels are launched with programmatic dependent launch: each waits for the kernel
// before it (and its memory) before touching memory, and at once lets the next kernel in the
// stream be scheduled, so a launch's set-up overlaps the tail of the previous one (a fold kernel
// is resident before its row kernel ends).
constexpr const char* kPdlPrologue =
    "  asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n"
    "  asm volatile(\"griddepcontrol.launch_dependents;\" ::: \"memory\");\n";
constexpr int64_t kSharedMax = 16384;  // largest row-invariant vector kept per CTA
// fold kernel: 8 warps per 32-column slice (32 warps measured 2% slower per tape step)
constexpr int kFoldThreads = 256;
constexpr int64_t kRowMax = 16384;     // widest row a CTA keeps in registers
constexpr int kMaxPtrs = 96;

using Shape = std::vector<int64_t>;

int64_t numel(const Shape& s) {
  int64_t n = 1;
  for (int64_t d : s) n *= d;
  return n;
}

struct TCall {
  int op = 0, out = -1;
  std::vector<int> ins;
  std::vector<int64_t> at;
};

struct TapeIR {
  std::vector<Shape> shape;
  std::vector<int64_t> size;
  std::vector<int> inputs, outputs;
  std::vector<TCall> calls;
};

// ---------------------------------------------------------------------------------------------
// elementwise expressions (fused programs), deduplicated by structure
// ---------------------------------------------------------------------------------------------

struct ENode {
  int kind = 0;  // 0 input, 1 unary, 2 binary, 3 scalar
  int op = 0, a = -1, b = -1, idx = -1;
  double val = 0;
};

bool parse_program(const std::vector<int64_t>& w, int nin, std::vector<ENode>& nodes, int* root,
                   std::string& err) {
  std::map<std::tuple<int, int, int, int, int, uint64_t>, int> memo;
  std::vector<int> stack;
  auto intern = [&](ENode n) {
    uint64_t vb;
    std::memcpy(&vb, &n.val, 8);
    auto key = std::make_tuple(n.kind, n.op, n.a, n.b, n.idx, vb);
    auto it = memo.find(key);
    if (it != memo.end()) return it->second;
    nodes.push_back(n);
    memo[key] = (int)nodes.size() - 1;
    return (int)nodes.size() - 1;
  };
  for (size_t pc = 0; pc < w.size();) {
    int kind = (int)w[pc];
    if (kind == 0 && pc + 1 < w.size()) {
      int idx = (int)w[pc + 1];
      if (idx < 0 || idx >= nin) { err = "fused program input out of range"; return false; }
      ENode n; n.kind = 0; n.idx = idx;
      stack.push_back(intern(n));
      pc += 2;
    } else if (kind == 1 && pc + 1 < w.size()) {
      int op = (int)w[pc + 1];
      if (op < J4B_NEG || op > J4B_SIGN || stack.empty()) { err = "bad unary in fused program"; return false; }
      ENode n; n.kind = 1; n.op = op; n.a = stack.back();
      stack.back() = intern(n);
      pc += 2;
    } else if (kind == 2 && pc + 1 < w.size()) {
      int op = (int)w[pc + 1];
      if (op < J4B_ADD || op > J4B_MIN || stack.size() < 2) { err = "bad binary in fused program"; return false; }
      ENode n; n.kind = 2; n.op = op; n.b = stack.back(); stack.pop_back(); n.a = stack.back();
      stack.back() = intern(n);
      pc += 2;
    } else if (kind == 3 && pc + 3 < w.size()) {
      int op = (int)w[pc + 1];
      if (op < J4B_ADD || op > J4B_MIN || stack.empty()) { err = "bad scalar in fused program"; return false; }
      uint32_t lo = (uint32_t)w[pc + 2], hi = (uint32_t)w[pc + 3];
      uint64_t bits = ((uint64_t)hi << 32) | lo;
      ENode n; n.kind = 3; n.op = op; n.a = stack.back();
      std::memcpy(&n.val, &bits, 8);
      stack.back() = intern(n);
      pc += 4;
    } else {
      err = "malformed fused program";
      return false;
    }
  }
  if (stack.size() != 1) { err = "fused program must leave one value"; return false; }
  *root = stack[0];
  return true;
}

// ---------------------------------------------------------------------------------------------
// index maps of reindex / scatterAdd: affine (offset + strides over the gather-side multi-index)
// or an explicit table, as serialised by the front end.
// ---------------------------------------------------------------------------------------------

struct IndexMap {
  bool affine = false;
  int64_t off = 0;
  Shape dims, strides;             // affine: over the gather side's shape
  std::vector<int64_t> table;      // explicit
  int64_t at(int64_t f) const {
    if (!affine) return table[(size_t)f];
    int64_t v = off;
    for (int d = (int)dims.size() - 1; d >= 0; --d) {
      int64_t c = f % dims[d];
      f /= dims[d];
      v += c * strides[d];
    }
    return v;
  }
};

bool decode_map(const std::vector<int64_t>& at, const Shape& side, int64_t limit, IndexMap& m,
                std::string& err) {
  if (at.empty()) { err = "missing index map"; return false; }
  if (at[0] == 1) {
    if (at.size() < 3 || at[2] != (int64_t)side.size() || at.size() != 3 + side.size()) {
      err = "bad affine map"; return false;
    }
    m.affine = true;
    m.off = at[1];
    m.dims = side;
    m.strides.assign(at.begin() + 3, at.end());
    int64_t lo = m.off, hi = m.off;
    for (size_t d = 0; d < side.size(); ++d) {
      if (side[d] == 0) { lo = 0; hi = -1; break; }
      int64_t span = m.strides[d] * (side[d] - 1);
      (span < 0 ? lo : hi) += span;
    }
    if (numel(side) > 0 && (lo < 0 || hi >= limit)) { err = "index out of bounds"; return false; }
    return true;
  }
  if (at[0] == 0 && at.size() >= 2 && at[1] == numel(side) && (int64_t)at.size() == 2 + at[1]) {
    m.affine = false;
    m.table.assign(at.begin() + 2, at.end());
    for (int64_t v : m.table)
      if (v < -1 || v >= limit) { err = "index out of bounds"; return false; }
    return true;
  }
  err = "bad index map";
  return false;
}

// ---------------------------------------------------------------------------------------------
// parsing and validation
// ---------------------------------------------------------------------------------------------

bool parse_tape(const int64_t* w, size_t n, TapeIR& t, std::string& err) {
  size_t p = 0;
  auto take = [&](int64_t* v) {
    if (p >= n) return false;
    *v = w[p++];
    return true;
  };
  int64_t magic, nb, ni, no, nc;
  if (!take(&magic) || magic != kTapeMagic || !take(&nb) || !take(&ni) || !take(&no) || !take(&nc)) {
    err = "bad tape header"; return false;
  }
  if (nb < 0 || nb > (1 << 24) || ni < 0 || ni > nb || no < 0 || no > nb || nc < 0 || nc > (1 << 24)) {
    err = "bad tape counts"; return false;
  }
  t.shape.resize(nb);
  t.size.resize(nb);
  for (int64_t b = 0; b < nb; ++b) {
    int64_t rank;
    if (!take(&rank) || rank < 0 || rank > 8) { err = "bad buffer rank"; return false; }
    int64_t sz = 1;
    for (int64_t d = 0; d < rank; ++d) {
      int64_t v;
      if (!take(&v) || v < 0 || v > (int64_t(1) << 40)) { err = "bad buffer dim"; return false; }
      t.shape[b].push_back(v);
      sz *= v;
      if (sz > (int64_t(1) << 40)) { err = "buffer too large"; return false; }
    }
    t.size[b] = sz;
  }
  auto id_ok = [&](int64_t v) { return v >= 0 && v < nb; };
  for (int64_t i = 0; i < ni; ++i) {
    int64_t v;
    if (!take(&v) || !id_ok(v)) { err = "bad input id"; return false; }
    t.inputs.push_back((int)v);
  }
  for (int64_t i = 0; i < no; ++i) {
    int64_t v;
    if (!take(&v) || !id_ok(v)) { err = "bad output id"; return false; }
    t.outputs.push_back((int)v);
  }
  for (int64_t c = 0; c < nc; ++c) {
    TCall call;
    int64_t op, out, nin, nat;
    if (!take(&op) || op < T_FULL || op >= T_LAST || !take(&out) || !id_ok(out) || !take(&nin) ||
        nin < 0 || nin > nb) {
      err = "bad call header"; return false;
    }
    call.op = (int)op;
    call.out = (int)out;
    for (int64_t i = 0; i < nin; ++i) {
      int64_t v;
      if (!take(&v) || !id_ok(v)) { err = "bad call operand"; return false; }
      call.ins.push_back((int)v);
    }
    if (!take(&nat) || nat < 0 || (size_t)nat > n - p) { err = "bad call attributes"; return false; }
    call.at.assign(w + p, w + p + nat);
    p += (size_t)nat;
    t.calls.push_back(std::move(call));
  }
  if (p != n) { err = "trailing words after tape"; return false; }
  return true;
}

Shape reduced_shape(const Shape& s, int axis, bool keep) {
  Shape o;
  for (int i = 0; i < (int)s.size(); ++i) {
    if (i == axis) {
      if (keep) o.push_back(1);
    } else {
      o.push_back(s[i]);
    }
  }
  return o;
}

void axis_split(const Shape& s, int axis, int64_t* outer, int64_t* n, int64_t* inner) {
  *outer = 1;
  *inner = 1;
  for (int i = 0; i < axis; ++i) *outer *= s[i];
  *n = s[axis];
  for (int i = axis + 1; i < (int)s.size(); ++i) *inner *= s[i];
}

bool broadcastable(const Shape& s, const Shape& t) {
  if (s.size() > t.size()) return false;
  size_t pad = t.size() - s.size();
  for (size_t i = 0; i < s.size(); ++i)
    if (s[i] != t[pad + i] && s[i] != 1) return false;
  return true;
}

// Checks operand counts, attributes and shapes of every call against the SPI's contracts
// (ComputeBackend.java and CpuBackend.java argument checks), and the def-before-use order.
bool validate(TapeIR& t, std::string& err) {
  std::vector<char> defined(t.shape.size(), 0);
  for (int b : t.inputs) {
    if (defined[b]) { err = "duplicate input"; return false; }
    defined[b] = 1;
  }
  for (size_t ci = 0; ci < t.calls.size(); ++ci) {
    TCall& c = t.calls[ci];
    for (int b : c.ins)
      if (!defined[b]) { err = "operand used before definition"; return false; }
    if (defined[c.out]) { err = "buffer defined twice"; return false; }
    const Shape& os = t.shape[c.out];
    auto in_shape = [&](int i) -> const Shape& { return t.shape[c.ins[i]]; };
    auto in_size = [&](int i) { return t.size[c.ins[i]]; };
    auto arity = [&](size_t k) { return c.ins.size() == k; };
    bool ok = true;
    switch (c.op) {
      case T_FULL: ok = arity(0) && c.at.size() == 1; break;
      case T_FUSED: {
        ok = !c.ins.empty();
        for (size_t i = 0; ok && i < c.ins.size(); ++i) ok = in_size((int)i) == t.size[c.out];
        if (!ok) { err = "fused inputs must share element count"; return false; }
        std::vector<ENode> nodes;
        int root;
        if (!parse_program(c.at, (int)c.ins.size(), nodes, &root, err)) return false;
        break;
      }
      case T_BINARY:
        ok = arity(2) && c.at.size() == 1 && c.at[0] >= J4B_ADD && c.at[0] <= J4B_MIN &&
             in_size(0) == in_size(1) && t.size[c.out] == in_size(0);
        break;
      case T_SCALAR:
        ok = arity(1) && c.at.size() == 2 && c.at[0] >= J4B_ADD && c.at[0] <= J4B_MIN &&
             t.size[c.out] == in_size(0);
        break;
      case T_UNARY:
        ok = arity(1) && c.at.size() == 1 && c.at[0] >= J4B_NEG && c.at[0] <= J4B_SIGN &&
             t.size[c.out] == in_size(0);
        break;
      case T_RELUBWD: ok = arity(2) && in_size(0) == in_size(1) && t.size[c.out] == in_size(0); break;
      case T_TRANSPOSE:
        ok = arity(1) && in_shape(0).size() == 2 && os.size() == 2 && os[0] == in_shape(0)[1] &&
             os[1] == in_shape(0)[0];
        break;
      case T_MATMUL:
        ok = arity(2) && in_shape(0).size() == 2 && in_shape(1).size() == 2 &&
             in_shape(0)[1] == in_shape(1)[0] && os == Shape{in_shape(0)[0], in_shape(1)[1]};
        if (!ok) { err = "incompatible matmul shapes"; return false; }
        break;
      case T_BMM:
        ok = arity(2) && in_shape(0).size() == 3 && in_shape(1).size() == 3 &&
             in_shape(0)[0] == in_shape(1)[0] && in_shape(0)[2] == in_shape(1)[1] &&
             os == Shape{in_shape(0)[0], in_shape(0)[1], in_shape(1)[2]};
        if (!ok) { err = "incompatible batched matmul shapes"; return false; }
        break;
      case T_SLICE0:
        ok = arity(1) && c.at.size() == 1 && !in_shape(0).empty() && c.at[0] >= 0 &&
             c.at[0] < in_shape(0)[0] && os == Shape(in_shape(0).begin() + 1, in_shape(0).end());
        break;
      case T_STACK0: {
        ok = !c.ins.empty();
        for (size_t i = 0; ok && i < c.ins.size(); ++i) ok = in_shape((int)i) == in_shape(0);
        if (ok) {
          Shape want{(int64_t)c.ins.size()};
          want.insert(want.end(), in_shape(0).begin(), in_shape(0).end());
          ok = os == want;
        }
        break;
      }
      case T_RSUM: case T_RMAX: ok = arity(1) && t.size[c.out] == 1; break;
      case T_SUMAX: case T_MAXAX:
        ok = arity(1) && c.at.size() == 2 && c.at[0] >= 0 && c.at[0] < (int64_t)in_shape(0).size() &&
             os == reduced_shape(in_shape(0), (int)c.at[0], c.at[1] != 0);
        break;
      case T_ARGMAX:
        ok = arity(1) && c.at.size() == 1 && c.at[0] >= 0 && c.at[0] < (int64_t)in_shape(0).size() &&
             os == reduced_shape(in_shape(0), (int)c.at[0], false);
        break;
      case T_MAXBWD: {
        ok = arity(2) && c.at.size() == 1 && c.at[0] >= 0 && c.at[0] < (int64_t)in_shape(1).size() &&
             os == in_shape(1);
        if (ok) {
          int64_t o, nn, in;
          axis_split(in_shape(1), (int)c.at[0], &o, &nn, &in);
          ok = in_size(0) == o * in;
        }
        break;
      }
      case T_RESHAPE: ok = arity(1) && t.size[c.out] == in_size(0); break;
      case T_BCAST: ok = arity(1) && broadcastable(in_shape(0), os); break;
      case T_REINDEX: case T_SCATTER: {
        ok = arity(1);
        if (ok) {
          IndexMap m;
          const Shape& side = c.op == T_REINDEX ? os : in_shape(0);
          int64_t limit = c.op == T_REINDEX ? in_size(0) : t.size[c.out];
          if (!decode_map(c.at, side, limit, m, err)) return false;
        }
        break;
      }
      case T_RUNIF: case T_RNORM: ok = arity(0) && c.at.size() == 2; break;
      default: ok = false;
    }
    if (!ok) {
      char buf[96];
      snprintf(buf, sizeof buf, "invalid call %zu (op %d): operands, attributes or shapes", ci, c.op);
      err = buf;
      return false;
    }
    defined[c.out] = 1;
  }
  for (int b : t.outputs)
    if (!defined[b]) { err = "output never defined"; return false; }
  return true;
}

// ---------------------------------------------------------------------------------------------
// planning: contexts, views and groups
// ---------------------------------------------------------------------------------------------

enum Ctx : int { X_NONE = 0, X_GLOBAL, X_CONST, X_ROW, X_SHARED, X_POST };

// Per-row (or per-vector) index table of a view: element j of the view reads element tbl[j] of
// its base (-1 reads zero).
using Table = std::shared_ptr<const std::vector<int64_t>>;

struct Val {
  int ctx = X_NONE;
  int kernel = -1;
  int64_t W = 0;          // ROW: row width; SHARED / POST / GLOBAL: element count
  int base = -1;          // view: base value id (never itself a view)
  bool base_rows = false; // view over a per-row base (row r of it) rather than a whole vector
  Table tbl;
  float cval = 0;
  int root = -1;          // GLOBAL: storage root and element offset
  int64_t off = 0;
  bool need_store = false;
};

// What one fused call computes inside a group.
enum GKind : int {
  G_EXPR = 1,   // elementwise expression
  G_VIEW,       // broadcast / reindex / scatter / view: no code
  G_RRED,       // reduction inside a row (or inside a shared vector)
  G_COLRED,     // reduction across rows, one value per column
  G_GLOBRED,    // reduction of everything
};

struct GCall {
  int call = -1;
  int kind = 0;
  int ctx = 0;            // context the result lives in
  int red = 0;            // T_SUMAX/T_MAXAX/T_ARGMAX/T_MAXBWD/T_RSUM/T_RMAX
  int64_t n = 0, inner = 1;  // in-row reduction: reduced extent and inner stride
};

struct Group {
  int64_t R = -1;
  std::vector<GCall> calls;
  bool has_post = false;
  bool has_rows = false;
};

enum StepKind : int { S_GROUP = 1, S_EAGER, S_FILL, S_COPY };

struct Step {
  int kind = 0;
  int group = -1;
  int call = -1;
  int buf = -1;     // fill: buffer; copy: source value
  int out_index = -1;
};

struct Planner {
  TapeIR& t;
  std::vector<Val> V;
  std::vector<Group> groups;
  std::vector<Step> steps;
  std::vector<int> fills;
  // tsrc[b] = the source of transpose output b when every consumer of b is a matmul, which then
  // reads the source transposed in place (b is never materialised); else -1
  std::vector<int> tsrc;
  int cur = -1;
  std::string err;

  explicit Planner(TapeIR& tape) : t(tape), V(tape.shape.size()), tsrc(tape.shape.size(), -1) {}

  // ---- helpers ----
  int64_t choose_R(const Shape& s) const {
    int64_t n = numel(s);
    if (s.size() >= 2) return s[0];
    for (int64_t w = 4096; w >= 1; w /= 2)
      if (n % w == 0) return n / w;
    return n;
  }

  // How value b appears inside group g.
  int ctx_in(int b, int g) const {
    const Val& v = V[b];
    if (v.ctx == X_CONST) return X_CONST;
    if ((v.ctx == X_ROW || v.ctx == X_SHARED || v.ctx == X_POST) && v.kernel == g) return v.ctx;
    return X_GLOBAL;
  }

  static Table compose(const Table& inner_tbl, const std::vector<int64_t>& outer) {
    // view of a view: outer maps into the inner view's elements, inner into the base
    if (!inner_tbl) return std::make_shared<const std::vector<int64_t>>(outer);
    auto res = std::make_shared<std::vector<int64_t>>(outer.size());
    for (size_t j = 0; j < outer.size(); ++j)
      (*res)[j] = outer[j] < 0 ? -1 : (*inner_tbl)[(size_t)outer[j]];
    return res;
  }

  // Makes value `out` a view of value `src` through `tbl`. `rows` says whether the table indexes
  // the source's row r (a per-row source) or the whole source vector.
  void make_view(Val& out, int src, bool src_rows, std::vector<int64_t>&& tbl) {
    const Val& s = V[src];
    if (s.base >= 0) {
      out.base = s.base;
      out.base_rows = s.base_rows;
      out.tbl = compose(s.tbl, tbl);
    } else {
      out.base = src;
      out.base_rows = src_rows;
      out.tbl = std::make_shared<const std::vector<int64_t>>(std::move(tbl));
    }
  }

  // A rank >= 2 tensor with more than one leading row is computed per row (one CTA per row)
  // rather than as a row-invariant vector, when its rows match the group's.
  static bool rowish(const Shape& s, int64_t R) { return s.size() >= 2 && s[0] > 1 && (R < 0 || s[0] == R); }

  bool row_ok(int64_t R, int64_t n, int64_t* W) const {
    if (R <= 0 || n % R != 0) return false;
    *W = n / R;
    return *W <= kRowMax;
  }

  // Attempts to place call ci in group g (which may be fresh, R = -1). On success fills `out`
  // (the result value), `gc` and `newR`. No side effects.
  bool classify(int ci, int g, Val& out, GCall& gc, int64_t& newR) {
    const TCall& c = t.calls[ci];
    const Group& G = groups[g];
    newR = G.R;
    gc = GCall();
    gc.call = ci;
    out = Val();
    out.kernel = g;
    const int64_t n_out = t.size[c.out];
    auto need_R = [&](const Shape& s) -> bool {
      if (newR < 0) newR = choose_R(s);
      return newR > 0;
    };

    switch (c.op) {
      case T_FUSED: case T_BINARY: case T_SCALAR: case T_UNARY: case T_RELUBWD: {
        bool row = false, post = false, shared = false, big_global = false;
        for (int b : c.ins) {
          int x = ctx_in(b, g);
          row |= x == X_ROW;
          post |= x == X_POST;
          shared |= x == X_SHARED;
          big_global |= x == X_GLOBAL && t.size[b] > kSharedMax;
        }
        gc.kind = G_EXPR;
        if (row && post) return false;
        if (post) {
          if (big_global) return false;
          gc.ctx = out.ctx = X_POST;
          out.W = n_out;
          return true;
        }
        if (row || big_global || n_out > kSharedMax || (!shared && rowish(t.shape[c.out], newR))) {
          if (!need_R(t.shape[c.out])) return false;
          int64_t W;
          if (!row_ok(newR, n_out, &W)) return false;
          if (shared && newR != 1) return false;  // a shared vector indexed by (row, column)
          gc.ctx = out.ctx = X_ROW;
          out.W = W;
          return true;
        }
        gc.ctx = out.ctx = X_SHARED;
        out.W = n_out;
        return true;
      }
      case T_BCAST: {
        int b = c.ins[0];
        const Shape& S = t.shape[b];
        const Shape& T = t.shape[c.out];
        Shape Sp(T.size() - S.size(), 1);
        Sp.insert(Sp.end(), S.begin(), S.end());
        int x = ctx_in(b, g);
        gc.kind = G_VIEW;
        if (x == X_CONST) { out = V[b]; gc.ctx = X_CONST; return true; }
        // stride of each target dim into the source (0 where broadcast)
        Shape sstr(T.size(), 0);
        {
          int64_t st = 1;
          for (int d = (int)T.size() - 1; d >= 0; --d) {
            sstr[d] = Sp[d] == 1 ? 0 : st;
            st *= Sp[d];
          }
        }
        auto table_over = [&](int d0) {
          // element j of dims T[d0:] -> source index (dims d0.. of Sp)
          int64_t w = 1;
          for (size_t d = d0; d < T.size(); ++d) w *= T[d];
          std::vector<int64_t> tb((size_t)w);
          for (int64_t j = 0; j < w; ++j) {
            int64_t f = j, src = 0;
            for (int d = (int)T.size() - 1; d >= d0; --d) {
              int64_t cc = f % T[d];
              f /= T[d];
              src += cc * sstr[d];
            }
            tb[(size_t)j] = src;
          }
          return tb;
        };
        if (x == X_POST) {
          // the fold kernel handles scalar broadcasts and identity views only
          if (t.size[b] != 1 && t.size[b] != n_out) return false;
          if (V[b].base >= 0) return false;
          gc.ctx = out.ctx = X_POST;
          out.W = n_out;
          out.base = b;
          if (t.size[b] == 1 && n_out != 1)
            out.tbl = std::make_shared<const std::vector<int64_t>>((size_t)n_out, 0);
          return true;
        }
        bool as_rows = x == X_ROW || (x == X_GLOBAL && (t.size[b] > kSharedMax || rowish(S, newR)));
        if (as_rows) {
          if (T.empty()) return false;
          if (newR < 0) newR = T[0];
          if (T[0] != newR || Sp[0] != newR) return false;
          int64_t W;
          if (!row_ok(newR, n_out, &W)) return false;
          gc.ctx = out.ctx = X_ROW;
          out.W = W;
          make_view(out, b, true, table_over(1));
          return true;
        }
        // shared or small global source: a row view when the target is per-row data
        bool shared_ok = n_out <= kSharedMax;
        if (!T.empty() && Sp[0] == 1 && (n_out > kSharedMax || rowish(T, newR))) {
          int64_t R2 = newR < 0 ? T[0] : newR;
          int64_t W;
          if (T[0] == R2 && row_ok(R2, n_out, &W)) {
            newR = R2;
            gc.ctx = out.ctx = X_ROW;
            out.W = W;
            make_view(out, b, false, table_over(1));
            return true;
          }
        }
        if (!shared_ok) return false;
        gc.ctx = out.ctx = X_SHARED;
        out.W = n_out;
        make_view(out, b, false, table_over(0));
        return true;
      }
      case T_REINDEX: case T_SCATTER: {
        int b = c.ins[0];
        int x = ctx_in(b, g);
        if (x == X_POST || x == X_CONST) return false;
        IndexMap m;
        std::string e2;
        const Shape& side = c.op == T_REINDEX ? t.shape[c.out] : t.shape[b];
        int64_t limit = c.op == T_REINDEX ? t.size[b] : n_out;
        if (!decode_map(c.at, side, limit, m, e2)) return false;
        const int64_t n_in = t.size[b];
        gc.kind = G_VIEW;
        bool as_rows = x == X_ROW || (x == X_GLOBAL && (n_in > kSharedMax || rowish(t.shape[b], newR)));
        auto shared_table = [&]() -> bool {
          std::vector<int64_t> tb((size_t)n_out, -1);
          if (c.op == T_REINDEX) {
            for (int64_t f = 0; f < n_out; ++f) tb[(size_t)f] = m.at(f);
          } else {
            for (int64_t f = 0; f < n_in; ++f) {
              int64_t k = m.at(f);
              if (k < 0) continue;
              if (tb[(size_t)k] >= 0) return false;  // not injective: a real scatter-add
              tb[(size_t)k] = f;
            }
          }
          gc.ctx = out.ctx = X_SHARED;
          out.W = n_out;
          make_view(out, b, false, std::move(tb));
          return true;
        };
        const bool small = !as_rows && n_out <= kSharedMax;
        if (small && !rowish(t.shape[c.out], newR)) return shared_table();
        const int64_t R0 = newR;
        if (newR < 0) newR = side.size() >= 1 ? side[0] : -1;
        if (newR <= 0 || n_out % newR || n_in % newR) {
          newR = R0;
          return small && shared_table();
        }
        const int64_t Wout = n_out / newR, Win = n_in / newR;
        if (Wout > kRowMax || Win > kRowMax) return false;
        std::vector<int64_t> tb((size_t)Wout, -1);
        if (c.op == T_REINDEX) {
          for (int64_t j = 0; j < Wout; ++j) {
            int64_t v = m.at(j);
            if (as_rows && v >= Win) return false;
            tb[(size_t)j] = v;
          }
          for (int64_t r = 1; r < newR; ++r)
            for (int64_t j = 0; j < Wout; ++j) {
              int64_t v = m.at(r * Wout + j), h = tb[(size_t)j];
              int64_t want = h < 0 ? -1 : (as_rows ? r * Win + h : h);
              if (v != want) return false;
            }
        } else {
          if (!as_rows) {
            newR = R0;
            return small && shared_table();
          }
          std::vector<int64_t> g0((size_t)Win);
          for (int64_t cidx = 0; cidx < Win; ++cidx) {
            int64_t k = m.at(cidx);
            if (k >= Wout) return false;
            g0[(size_t)cidx] = k;
            if (k >= 0) {
              if (tb[(size_t)k] >= 0) return false;
              tb[(size_t)k] = cidx;
            }
          }
          for (int64_t r = 1; r < newR; ++r)
            for (int64_t cidx = 0; cidx < Win; ++cidx) {
              int64_t v = m.at(r * Win + cidx), h = g0[(size_t)cidx];
              if (v != (h < 0 ? -1 : r * Wout + h)) return false;
            }
        }
        gc.ctx = out.ctx = X_ROW;
        out.W = Wout;
        make_view(out, b, as_rows, std::move(tb));
        return true;
      }
      case T_SUMAX: case T_MAXAX: case T_ARGMAX: case T_MAXBWD: {
        int src = c.op == T_MAXBWD ? c.ins[1] : c.ins[0];
        int axis = (int)c.at[0];
        int64_t outer, nn, inner;
        axis_split(t.shape[src], axis, &outer, &nn, &inner);
        int x = ctx_in(src, g);
        if (x == X_POST || x == X_CONST) return false;
        if (c.op == T_MAXBWD) {
          int xu = ctx_in(c.ins[0], g);
          if (xu == X_POST) return false;
        }
        gc.red = c.op;
        gc.n = nn;
        gc.inner = inner;
        const int64_t n_in = t.size[src];
        bool as_rows = x == X_ROW || (x == X_GLOBAL && (n_in > kSharedMax || rowish(t.shape[src], newR)));
        if (!as_rows) {
          if (n_in > kSharedMax || nn == 0) return false;
          if (c.op == T_MAXBWD && ctx_in(c.ins[0], g) == X_ROW) return false;
          gc.kind = G_RRED;
          gc.ctx = out.ctx = X_SHARED;
          out.W = n_out;
          return true;
        }
        if (newR < 0) newR = t.shape[src].empty() ? -1 : t.shape[src][0];
        int64_t W;
        if (!row_ok(newR, n_in, &W)) return false;
        if (nn > 0 && W % (nn * inner) == 0) {
          if (c.op == T_MAXBWD) {
            int xu = ctx_in(c.ins[0], g);
            if (xu == X_SHARED && newR != 1) return false;
          }
          gc.kind = G_RRED;
          gc.ctx = out.ctx = X_ROW;
          out.W = c.op == T_MAXBWD ? W : W / nn;
          return true;
        }
        if ((c.op == T_SUMAX || c.op == T_MAXAX) && outer == 1 && nn == newR && inner == W) {
          gc.kind = G_COLRED;
          gc.ctx = out.ctx = X_POST;
          out.W = W;
          return true;
        }
        return false;
      }
      case T_RSUM: case T_RMAX: {
        int b = c.ins[0];
        int x = ctx_in(b, g);
        if (x == X_POST || x == X_CONST) return false;
        gc.red = c.op;
        bool as_rows = x == X_ROW || (x == X_GLOBAL && (t.size[b] > kSharedMax || rowish(t.shape[b], newR)));
        if (!as_rows) {
          if (t.size[b] == 0) return false;
          gc.kind = G_RRED;
          gc.n = t.size[b];
          gc.inner = 1;
          gc.ctx = out.ctx = X_SHARED;
          out.W = 1;
          return true;
        }
        if (!need_R(t.shape[b])) return false;
        int64_t W;
        if (!row_ok(newR, t.size[b], &W)) return false;
        gc.kind = G_GLOBRED;
        gc.ctx = out.ctx = X_POST;
        out.W = 1;
        return true;
      }
      default:
        return false;
    }
  }

  void commit(int ci, int g, Val& out, GCall& gc, int64_t newR) {
    const TCall& c = t.calls[ci];
    Group& G = groups[g];
    G.R = newR;
    for (int b : c.ins) {
      int x = ctx_in(b, g);
      if (x == X_GLOBAL) ensure_global(b);
      if (x == X_SHARED && gc.ctx == X_POST) ensure_global(b);
    }
    if (out.base >= 0 && ctx_in(out.base, g) == X_GLOBAL) ensure_global(out.base);
    if (gc.ctx == X_POST) G.has_post = true;
    if (gc.ctx == X_ROW || gc.kind == G_COLRED || gc.kind == G_GLOBRED) G.has_rows = true;
    G.calls.push_back(gc);
    V[c.out] = out;
  }

  // The value must exist in device memory (for an eager step, a later group or an output).
  // An identity alias (a reshape of a group value) is materialised through its base.
  void ensure_global(int b) {
    b = canon(b);
    Val& v = V[b];
    if (v.ctx == X_GLOBAL) return;
    if (v.ctx == X_CONST) {
      if (!v.need_store) fills.push_back(b);
      v.need_store = true;
      return;
    }
    v.need_store = true;
  }

  int canon(int b) const {
    while (V[b].base >= 0 && !V[b].tbl && V[b].ctx != X_GLOBAL && V[b].ctx != X_CONST) b = V[b].base;
    return b;
  }

  // storage root of a materialised value
  std::pair<int, int64_t> storage(int b) const {
    b = canon(b);
    const Val& v = V[b];
    if (v.ctx == X_GLOBAL) return {v.root, v.off};
    return {b, 0};
  }

  void eager(int ci) {
    const TCall& c = t.calls[ci];
    for (int b : c.ins) ensure_global(tsrc[(size_t)b] >= 0 ? tsrc[(size_t)b] : b);
    cur = -1;
    Step s;
    s.kind = S_EAGER;
    s.call = ci;
    steps.push_back(s);
    Val& o = V[c.out];
    o = Val();
    o.ctx = X_GLOBAL;
    o.root = c.out;
    o.off = 0;
  }

  bool plan() {
    for (int b : t.inputs) {
      V[b].ctx = X_GLOBAL;
      V[b].root = b;
    }
    // calls whose results reach no output are dropped (a gradient's backward also produces
    // the cotangents of constants, which nothing reads)
    std::vector<char> live(t.shape.size(), 0);
    for (int b : t.outputs) live[(size_t)b] = 1;
    for (int ci = (int)t.calls.size() - 1; ci >= 0; --ci) {
      const TCall& c = t.calls[(size_t)ci];
      if (!live[(size_t)c.out]) continue;
      for (int b : c.ins) live[(size_t)b] = 1;
    }
    // transposes read only by matmuls (as either operand) and not outputs are absorbed
    {
      std::vector<int> uses(t.shape.size(), 0), mm_uses(t.shape.size(), 0);
      for (const TCall& c : t.calls) {
        if (!live[(size_t)c.out]) continue;
        for (int b : c.ins) {
          uses[(size_t)b]++;
          if (c.op == T_MATMUL) mm_uses[(size_t)b]++;
        }
      }
      std::vector<char> is_out(t.shape.size(), 0);
      for (int b : t.outputs) is_out[(size_t)b] = 1;
      for (const TCall& c : t.calls)
        if (c.op == T_TRANSPOSE && live[(size_t)c.out] && !is_out[(size_t)c.out] && uses[(size_t)c.out] > 0 &&
            uses[(size_t)c.out] == mm_uses[(size_t)c.out])
          tsrc[(size_t)c.out] = c.ins[0];
    }
    for (int ci = 0; ci < (int)t.calls.size(); ++ci) {
      const TCall& c = t.calls[ci];
      if (!live[(size_t)c.out]) continue;
      if (tsrc[(size_t)c.out] >= 0) continue;  // absorbed transpose: its matmul reads the source
      if (c.op == T_RESHAPE) {
        V[c.out] = V[c.ins[0]];
        // a reshape of a stored value shares its storage; of a kernel value, its slots
        if (V[c.out].ctx == X_ROW || V[c.out].ctx == X_SHARED || V[c.out].ctx == X_POST) {
          if (V[c.out].base < 0) {
            // alias: view with identity table over the same value
            Val a = V[c.ins[0]];
            a.base = c.ins[0];
            a.base_rows = a.ctx == X_ROW;
            a.tbl = nullptr;
            a.need_store = false;
            V[c.out] = a;
          }
        }
        continue;
      }
      if (c.op == T_FULL) {
        Val v;
        v.ctx = X_CONST;
        double d;
        std::memcpy(&d, &c.at[0], 8);
        v.cval = (float)d;
        V[c.out] = v;
        continue;
      }
      if (c.op == T_SLICE0) {
        int b = c.ins[0];
        ensure_global(b);
        auto st = storage(b);
        Val v;
        v.ctx = X_GLOBAL;
        v.root = st.first;
        v.off = st.second + c.at[0] * t.size[c.out];
        V[c.out] = v;
        continue;
      }
      bool placed = false;
      Val out;
      GCall gc;
      int64_t newR;
      if (cur >= 0 && classify(ci, cur, out, gc, newR)) {
        commit(ci, cur, out, gc, newR);
        placed = true;
      } else {
        groups.push_back(Group());
        int g = (int)groups.size() - 1;
        if (classify(ci, g, out, gc, newR)) {
          cur = g;
          Step s;
          s.kind = S_GROUP;
          s.group = g;
          steps.push_back(s);
          commit(ci, g, out, gc, newR);
          placed = true;
        } else {
          groups.pop_back();
        }
      }
      if (!placed) eager(ci);
    }
    // outputs
    for (size_t k = 0; k < t.outputs.size(); ++k) ensure_global(t.outputs[k]);
    return true;
  }
};

// ---------------------------------------------------------------------------------------------
// NVRTC
// ---------------------------------------------------------------------------------------------

const char* kPrelude = R"PRELUDE(
typedef unsigned long long u64;
#define J4B_INF __int_as_float(0x7f800000)
__device__ __forceinline__ float jmax(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == 0.0f && b == 0.0f) return signbit(a) ? b : a;
  return a >= b ? a : b;
}
__device__ __forceinline__ float jmin(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == 0.0f && b == 0.0f) return signbit(a) ? a : b;
  return a <= b ? a : b;
}
__device__ __forceinline__ float jsign(float x) { return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f); }
// exp and sigmoid use the fast exponential (ex2.approx: a few ulp, far inside the engine's
// fp32 tolerance against the reference's double-evaluated transcendentals). rsqrt stays the
// correctly rounded reciprocal of the correctly rounded root: rsqrtf measured 40% slower on the
// RMSNorm gradient tape (62 -> 88 us), although it executes fewer instructions.
__device__ __forceinline__ float jexp(float x) { return __expf(x); }
__device__ __forceinline__ float jsigmoid(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
__device__ __forceinline__ float jrsqrt(float x) { return __frcp_rn(__fsqrt_rn(x)); }
// first-NaN, else first-maximum (argMaxAxis / maxAxisBackward, CpuBackend.java:331-391)
__device__ __forceinline__ void amax_combine(float& v, long long& i, float v2, long long i2) {
  bool n1 = v != v, n2 = v2 != v2;
  bool take;
  if (n1 || n2) take = n2 && (!n1 || i2 < i);
  else take = v2 > v || (v2 == v && i2 < i);
  if (take) { v = v2; i = i2; }
}
// reduceMax: strict '>' from -inf, NaN skipped, first of equal values (CpuBackend.java:274-284)
__device__ __forceinline__ void rmax_combine(float& v, long long& i, float v2, long long i2) {
  if (v2 != v2) return;
  if (v2 > v || (v2 == v && i2 < i)) { v = v2; i = i2; }
}
// Block reductions, identical in every thread: butterfly within warps, then each warp combines
// the per-warp values (same order in every warp). Consecutive reductions alternate between the two
// halves of `red` (rp counts the reductions a thread has made; every thread makes the same ones),
// so one barrier per reduction suffices: a warp writes half h again only after the barrier of the
// next reduction, which every warp reaches after its reads of half h.
template <int NT> __device__ __forceinline__ double block_sum(double v, double* red, int& rp) {
  double* r = red + (rp++ & 1) * (2 * (NT / 32));
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) r[threadIdx.x >> 5] = v;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  double tot = lane < NT / 32 ? r[lane] : 0.0;
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
  return tot;
}
// Row sums: the same in float, and the per-warp values summed by every thread straight from
// shared memory in warp order (broadcast vector loads instead of a second shuffle butterfly: a
// short dependent chain, since every row waits on its reductions). The partials are per-thread
// float sums of at most a few dozen elements, so float here stays far inside the fp32 tolerance
// of the reference's double accumulator.
template <int NT> __device__ __forceinline__ float block_sumf(float v, double* red, int& rp) {
  float* r = reinterpret_cast<float*>(red + (rp++ & 1) * (2 * (NT / 32)));
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) r[threadIdx.x >> 5] = v;
  __syncthreads();
  float tot = 0.0f;
  if constexpr (NT / 32 >= 4) {
    #pragma unroll
    for (int w = 0; w < NT / 32; w += 4) {
      const float4 p = *reinterpret_cast<const float4*>(r + w);
      tot += (p.x + p.y) + (p.z + p.w);
    }
  } else {
    #pragma unroll
    for (int w = 0; w < NT / 32; ++w) tot += r[w];
  }
  return tot;
}
template <int NT> __device__ __forceinline__ float block_jmax(float v, double* red, int& rp) {
  double* r = red + (rp++ & 1) * (2 * (NT / 32));
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = jmax(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) r[threadIdx.x >> 5] = (double)v;
  __syncthreads();
  float tot = -J4B_INF;
  #pragma unroll
  for (int w = 0; w < NT / 32; ++w) tot = jmax(tot, (float)r[w]);
  return tot;
}
template <int NT, int MODE> __device__ __forceinline__ long long block_pair(float& v, long long i, double* red, int& rp) {
  double* r = red + (rp++ & 1) * (2 * (NT / 32));
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float v2 = __shfl_xor_sync(0xffffffffu, v, o);
    long long i2 = __shfl_xor_sync(0xffffffffu, i, o);
    if (MODE == 0) amax_combine(v, i, v2, i2); else rmax_combine(v, i, v2, i2);
  }
  if ((threadIdx.x & 31) == 0) {
    r[2 * (threadIdx.x >> 5)] = (double)v;
    r[2 * (threadIdx.x >> 5) + 1] = (double)i;
  }
  __syncthreads();
  float bv = (float)r[0];
  long long bi = (long long)r[1];
  #pragma unroll
  for (int w = 1; w < NT / 32; ++w) {
    if (MODE == 0) amax_combine(bv, bi, (float)r[2 * w], (long long)r[2 * w + 1]);
    else rmax_combine(bv, bi, (float)r[2 * w], (long long)r[2 * w + 1]);
  }
  v = bv;
  return bi;
}
)PRELUDE";

// ---------------------------------------------------------------------------------------------
// code generation for one group
// ---------------------------------------------------------------------------------------------

// Where a kernel pointer parameter points at launch.
struct PtrRef {
  int kind = 0;   // 1 input k, 2 output k, 3 arena byte offset, 4 constant table blob offset
  int index = -1;
  int64_t bytes = 0;
};

std::string fstr(float v) {
  if (std::isnan(v)) return "__int_as_float(0x7fc00000)";
  if (std::isinf(v)) return v > 0 ? "J4B_INF" : "(-J4B_INF)";
  uint32_t bits;
  std::memcpy(&bits, &v, 4);
  char b[64];
  snprintf(b, sizeof b, "__int_as_float(0x%08x)", bits);
  return b;
}

std::string istr(int64_t v) { return std::to_string(v) + "LL"; }

struct GroupCode {
  std::string src, row_name, fold_name;
  int NT = 32;
  size_t smem = 0;
  bool fold = false;
  int64_t fold_len = 1;
  std::vector<int> ptr_values;          // value id per pointer slot (kind from Val)
  std::vector<std::pair<int, int64_t>> partials;  // per partial slot: (value, doubles per CTA)
  std::vector<int> tables;              // ids of table-blob entries
};

struct Gen;  // forward

}  // namespace
}  // namespace j4b

// The compiled tape.
struct j4b_tape {
  int dev = 0;
  j4b::TapeIR ir;
  std::vector<j4b::Val> V;
  std::vector<j4b::Group> groups;
  std::vector<j4b::Step> steps;
  std::vector<int> fills;
  std::vector<int> tsrc;  // absorbed transposes: output id -> source id (else -1)
  struct GroupRun {
    CUmodule mod = nullptr;
    CUfunction row = nullptr, fold = nullptr;
    int NT = 32;
    size_t smem = 0;
    int grid = 1, fold_grid = 1;
    int64_t R = 0;
    std::vector<j4b::PtrRef> ptrs;
    std::string src;
  };
  std::vector<GroupRun> runs;
  // storage of materialised values
  std::vector<j4b::PtrRef> loc;       // per buffer id (root values)
  std::vector<std::vector<int>> maps; // per eager reindex/scatter call: device map offset
  std::vector<int64_t> map_off;       // per call index: byte offset of its int32 map in the arena (-1)
  std::vector<int64_t> tbl_off;       // per table id: byte offset into the table blob
  void* arena = nullptr;
  size_t arena_bytes = 0;
  void* tblob = nullptr;
  size_t tblob_bytes = 0;
  int launches_per_replay = 0;
  std::mutex mu;
};

namespace j4b {
namespace {

struct Gen {
  j4b_tape& T;
  const TapeIR& t;
  std::vector<Val>& V;
  const Group& G;
  int gi;
  int NT = 32;
  std::ostringstream o;       // row kernel body
  std::ostringstream pro;     // prologue
  std::ostringstream fin;     // after the row loop
  std::ostringstream fold;    // fold kernel body
  std::map<int, int> ptr_slot;            // value/root id -> pointer slot
  std::vector<PtrRef>& ptrs;
  std::vector<std::vector<int64_t>>& tables;  // table blob entries (host copies)
  std::map<const std::vector<int64_t>*, int> table_id;  // table -> pointer slot
  std::map<int, size_t> smem_off;         // staged value -> float offset
  size_t smem_floats = 0;
  std::map<int, int> part_slot;           // reduction value -> partial pointer slot
  std::vector<std::pair<int, int64_t>> partials;  // (value, doubles per CTA)
  std::vector<char> row_loaded;           // stored tensors hoisted as row tiles (per value id)
  std::vector<char> staged_now;
  int tmp = 0;
  std::map<std::string, std::string> scalar_cse;  // per-row scalar subexpressions -> temporaries
  const std::ostringstream* scalar_os = nullptr;   // the stream (scope) scalar_cse belongs to

  Gen(j4b_tape& tp, int g, std::vector<PtrRef>& p, std::vector<std::vector<int64_t>>& tb)
      : T(tp), t(tp.ir), V(tp.V), G(tp.groups[g]), gi(g), ptrs(p), tables(tb) {}

  int E(int64_t W) const { return (int)((W + 4LL * NT - 1) / (4LL * NT)); }

  // Bounds test `var + off < lim` of the slot j = (e * NT + t) * 4 + q of a row loop (c4 * 4
  // for the float4 form), with a leading term that is a compile-time constant once e is
  // unrolled: when even thread NT - 1's slots of step e are in range, (e + 1) * 4 NT + off <=
  // lim, the whole test folds to true and no per-element compare is executed.
  std::string jlt(int64_t off, int64_t lim, const char* var = "j") const {
    const std::string o = off ? " + " + istr(off) : "";
    return "((e + 1) * " + istr(4LL * NT) + o + " <= " + istr(lim) + " || " + var + o + " < " + istr(lim) + ")";
  }

  // pointer slot for a materialised value (its storage root + element offset) -> "P<k>" symbol
  int canon(int b) const {
    while (V[b].base >= 0 && !V[b].tbl && V[b].ctx != X_GLOBAL && V[b].ctx != X_CONST) b = V[b].base;
    return b;
  }

  std::string gptr(int b) {
    b = canon(b);
    int root = V[b].ctx == X_GLOBAL ? V[b].root : b;
    int64_t off = V[b].ctx == X_GLOBAL ? V[b].off : 0;
    int key = root;
    auto it = ptr_slot.find(key);
    int slot;
    if (it == ptr_slot.end()) {
      slot = (int)ptrs.size();
      PtrRef pr;
      pr.kind = 10;  // resolved later from the root's storage
      pr.index = root;
      ptrs.push_back(pr);
      ptr_slot[key] = slot;
    } else {
      slot = it->second;
    }
    std::string s = "((float*)A.p[" + std::to_string(slot) + "])";
    if (off) s = "(" + s + " + " + istr(off) + ")";
    return s;
  }

  std::string tptr(const Table& tb) {
    auto it = table_id.find(tb.get());
    int slot;
    if (it == table_id.end()) {
      tables.push_back(*tb);
      slot = (int)ptrs.size();
      PtrRef pr;
      pr.kind = 4;
      pr.index = (int)tables.size() - 1;
      ptrs.push_back(pr);
      table_id[tb.get()] = slot;
    } else {
      slot = it->second;
    }
    return "((const long long*)A.p[" + std::to_string(slot) + "])";
  }

  std::string vname(int b) const { return "v" + std::to_string(b); }

  // Is value b (non-view, computed in this group) held in slots / uniform?

  // ---- table classification ----
  enum { TB_ID = 0, TB_SHIFT, TB_CONST, TB_GEN };
  int tclass(const Table& tb, int64_t Wb, int64_t* param) const {
    if (!tb) return TB_ID;
    const auto& v = *tb;
    int64_t W = (int64_t)v.size();
    bool all_const = W > 0 && v[0] >= 0;
    for (int64_t j = 1; all_const && j < W; ++j) all_const = v[(size_t)j] == v[0];
    if (all_const) { *param = v[0]; return TB_CONST; }
    // shift: v[j] = j + S where 0 <= j + S < Wb, else -1
    int64_t S = 0;
    bool found = false;
    for (int64_t j = 0; j < W; ++j)
      if (v[(size_t)j] >= 0) { S = v[(size_t)j] - j; found = true; break; }
    if (!found) { *param = -1; return TB_CONST; }  // all -1: zeros
    for (int64_t j = 0; j < W; ++j) {
      int64_t want = (j + S >= 0 && j + S < Wb) ? j + S : -1;
      if (v[(size_t)j] != want) return TB_GEN;
    }
    *param = S;
    if (S == 0 && W == Wb) return TB_ID;
    return TB_SHIFT;
  }

  // width of a base value as indexed by a table (its row width or vector length)
  int64_t base_width(int base, bool rows) const {
    if (rows) return V[base].ctx == X_GLOBAL ? t.size[base] / G.R : V[base].W;
    return V[base].ctx == X_GLOBAL ? t.size[base] : V[base].W;
  }

  // The context code is being generated for: row (inside the row loop, row r) or shared.
  bool rowctx = false;

  // A value's base and table as seen from the current context: non-view values read
  // themselves; in the row context a value that is not local to the group is row r of its
  // storage, in the shared context its whole storage.
  struct Access {
    int base;
    bool rows;
    int k;
    int64_t param;
    int64_t Wb;
    bool local;
  };

  bool is_local(int b) const {
    const Val& v = V[b];
    return v.ctx != X_GLOBAL && v.ctx != X_CONST && v.kernel == gi;
  }

  Access access(int b) const {
    const Val& v = V[b];
    Access a;
    if (v.base >= 0) {
      a.base = v.base;
      a.rows = v.base_rows;
      a.Wb = base_width(a.base, a.rows);
      a.param = 0;
      a.k = tclass(v.tbl, a.Wb, &a.param);
    } else {
      a.base = b;
      a.rows = is_local(b) ? v.ctx == X_ROW : rowctx;
      a.Wb = base_width(b, a.rows);
      a.param = 0;
      a.k = TB_ID;
    }
    a.local = is_local(a.base);
    return a;
  }

  // C expression for element `x` (any index expression) of value b in the current context.
  // Collects local bases that must be staged in shared memory.
  std::string elem(int b, const std::string& x, std::vector<int>& need) {
    const Val& v = V[b];
    if (v.ctx == X_CONST) return fstr(v.cval);
    Access a = access(b);
    if (V[a.base].ctx == X_CONST) return fstr(V[a.base].cval);
    if (a.k == TB_CONST) {
      if (a.param < 0) return "0.0f";
      return elem_base(a.base, a.rows, istr(a.param), need);
    }
    if (a.k == TB_ID) return elem_base(a.base, a.rows, x, need);
    if (a.k == TB_SHIFT) {
      std::string ix = "(" + x + " + " + istr(a.param) + ")";
      return "((" + ix + " >= 0 && " + ix + " < " + istr(a.Wb) + ") ? " +
             elem_base(a.base, a.rows, ix, need) + " : 0.0f)";
    }
    std::string tb = tptr(v.tbl);
    std::string nm = "ix" + std::to_string(tmp++);
    return "([&]{ const long long " + nm + " = __ldg(" + tb + " + (" + x + ")); return " + nm +
           " >= 0 ? " + elem_base(a.base, a.rows, nm, need) + " : 0.0f; }())";
  }

  std::string elem_base(int b, bool rows, const std::string& x, std::vector<int>& need) {
    const Val& v = V[b];
    if (v.ctx == X_CONST) return fstr(v.cval);
    if (!is_local(b)) {
      std::string p = gptr(b);
      if (rows) return "__ldg(" + p + " + r * " + istr(t.size[b] / G.R) + " + (" + x + "))";
      return "__ldg(" + p + " + (" + x + "))";
    }
    if (v.W == 1) return vname(b);
    need.push_back(b);
    return "sm[" + istr((int64_t)smem_of(b)) + " + (" + x + ")]";
  }

  size_t smem_of(int b) {
    auto it = smem_off.find(b);
    if (it != smem_off.end()) return it->second;
    size_t off = smem_floats;
    smem_floats += (size_t)((V[b].W + 3) / 4 * 4);
    smem_off[b] = off;
    return off;
  }

  std::vector<int> row_loads, shared_loads;   // global bases hoisted into registers
  std::vector<char> shared_loaded;

  // C expression for slot (e, q) (element j) of value b in a context of width W.
  std::string slot(int b, int64_t W, std::vector<int>& need) {
    const Val& v = V[b];
    if (v.ctx == X_CONST) return fstr(v.cval);
    Access a = access(b);
    const Val& bv = V[a.base];
    if (bv.ctx == X_CONST) return fstr(bv.cval);
    if (a.k == TB_CONST && a.param < 0) return "0.0f";
    if (a.local) {
      if (bv.W == 1 && (a.k == TB_ID || a.k == TB_CONST)) return vname(a.base);
      if (a.k == TB_ID && a.Wb == W) return vname(a.base) + "[e * 4 + q]";
      if (a.k == TB_SHIFT && a.param % (4LL * NT) == 0 && bv.W > 1) {  // width-1 bases are scalars
        int64_t se = a.param / (4LL * NT);
        std::string es = "(e + " + std::to_string(se) + ")";
        std::string eb = std::to_string(E(a.Wb));
        return "((" + es + " >= 0 && " + es + " < " + eb + " && " + jlt(a.param, a.Wb) +
               ") ? " + vname(a.base) + "[(" + es + " < 0 ? 0 : (" + es + " >= " + eb + " ? 0 : " + es +
               ")) * 4 + q] : 0.0f)";
      }
    } else if (a.k == TB_ID && a.Wb == W && W > 1) {
      // identity read of a stored tensor: hoisted into registers (per row, or once per CTA)
      if (a.rows && rowctx) {
        if (!row_loaded[a.base]) { row_loaded[a.base] = 1; row_loads.push_back(a.base); }
        return "L" + std::to_string(a.base) + "[e * 4 + q]";
      }
      if (!a.rows && W <= kSharedMax) {
        if (!shared_loaded[a.base]) { shared_loaded[a.base] = 1; shared_loads.push_back(a.base); }
        return "S" + std::to_string(a.base) + "[e * 4 + q]";
      }
    }
    return elem(b, "j", need);
  }

  void emit_load(std::ostringstream& os, int b, bool rows, const char* prefix = nullptr,
                 const std::string& rowexpr = "r", bool declare = true) {
    int64_t W = rows ? t.size[b] / G.R : t.size[b];
    std::string p = gptr(b);
    std::string nm = (prefix ? std::string(prefix) : std::string(rows ? "L" : "S")) + std::to_string(b);
    std::string rowoff = rows ? " + " + rowexpr + " * " + istr(W) : "";
    int64_t off = V[b].ctx == X_GLOBAL ? V[b].off : 0;
    bool vec = W % 4 == 0 && off % 4 == 0;
    if (declare) os << "  float " << nm << "[" << E(W) * 4 << "];\n";
    if (vec) {
      os << "  #pragma unroll\n  for (int e = 0; e < " << E(W) << "; ++e) {\n"
         << "    const long long c4 = (long long)e * " << NT << " + t;\n"
         << "    float4 x4 = make_float4(0.f, 0.f, 0.f, 0.f);\n"
         << "    if (" << jlt(0, W, "c4 * 4") << ") x4 = __ldg(reinterpret_cast<const float4*>(" << p << rowoff
         << ") + c4);\n"
         << "    " << nm << "[e * 4] = x4.x; " << nm << "[e * 4 + 1] = x4.y; " << nm << "[e * 4 + 2] = x4.z; "
         << nm << "[e * 4 + 3] = x4.w;\n  }\n";
    } else {
      os << "  #pragma unroll\n  for (int e = 0; e < " << E(W) << "; ++e) {\n"
         << "    #pragma unroll\n    for (int q = 0; q < 4; ++q) {\n"
         << "      const long long j = ((long long)e * " << NT << " + t) * 4 + q;\n"
         << "      " << nm << "[e * 4 + q] = " << jlt(0, W) << " ? __ldg(" << p << rowoff
         << " + j) : 0.0f;\n    }\n  }\n";
    }
  }

  void stage(std::ostringstream& os, int b) {
    // writes the slots of b into its shared-memory region
    size_t off = smem_of(b);
    os << "  #pragma unroll\n  for (int e = 0; e < " << E(V[b].W) << "; ++e) {\n"
       << "    #pragma unroll\n    for (int q = 0; q < 4; ++q) {\n"
       << "      const long long j = ((long long)e * " << NT << " + t) * 4 + q;\n"
       << "      if (" << jlt(0, V[b].W) << ") sm[" << off << " + j] = " << vname(b) << "[e * 4 + q];\n"
       << "    }\n  }\n  __syncthreads();\n";
  }

  void ensure_staged(std::ostringstream& os, std::vector<int>& need) {
    for (int b : need) {
      if (staged_now[b]) continue;
      staged_now[b] = 1;
      stage(os, b);
    }
    need.clear();
  }

  // expression code for a fused program / binary / scalar / unary / reluBackward, elementwise;
  // `acc(i)` gives the C expression of input i at the current element.
  std::string expr_code(const TCall& c, const std::vector<std::string>& in, std::ostringstream& os,
                        const std::string& ind, std::map<std::string, std::string>* cse = nullptr) {
    auto un = [](int op, const std::string& a) -> std::string {
      switch (op) {
        case J4B_NEG: return "(-" + a + ")";
        case J4B_EXP: return "jexp(" + a + ")";
        case J4B_LOG: return "logf(" + a + ")";
        case J4B_SQRT: return "__fsqrt_rn(" + a + ")";
        case J4B_RSQRT: return "jrsqrt(" + a + ")";
        case J4B_TANH: return "tanhf(" + a + ")";
        case J4B_SIGMOID: return "jsigmoid(" + a + ")";
        case J4B_RELU: return "jmax(0.0f, " + a + ")";
        case J4B_ABS: return "fabsf(" + a + ")";
        case J4B_SIGN: return "jsign(" + a + ")";
      }
      return "0.0f";
    };
    // x / c for a power-of-two constant c is x * (1/c) exactly (one rounding of the same value)
    auto scal = [](int op, double d) -> std::string {
      float fv = (float)d;
      int ex = 0;
      if (op == J4B_DIV && std::isfinite(fv) && fv != 0.0f && std::fabs(std::frexp(fv, &ex)) == 0.5f &&
          ex > -120 && ex < 120)
        return "*" + fstr(1.0f / fv);
      return fstr(fv);
    };
    // + - * are plain IEEE operations that the compiler may contract into fused multiply-adds
    // (one rounding instead of two: within the fp32 tolerance of the reference's separately
    // rounded float ops, and ~a quarter fewer instructions in gradient tapes)
    auto bin = [](int op, const std::string& a, const std::string& b) -> std::string {
      if (!b.empty() && b[0] == '*') return "(" + a + " * " + b.substr(1) + ")";
      // 1 / x is the correctly rounded reciprocal: identical to the IEEE division
      if (op == J4B_DIV && a == fstr(1.0f)) return "__frcp_rn(" + b + ")";
      switch (op) {
        case J4B_ADD: return "(" + a + " + " + b + ")";
        case J4B_SUB: return "(" + a + " - " + b + ")";
        case J4B_MUL: return "(" + a + " * " + b + ")";
        case J4B_DIV: return "__fdiv_rn(" + a + ", " + b + ")";
        case J4B_MAX: return "jmax(" + a + ", " + b + ")";
        case J4B_MIN: return "jmin(" + a + ", " + b + ")";
      }
      return "0.0f";
    };
    switch (c.op) {
      case T_BINARY: return bin((int)c.at[0], in[0], in[1]);
      case T_SCALAR: {
        double d;
        std::memcpy(&d, &c.at[1], 8);
        return bin((int)c.at[0], in[0], scal((int)c.at[0], d));
      }
      case T_UNARY: return un((int)c.at[0], in[0]);
      case T_RELUBWD: return "(" + in[1] + " > 0.0f ? " + in[0] + " : 0.0f)";
      default: break;
    }
    std::vector<ENode> nodes;
    int root = 0;
    std::string e2;
    parse_program(c.at, (int)c.ins.size(), nodes, &root, e2);
    std::vector<std::string> nm(nodes.size());
    int base = tmp;
    tmp += (int)nodes.size();
    for (size_t i = 0; i < nodes.size(); ++i) {
      const ENode& n = nodes[i];
      std::string rhs;
      if (n.kind == 0) rhs = in[(size_t)n.idx];
      else if (n.kind == 1) rhs = un(n.op, nm[(size_t)n.a]);
      else if (n.kind == 2) rhs = bin(n.op, nm[(size_t)n.a], nm[(size_t)n.b]);
      else rhs = bin(n.op, nm[(size_t)n.a], scal(n.op, n.val));
      if (cse) {
        auto it = cse->find(rhs);
        if (it != cse->end()) {
          nm[i] = it->second;
          continue;
        }
      }
      nm[i] = "x" + std::to_string(base + (int)i);
      os << ind << "const float " << nm[i] << " = " << rhs << ";\n";
      if (cse) (*cse)[rhs] = nm[i];
    }
    return nm[(size_t)root];
  }

  // ---- stores ----
  void store_row(std::ostringstream& os, int b) {
    // stores row r of value b (slots, uniform or view) to its storage
    const Val& v = V[b];
    std::string p = gptr(b);
    int64_t W = v.W;
    std::vector<int> need;
    if (W == 1 && v.base < 0) {
      os << "  if (t == 0) " << p << "[r] = " << vname(b) << ";\n";
      return;
    }
    // element expressions first (may need staging)
    std::ostringstream body;
    std::string val = slot(b, W, need);
    ensure_staged(os, need);
    bool vec = W % 4 == 0 && v.base < 0;
    if (vec) {
      os << "  #pragma unroll\n  for (int e = 0; e < " << E(W) << "; ++e) {\n"
         << "    const long long c4 = (long long)e * " << NT << " + t;\n"
         << "    if (" << jlt(0, W, "c4 * 4") << ") reinterpret_cast<float4*>(" << p << " + r * " << istr(W)
         << ")[c4] = make_float4(" << vname(b) << "[e * 4], " << vname(b) << "[e * 4 + 1], " << vname(b)
         << "[e * 4 + 2], " << vname(b) << "[e * 4 + 3]);\n  }\n";
      return;
    }
    os << "  #pragma unroll\n  for (int e = 0; e < " << E(W) << "; ++e) {\n"
       << "    #pragma unroll\n    for (int q = 0; q < 4; ++q) {\n"
       << "      const long long j = ((long long)e * " << NT << " + t) * 4 + q;\n"
       << "      if (" << jlt(0, W) << ") " << p << "[r * " << istr(W) << " + j] = " << val << ";\n"
       << "    }\n  }\n";
  }

  void store_shared(std::ostringstream& os, int b) {
    const Val& v = V[b];
    std::string p = gptr(b);
    std::vector<int> need;
    if (v.W == 1 && v.base < 0) {
      os << "  if (blockIdx.x == 0 && t == 0) " << p << "[0] = " << vname(b) << ";\n";
      return;
    }
    std::string val = slot(b, v.W, need);
    ensure_staged(os, need);
    os << "  if (blockIdx.x == 0) {\n  #pragma unroll\n  for (int e = 0; e < " << E(v.W) << "; ++e) {\n"
       << "    #pragma unroll\n    for (int q = 0; q < 4; ++q) {\n"
       << "      const long long j = ((long long)e * " << NT << " + t) * 4 + q;\n"
       << "      if (" << jlt(0, v.W) << ") " << p << "[j] = " << val << ";\n"
       << "    }\n  }\n  }\n";
  }

  // ---- one call in the row / shared context ----
  // Consecutive elementwise calls of one width share one slot loop, with common
  // subexpressions computed once (the fused calls of a gradient repeat their forward parts).
  std::vector<GCall> batch;
  int64_t batch_W = 0;
  bool batch_row = false;
  std::ostringstream* batch_os = nullptr;

  bool reads_batch_view(const TCall& c) const {
    for (int x : c.ins) {
      if (V[x].base < 0) continue;
      for (const GCall& m : batch)
        if (t.calls[(size_t)m.call].out == V[x].base && V[x].tbl) return true;
    }
    return false;
  }

  void flush() {
    if (batch.empty()) return;
    std::ostringstream& os = *batch_os;
    rowctx = batch_row;
    const int64_t W = batch_W;
    std::vector<int> need;
    std::ostringstream body;
    std::map<std::string, std::string> cse;
    for (const GCall& m : batch) {
      const TCall& c = t.calls[(size_t)m.call];
      if (m.kind == G_COLRED || m.kind == G_GLOBRED) {
        // per-thread accumulation of a cross-row reduction, folded after the row loop
        std::string val = slot(c.ins[0], W, need);
        auto it = cse.find(val);
        if (it != cse.end()) val = it->second;
        const int b = c.out;
        if (m.kind == G_COLRED) {
          if (c.op == T_MAXAX) body << "      cm" << b << "[e * 4 + q] = jmax(cm" << b << "[e * 4 + q], " << val << ");\n";
          else body << "      ca" << b << "[e * 4 + q] += " << val << ";\n";
        } else {
          if (c.op == T_RMAX) body << "      rmax_combine(gm" << b << ", gi" << b << ", " << val << ", r * " << istr(W) << " + j);\n";
          else body << "      gr" << b << " += " << val << ";\n";
        }
        continue;
      }
      std::vector<std::string> in;
      for (int x : c.ins) in.push_back(slot(x, W, need));
      std::string r = expr_code(c, in, body, "      ", &cse);
      auto it = cse.find(r);
      std::string nm;
      if (it != cse.end()) {
        nm = it->second;
      } else {
        nm = "x" + std::to_string(tmp++);
        body << "      const float " << nm << " = " << r << ";\n";
        cse[r] = nm;
      }
      body << "      " << vname(c.out) << "[e * 4 + q] = " << nm << ";\n";
    }
    ensure_staged(os, need);
    const bool full = W % (4LL * NT) == 0;
    for (const GCall& m : batch) {
      const TCall& c = t.calls[(size_t)m.call];
      if (m.kind == G_EXPR) os << "  float " << vname(c.out) << "[" << E(W) * 4 << "];\n";
      if (m.kind == G_GLOBRED && c.op != T_RMAX) os << "  float gr" << c.out << " = 0.0f;\n";
    }
    os << "  #pragma unroll\n  for (int e = 0; e < " << E(W) << "; ++e) {\n"
       << "    #pragma unroll\n    for (int q = 0; q < 4; ++q) {\n"
       << "      const long long j = ((long long)e * " << NT << " + t) * 4 + q;\n      (void)j;\n";
    if (full) {
      os << body.str();
    } else {
      os << "      if (" << jlt(0, W) << ") {\n" << body.str() << "      } else {\n";
      for (const GCall& m : batch)
        if (m.kind == G_EXPR) os << "        " << vname(t.calls[(size_t)m.call].out) << "[e * 4 + q] = 0.0f;\n";
      os << "      }\n";
    }
    os << "    }\n  }\n";
    // a row's share of a global sum is added in double once per row and thread
    for (const GCall& m : batch) {
      const TCall& c = t.calls[(size_t)m.call];
      if (m.kind == G_GLOBRED && c.op != T_RMAX) os << "  ga" << c.out << " += (double)gr" << c.out << ";\n";
    }
    std::vector<GCall> done;
    done.swap(batch);
    for (const GCall& m : done) {
      int b = t.calls[(size_t)m.call].out;
      if (m.kind == G_EXPR && V[b].need_store) (batch_row ? store_row(os, b) : store_shared(os, b));
    }
  }

  void emit_rowlike(std::ostringstream& os, const GCall& gc) {
    const TCall& c = t.calls[(size_t)gc.call];
    const int b = c.out;
    Val& v = V[b];
    // cross-row reductions accumulate inside the row loop; their results live in the fold
    const bool row = gc.ctx == X_ROW || gc.kind == G_COLRED || gc.kind == G_GLOBRED;
    if (gc.kind == G_VIEW && !v.need_store) return;  // views emit no code of their own
    const bool cross = (gc.kind == G_COLRED || gc.kind == G_GLOBRED) && row;
    const int64_t bw = gc.kind == G_EXPR ? v.W : (cross ? t.size[c.ins[0]] / G.R : 0);
    if ((gc.kind == G_EXPR && v.W > 1) || (cross && bw > 1)) {
      if (!batch.empty() && (batch_W != bw || batch_row != row || batch_os != &os || reads_batch_view(c)))
        flush();
      batch.push_back(gc);
      batch_W = bw;
      batch_row = row;
      batch_os = &os;
      return;
    }
    flush();
    rowctx = row;
    if (gc.kind == G_VIEW) {
      if (v.need_store) (row ? store_row(os, b) : store_shared(os, b));
      return;
    }
    std::vector<int> need;
    if (gc.kind == G_EXPR) {
      if (v.W == 1) {
        std::vector<std::string> in;
        for (int x : c.ins) in.push_back(slot_uniform(x, need));
        ensure_staged(os, need);
        // per-row scalars share subexpressions across calls (a gradient recomputes its forward's
        // scalars, e.g. the rsqrt of a mean square): temporaries live at the scope of the stream
        // they are emitted into (kernel prologue or row body), so the table is reset per stream
        if (&os != scalar_os) {
          scalar_cse.clear();
          scalar_os = &os;
        }
        std::ostringstream body;
        std::string r = expr_code(c, in, body, "  ", &scalar_cse);
        os << body.str() << "  float " << vname(b) << " = " << r << ";\n";
      } else {
        std::vector<std::string> in;
        for (int x : c.ins) in.push_back(slot(x, v.W, need));
        ensure_staged(os, need);
        std::ostringstream body;
        std::string r = expr_code(c, in, body, "      ");
        os << "  float " << vname(b) << "[" << E(v.W) * 4 << "];\n"
           << "  #pragma unroll\n  for (int e = 0; e < " << E(v.W) << "; ++e) {\n"
           << "    #pragma unroll\n    for (int q = 0; q < 4; ++q) {\n"
           << "      const long long j = ((long long)e * " << NT << " + t) * 4 + q;\n"
           << "      float res = 0.0f;\n"
           << "      if (" << jlt(0, v.W) << ") {\n" << body.str() << "      res = " << r << ";\n      }\n"
           << "      " << vname(b) << "[e * 4 + q] = res;\n    }\n  }\n";
      }
      if (v.need_store) (row ? store_row(os, b) : store_shared(os, b));
      return;
    }
    if (gc.kind == G_RRED) {
      emit_rred(os, gc, row);
      if (v.need_store) (row ? store_row(os, b) : store_shared(os, b));
      return;
    }
    if (gc.kind == G_COLRED) {
      int src = c.ins[0];
      int64_t W = V[b].W;
      std::string val = slot(src, W, need);
      ensure_staged(os, need);
      bool mx = c.op == T_MAXAX;
      os << "  #pragma unroll\n  for (int e = 0; e < " << E(W) << "; ++e) {\n"
         << "    #pragma unroll\n    for (int q = 0; q < 4; ++q) {\n"
         << "      const long long j = ((long long)e * " << NT << " + t) * 4 + q;\n"
         << "      if (" << jlt(0, W) << ") ";
      if (mx) os << "cm" << b << "[e * 4 + q] = jmax(cm" << b << "[e * 4 + q], " << val << ");\n";
      else os << "ca" << b << "[e * 4 + q] += " << val << ";\n";
      os << "    }\n  }\n";
      return;
    }
    if (gc.kind == G_GLOBRED) {
      int src = c.ins[0];
      int64_t W = t.size[src] / G.R;
      std::string val = slot(src, W, need);
      ensure_staged(os, need);
      bool mx = c.op == T_RMAX;
      os << "  #pragma unroll\n  for (int e = 0; e < " << E(W) << "; ++e) {\n"
         << "    #pragma unroll\n    for (int q = 0; q < 4; ++q) {\n"
         << "      const long long j = ((long long)e * " << NT << " + t) * 4 + q;\n"
         << "      if (" << jlt(0, W) << ") ";
      if (mx) os << "rmax_combine(gm" << b << ", gi" << b << ", " << val << ", r * " << istr(W) << " + j);\n";
      else os << "ga" << b << " += (double)" << val << ";\n";
      os << "    }\n  }\n";
      return;
    }
  }

  // uniform (W == 1) operand in a uniform expression
  std::string slot_uniform(int x, std::vector<int>& need) {
    const Val& v = V[x];
    if (v.ctx == X_CONST) return fstr(v.cval);
    return elem(x, "0", need);
  }

  void emit_rred(std::ostringstream& os, const GCall& gc, bool row) {
    const TCall& c = t.calls[(size_t)gc.call];
    const int b = c.out;
    const int src = c.op == T_MAXBWD ? c.ins[1] : c.ins[0];
    const int64_t Win = row ? t.size[src] / G.R : t.size[src];
    const int64_t nn = gc.n, inner = gc.inner;
    std::vector<int> need;
    const bool full = (nn * inner == Win) && inner == 1;  // one output per row / vector
    if (full && c.op != T_MAXBWD) {
      std::string val = slot(src, Win, need);
      ensure_staged(os, need);
      std::string loop = "  #pragma unroll\n  for (int e = 0; e < " + std::to_string(E(Win)) +
                         "; ++e) {\n    #pragma unroll\n    for (int q = 0; q < 4; ++q) {\n"
                         "      const long long j = ((long long)e * " + std::to_string(NT) +
                         " + t) * 4 + q;\n      if (" + jlt(0, Win) + ") ";
      if (c.op == T_SUMAX || c.op == T_RSUM) {
        // per-thread partial in float, combined across threads in float (block_sumf)
        os << "  float " << vname(b) << ";\n  {\n  float acc = 0.0f;\n" << loop << "acc += " << val
           << ";\n    }\n  }\n  " << vname(b) << " = block_sumf<" << NT << ">(acc, red, rp);\n  }\n";
      } else if (c.op == T_MAXAX) {
        os << "  float " << vname(b) << ";\n  {\n  float acc = -J4B_INF;\n" << loop << "acc = jmax(acc, " << val
           << ");\n    }\n  }\n  " << vname(b) << " = block_jmax<" << NT << ">(acc, red, rp);\n  }\n";
      } else if (c.op == T_RMAX) {
        os << "  float " << vname(b) << ";\n  {\n  float bv = -J4B_INF; long long bi = 0x7fffffffffffffffLL;\n"
           << loop << "rmax_combine(bv, bi, " << val << ", j);\n    }\n  }\n"
           << "  block_pair<" << NT << ", 1>(bv, bi, red, rp);\n  " << vname(b) << " = bv;\n  }\n";
      } else {  // argmax
        os << "  float " << vname(b) << ";\n  {\n  float bv = -J4B_INF; long long bi = 0x7fffffffffffffffLL;\n"
           << loop << "amax_combine(bv, bi, " << val << ", j);\n    }\n  }\n"
           << "  long long w = block_pair<" << NT << ", 0>(bv, bi, red, rp);\n  " << vname(b)
           << " = (float)(w == 0x7fffffffffffffffLL ? 0 : w);\n  }\n";
      }
      return;
    }
    if (full && c.op == T_MAXBWD) {
      std::string val = slot(src, Win, need);
      std::string up = slot_uniform(c.ins[0], need);
      ensure_staged(os, need);
      os << "  long long am" << b << ";\n  {\n  float bv = -J4B_INF; long long bi = 0x7fffffffffffffffLL;\n"
         << "  #pragma unroll\n  for (int e = 0; e < " << E(Win) << "; ++e) {\n"
         << "    #pragma unroll\n    for (int q = 0; q < 4; ++q) {\n"
         << "      const long long j = ((long long)e * " << NT << " + t) * 4 + q;\n"
         << "      if (" << jlt(0, Win) << ") amax_combine(bv, bi, " << val << ", j);\n    }\n  }\n"
         << "  am" << b << " = block_pair<" << NT << ", 0>(bv, bi, red, rp);\n"
         << "  if (am" << b << " == 0x7fffffffffffffffLL) am" << b << " = 0;\n  }\n"
         << "  const float up" << b << " = " << up << ";\n"
         << "  float " << vname(b) << "[" << E(Win) * 4 << "];\n"
         << "  #pragma unroll\n  for (int e = 0; e < " << E(Win) << "; ++e) {\n"
         << "    #pragma unroll\n    for (int q = 0; q < 4; ++q) {\n"
         << "      const long long j = ((long long)e * " << NT << " + t) * 4 + q;\n"
         << "      " << vname(b) << "[e * 4 + q] = (j == am" << b << ") ? up" << b << " : 0.0f;\n    }\n  }\n";
      return;
    }
    // partial reduction: sequential per output element over the reduced extent (the
    // reference's own loop order), reading the source through shared memory / global memory
    const int64_t Wo = V[b].W;
    std::string rd_elem = elem(src, "src_ix", need);
    std::string up_elem = c.op == T_MAXBWD ? elem(c.ins[0], "up_ix", need) : "";
    ensure_staged(os, need);
    os << "  float " << vname(b) << "[" << E(Wo) * 4 << "];\n"
       << "  #pragma unroll\n  for (int e = 0; e < " << E(Wo) << "; ++e) {\n"
       << "    #pragma unroll\n    for (int q = 0; q < 4; ++q) {\n"
       << "      const long long j = ((long long)e * " << NT << " + t) * 4 + q;\n"
       << "      float res = 0.0f;\n      if (" << jlt(0, Wo) << ") {\n";
    if (c.op == T_MAXBWD) {
      // j indexes the input; find its group's first maximum
      os << "        const long long o = j / " << istr(nn * inner) << ", in_ = j % " << istr(inner)
         << ", k_ = (j / " << istr(inner) << ") % " << istr(nn) << ";\n"
         << "        float bv = -J4B_INF; long long bi = 0;\n"
         << "        for (long long k = 0; k < " << istr(nn) << "; ++k) {\n"
         << "          const long long src_ix = o * " << istr(nn * inner) << " + k * " << istr(inner) << " + in_;\n"
         << "          const float x = " << rd_elem << ";\n"
         << "          if (x != x || x > bv) { bv = x; bi = k; if (x != x) break; }\n        }\n"
         << "        const long long up_ix = o * " << istr(inner) << " + in_;\n"
         << "        res = (k_ == bi) ? " << up_elem << " : 0.0f;\n";
    } else {
      os << "        const long long o = j / " << istr(inner) << ", in_ = j % " << istr(inner) << ";\n";
      if (c.op == T_SUMAX || c.op == T_RSUM) os << "        double acc = 0.0;\n";
      else if (c.op == T_ARGMAX) os << "        float bv = -J4B_INF; long long bi = 0;\n";
      else if (c.op == T_RMAX) os << "        float acc = -J4B_INF;\n";
      else os << "        float acc = -J4B_INF;\n";
      os << "        for (long long k = 0; k < " << istr(nn) << "; ++k) {\n"
         << "          const long long src_ix = o * " << istr(nn * inner) << " + k * " << istr(inner) << " + in_;\n"
         << "          const float x = " << rd_elem << ";\n";
      if (c.op == T_SUMAX || c.op == T_RSUM) os << "          acc += (double)x;\n        }\n        res = (float)acc;\n";
      else if (c.op == T_MAXAX) os << "          acc = jmax(acc, x);\n        }\n        res = acc;\n";
      else if (c.op == T_RMAX) os << "          if (x > acc) acc = x;\n        }\n        res = acc;\n";
      else os << "          if (x != x) { bi = k; break; } else if (x > bv) { bv = x; bi = k; }\n        }\n        res = (float)bi;\n";
    }
    os << "      }\n      " << vname(b) << "[e * 4 + q] = res;\n    }\n  }\n";
  }

  // ---- fold kernel (POST context) ----
  std::string post_elem(int b) {
    const Val& v = V[b];
    if (v.ctx == X_CONST) return fstr(v.cval);
    if (v.ctx == X_POST && v.kernel == gi) {
      if (v.base >= 0) return post_elem_base(v.base, v.tbl);
      return "p" + std::to_string(b);
    }
    // stored value (global or another group's / this group's shared)
    int64_t L = t.size[b];
    std::string p = gptr(b);
    if (L == 1) return "__ldg(" + p + ")";
    return "(i < " + istr(L) + " ? __ldg(" + p + " + i) : 0.0f)";
  }

  std::string post_elem_base(int base, const Table& tb) {
    int64_t param = 0;
    int k = tclass(tb, V[base].W, &param);
    if (k == TB_CONST && param < 0) return "0.0f";
    return "p" + std::to_string(base);  // scalar broadcast or identity
  }

  void emit_post(const GCall& gc) {
    const TCall& c = t.calls[(size_t)gc.call];
    const int b = c.out;
    Val& v = V[b];
    std::ostringstream& os = fold;
    if (gc.kind == G_VIEW) {
      // identity / scalar-broadcast view: nothing to compute
    } else if (gc.kind == G_COLRED) {
      // 32 columns per CTA; warp w folds CTAs w, w + kFoldWarps, ...; the warp partials are
      // combined in warp order, so the sum is deterministic
      int slot = part_slot[b];
      bool mx = c.op == T_MAXAX;
      os << "  float p" << b << ";\n  {\n    const double* pp = (const double*)A.p[" << slot << "];\n";
      if (mx) os << "    float acc = -J4B_INF;\n    if (i < " << istr(v.W) << ") for (long long cta = warp; cta < A.G; cta += kFoldWarps) acc = jmax(acc, (float)pp[cta * " << istr(v.W) << " + i]);\n"
                 << "    fred[warp * 32 + lane] = (double)acc;\n    __syncthreads();\n"
                 << "    float tot = -J4B_INF;\n    for (int w = 0; w < kFoldWarps; ++w) tot = jmax(tot, (float)fred[w * 32 + lane]);\n";
      else os << "    double acc = 0.0;\n    if (i < " << istr(v.W) << ") {\n"
              << "      const double* q = pp + i;\n      long long cta = warp;\n"
              << "      // four loads in flight, the additions in the same (ascending CTA) order\n"
              << "      for (; cta + 3 * kFoldWarps < A.G; cta += 4 * kFoldWarps) {\n"
              << "        const double v0 = q[cta * " << istr(v.W) << "], v1 = q[(cta + kFoldWarps) * " << istr(v.W) << "];\n"
              << "        const double v2 = q[(cta + 2 * kFoldWarps) * " << istr(v.W) << "], v3 = q[(cta + 3 * kFoldWarps) * " << istr(v.W) << "];\n"
              << "        acc += v0; acc += v1; acc += v2; acc += v3;\n      }\n"
              << "      for (; cta < A.G; cta += kFoldWarps) acc += q[cta * " << istr(v.W) << "];\n    }\n"
              << "    fred[warp * 32 + lane] = acc;\n    __syncthreads();\n"
              << "    double tot = 0.0;\n    for (int w = 0; w < kFoldWarps; ++w) tot += fred[w * 32 + lane];\n";
      os << "    __syncthreads();\n    p" << b << " = (float)tot;\n  }\n";
    } else if (gc.kind == G_GLOBRED) {
      // every warp folds all CTA partials (lane-strided, then a butterfly): same value in all
      int slot = part_slot[b];
      os << "  float p" << b << ";\n  {\n    const double* pp = (const double*)A.p[" << slot << "];\n";
      if (c.op == T_RMAX)
        os << "    float bv = -J4B_INF; long long bi = 0x7fffffffffffffffLL;\n"
           << "    for (long long cta = lane; cta < A.G; cta += 32) rmax_combine(bv, bi, (float)pp[2 * cta], (long long)pp[2 * cta + 1]);\n"
           << "    for (int o = 16; o > 0; o >>= 1) { float v2 = __shfl_xor_sync(0xffffffffu, bv, o); long long i2 = __shfl_xor_sync(0xffffffffu, bi, o); rmax_combine(bv, bi, v2, i2); }\n"
           << "    p" << b << " = bv;\n  }\n";
      else
        os << "    double acc = 0.0;\n    long long cta = lane;\n"
           << "    for (; cta + 96 < A.G; cta += 128) {\n"
           << "      const double v0 = pp[cta], v1 = pp[cta + 32], v2 = pp[cta + 64], v3 = pp[cta + 96];\n"
           << "      acc += v0; acc += v1; acc += v2; acc += v3;\n    }\n"
           << "    for (; cta < A.G; cta += 32) acc += pp[cta];\n"
           << "    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);\n"
           << "    p" << b << " = (float)acc;\n  }\n";
    } else if (gc.kind == G_EXPR) {
      std::vector<std::string> in;
      for (int x : c.ins) in.push_back(post_elem(x));
      std::ostringstream body;
      std::string r = expr_code(c, in, body, "    ");
      os << "  float p" << b << ";\n  {\n" << body.str() << "    p" << b << " = " << r << ";\n  }\n";
    }
    if (v.need_store) {
      std::string p = gptr(b);
      std::string val = post_elem(b);
      if (v.W == 1) os << "  if (i == 0 && warp == 0) " << p << "[0] = " << val << ";\n";
      else os << "  if (i < " << istr(v.W) << " && warp == 0) " << p << "[i] = " << val << ";\n";
    }
  }

  int add_partial(int b, int64_t per_cta) {
    int slot = (int)ptrs.size();
    PtrRef pr;
    pr.kind = 5;  // partial buffer, resolved after the grid is known
    pr.index = (int)partials.size();
    pr.bytes = per_cta;
    ptrs.push_back(pr);
    partials.push_back({b, per_cta});
    part_slot[b] = slot;
    return slot;
  }

  bool generate(GroupCode& gcode) {
    // thread count from the widest row / shared vector
    int64_t wmax = 1;
    for (const GCall& gc : G.calls) {
      const TCall& c = t.calls[(size_t)gc.call];
      if (gc.ctx == X_ROW || gc.ctx == X_SHARED) wmax = std::max(wmax, V[c.out].W);
      for (int x : c.ins) {
        if (gc.ctx == X_ROW && V[x].ctx != X_CONST) wmax = std::max(wmax, t.size[x] / std::max<int64_t>(G.R, 1));
        if (gc.ctx == X_SHARED) wmax = std::max(wmax, t.size[x]);
      }
    }
    // about 16 elements of the widest row per thread. Measured on the RMSNorm + SwiGLU gradient
    // (x [4096, 8192]): 16 per thread at 512 threads 62.3 us per step; 8 per thread at 1024
    // threads 74.4 us (64-register cap); two 512-thread CTAs per SM (64-register cap, spills)
    // 116 us.
    NT = 32;
    while (NT < 1024 && (int64_t)NT * 16 < wmax) NT *= 2;
    row_loaded.assign(t.shape.size(), 0);
    staged_now.assign(t.shape.size(), 0);

    shared_loaded.assign(t.shape.size(), 0);

    // accumulators of cross-row reductions
    std::ostringstream acc, colflush, colstore;
    for (const GCall& gc : G.calls) {
      const TCall& c = t.calls[(size_t)gc.call];
      int b = c.out;
      if (gc.kind == G_COLRED) {
        int64_t W = V[b].W;
        if (c.op == T_MAXAX) acc << "  float cm" << b << "[" << E(W) * 4 << "];\n  #pragma unroll\n  for (int s = 0; s < " << E(W) * 4 << "; ++s) cm" << b << "[s] = -J4B_INF;\n";
        else acc << "  float ca" << b << "[" << E(W) * 4 << "];\n  #pragma unroll\n  for (int s = 0; s < " << E(W) * 4 << "; ++s) ca" << b << "[s] = 0.0f;\n";
        int slot = add_partial(b, W);
        if (c.op != T_MAXAX) {
          // column sums: float per thread for up to 32 rows, then stored (first flush) or added
          // (later flushes) into this CTA's double partial; each thread owns its columns of it,
          // so the partial needs no zeroing pass
          std::string loop = "  #pragma unroll\n  for (int e = 0; e < " + std::to_string(E(W)) +
                             "; ++e) {\n    #pragma unroll\n    for (int q = 0; q < 4; ++q) {\n"
                             "      const long long j = ((long long)e * " + std::to_string(NT) + " + t) * 4 + q;\n"
                             "      if (" + jlt(0, W) + ") ";
          std::string pp = "((double*)A.p[" + std::to_string(slot) + "])[(long long)blockIdx.x * " + istr(W) + " + j]";
          colstore << loop << pp << " = (double)ca" << b << "[e * 4 + q];\n      ca" << b
                   << "[e * 4 + q] = 0.0f;\n    }\n  }\n";
          colflush << loop << pp << " += (double)ca" << b << "[e * 4 + q];\n      ca" << b
                   << "[e * 4 + q] = 0.0f;\n    }\n  }\n";
        }
      } else if (gc.kind == G_GLOBRED) {
        if (c.op == T_RMAX) acc << "  float gm" << b << " = -J4B_INF; long long gi" << b << " = 0x7fffffffffffffffLL;\n";
        else acc << "  double ga" << b << " = 0.0;\n";
        add_partial(b, c.op == T_RMAX ? 2 : 1);
      }
    }

    // prologue (shared context) and row loop body; loads of stored tensors read by identity
    // are discovered while generating and hoisted: row tiles at the top of each row, row-
    // invariant vectors once per CTA
    for (const GCall& gc : G.calls)
      if (gc.ctx == X_SHARED) emit_rowlike(pro, gc);
    flush();
    std::vector<char> staged_pro = staged_now;
    std::ostringstream rowcode;
    for (const GCall& gc : G.calls)
      if (gc.ctx == X_ROW || gc.kind == G_COLRED || gc.kind == G_GLOBRED) emit_rowlike(rowcode, gc);
    flush();
    // row tiles of stored tensors: the next row's tile is loaded while this row computes
    std::ostringstream rowb, sload, pre;
    for (int b : row_loads) {
      emit_load(pre, b, true, "N", "(long long)blockIdx.x", false);
      rowb << "  float L" << b << "[" << E(t.size[b] / G.R) * 4 << "];\n  #pragma unroll\n  for (int s = 0; s < "
           << E(t.size[b] / G.R) * 4 << "; ++s) L" << b << "[s] = N" << b << "[s];\n";
    }
    if (!row_loads.empty()) {
      rowb << "  if (r + gridDim.x < R) {\n";
      for (int b : row_loads) emit_load(rowb, b, true, "N", "(r + gridDim.x)", false);
      rowb << "  }\n";
    }
    rowb << rowcode.str();
    for (int b : shared_loads) emit_load(sload, b, false);
    {
      std::string p2 = sload.str() + pro.str();
      pro.str(p2);
    }
    std::string prefetch = pre.str();
    // staging inside the row loop must not overrun the previous row's readers
    bool row_staging = false;
    for (size_t b = 0; b < staged_now.size(); ++b)
      if (staged_now[b] && !staged_pro[b]) row_staging = true;

    // partial writes after the loop
    for (const GCall& gc : G.calls) {
      const TCall& c = t.calls[(size_t)gc.call];
      int b = c.out;
      if (gc.kind == G_COLRED && c.op != T_MAXAX) {
        continue;  // flushed with the column-sum flush below
      } else if (gc.kind == G_COLRED) {
        int64_t W = V[b].W;
        int slot = part_slot[b];
        fin << "  {\n    double* pp = (double*)A.p[" << slot << "] + (long long)blockIdx.x * " << istr(W) << ";\n"
            << "    #pragma unroll\n    for (int e = 0; e < " << E(W) << "; ++e) {\n"
            << "      #pragma unroll\n      for (int q = 0; q < 4; ++q) {\n"
            << "        const long long j = ((long long)e * " << NT << " + t) * 4 + q;\n"
            << "        if (" << jlt(0, W) << ") pp[j] = "
            << (c.op == T_MAXAX ? "(double)cm" : "ca") << b << "[e * 4 + q];\n      }\n    }\n  }\n";
      } else if (gc.kind == G_GLOBRED) {
        int slot = part_slot[b];
        if (c.op == T_RMAX)
          fin << "  {\n    long long w = block_pair<" << NT << ", 1>(gm" << b << ", gi" << b << ", red, rp);\n"
              << "    if (t == 0) { double* pp = (double*)A.p[" << slot << "]; pp[2 * blockIdx.x] = gm" << b
              << "; pp[2 * blockIdx.x + 1] = (double)w; }\n  }\n";
        else
          fin << "  {\n    double s = block_sum<" << NT << ">(ga" << b << ", red, rp);\n"
              << "    if (t == 0) ((double*)A.p[" << slot << "])[blockIdx.x] = s;\n  }\n";
      }
    }

    // fold kernel
    int64_t flen = 1;
    bool has_fold = false;
    for (const GCall& gc : G.calls) {
      if (gc.ctx != X_POST) continue;
      has_fold = true;
      flen = std::max(flen, V[t.calls[(size_t)gc.call].out].W);
      emit_post(gc);
    }

    const int np = (int)ptrs.size();
    if (np > kMaxPtrs) return false;
    std::ostringstream src;
    src << kPrelude;
    src << "struct Args { u64 p[" << std::max(np, 1) << "]; long long R; long long G; };\n";
    std::string rn = "j4b_group" + std::to_string(gi);
    src << "extern \"C\" __global__ void __launch_bounds__(" << NT << ") " << rn << "(const Args A) {\n"
        << "  extern __shared__ __align__(16) unsigned char smraw[];\n"
        << "  double* red = reinterpret_cast<double*>(smraw);\n"
        << "  int rp = 0;\n  (void)rp;\n"
        << "  float* sm = reinterpret_cast<float*>(smraw + " << (4 * (NT / 32) * 8) << ");\n"
        << "  (void)red; (void)sm;\n"
        << "  const int t = threadIdx.x;\n"
        << "  const long long R = A.R;\n  (void)R;\n"
        << kPdlPrologue << pro.str() << acc.str();
    std::string cf;
    if (!colflush.str().empty()) {
      src << "  bool col_first = true;\n";
      cf = "  if (col_first) {\n" + colstore.str() + "  } else {\n" + colflush.str() + "  }\n  col_first = false;\n";
    }
    if (G.has_rows) {
      for (int b : row_loads) src << "  float N" << b << "[" << E(t.size[b] / G.R) * 4 << "];\n";
      if (!row_loads.empty()) src << "  if ((long long)blockIdx.x < R) {\n" << prefetch << "  }\n";
      if (!cf.empty()) src << "  int rows_in_acc = 0;\n";
      src << "  for (long long r = blockIdx.x; r < R; r += gridDim.x) {\n";
      if (row_staging) src << "  __syncthreads();\n";
      src << rowb.str();
      if (!cf.empty()) src << "  if (++rows_in_acc == 32) {\n  rows_in_acc = 0;\n" << cf << "  }\n";
      src << "  }\n";
    }
    src << cf << fin.str() << "}\n";
    if (has_fold) {
      src << "constexpr int kFoldWarps = " << kFoldThreads / 32 << ";\n"
          << "extern \"C\" __global__ void __launch_bounds__(" << kFoldThreads << ") " << rn << "_fold(const Args A) {\n"
          << "  __shared__ double fred[" << kFoldThreads << "];\n  (void)fred;\n"
          << "  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;\n  (void)warp;\n"
          << "  const long long i = (long long)blockIdx.x * 32 + lane;\n" << kPdlPrologue << fold.str() << "}\n";
    }
    gcode.src = src.str();
    gcode.row_name = rn;
    gcode.fold_name = rn + "_fold";
    gcode.NT = NT;
    gcode.smem = 4 * (NT / 32) * 8 + smem_floats * 4;
    gcode.fold = has_fold;
    gcode.fold_len = flen;
    gcode.partials = partials;
    return true;
  }
};

}  // namespace
}  // namespace j4b

// =============================================================================================
// C ABI
// =============================================================================================

using namespace j4b;

namespace {

int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

int canon_of(const std::vector<Val>& V, int b) {
  while (V[(size_t)b].base >= 0 && !V[(size_t)b].tbl && V[(size_t)b].ctx != X_GLOBAL &&
         V[(size_t)b].ctx != X_CONST)
    b = V[(size_t)b].base;
  return b;
}

// storage assignment: outputs first (a value that is an output lives in the caller's buffer),
// then arena slots for every other materialised value
int assign_storage(j4b_tape* tp, std::vector<int>& copy_outputs) {
  TapeIR& t = tp->ir;
  std::vector<Val>& V = tp->V;
  const size_t nb = t.shape.size();
  tp->loc.assign(nb, PtrRef());
  std::vector<char> is_input(nb, 0);
  for (size_t k = 0; k < t.inputs.size(); ++k) {
    tp->loc[(size_t)t.inputs[k]].kind = 1;
    tp->loc[(size_t)t.inputs[k]].index = (int)k;
    is_input[(size_t)t.inputs[k]] = 1;
  }
  std::vector<char> taken(nb, 0);
  for (size_t k = 0; k < t.outputs.size(); ++k) {
    int b = canon_of(V, t.outputs[k]);
    const Val& v = V[(size_t)b];
    // the output's own storage root
    int root = v.ctx == X_GLOBAL ? v.root : b;
    bool own = v.ctx != X_GLOBAL || (v.off == 0 && !is_input[(size_t)root] && t.size[(size_t)root] == t.size[(size_t)b]);
    if (own && !taken[(size_t)root] && tp->loc[(size_t)root].kind == 0) {
      tp->loc[(size_t)root].kind = 2;
      tp->loc[(size_t)root].index = (int)k;
      taken[(size_t)root] = 1;
    } else {
      copy_outputs.push_back((int)k);
    }
  }
  int64_t arena = 0;
  for (size_t b = 0; b < nb; ++b) {
    const Val& v = V[b];
    bool materialised = (v.ctx == X_GLOBAL && v.root == (int)b) || v.need_store;
    if (!materialised || tp->loc[b].kind != 0) continue;
    tp->loc[b].kind = 3;
    tp->loc[b].bytes = arena;
    arena = align_up(arena + t.size[b] * 4, 256);
  }
  tp->arena_bytes = (size_t)arena;
  return J4B_OK;
}

}  // namespace

namespace {

// Parses, validates, plans and generates code (no device work).
int build_tape(j4b_tape* tp, const int64_t* words, size_t nwords, std::vector<GroupCode>& codes,
               std::vector<std::vector<int64_t>>& tables, std::vector<int>& copy_outputs) {
  std::string err;
  if (!parse_tape(words, nwords, tp->ir, err) || !validate(tp->ir, err))
    return set_error(J4B_EINVAL, "%s", err.c_str());
  Planner pl(tp->ir);
  pl.plan();
  tp->V = pl.V;
  tp->groups = pl.groups;
  tp->steps = pl.steps;
  tp->fills = pl.fills;
  tp->tsrc = pl.tsrc;
  codes.assign(tp->groups.size(), GroupCode());
  tp->runs.assign(tp->groups.size(), j4b_tape::GroupRun());
  for (size_t g = 0; g < tp->groups.size(); ++g) {
    Gen gen(*tp, (int)g, tp->runs[g].ptrs, tables);
    if (!gen.generate(codes[g]))
      return set_error(J4B_EUNSUPPORTED, "tape group %zu needs too many buffers", g);
    tp->runs[g].src = codes[g].src;
  }
  assign_storage(tp, copy_outputs);
  return J4B_OK;
}

}  // namespace

extern "C" int j4b_tape_dryrun(const int64_t* words, size_t nwords, j4b_tape_stats* stats,
                               char* buf, size_t cap, size_t* len) {
  J4B_REQUIRE(words != nullptr, "null argument");
  std::unique_ptr<j4b_tape> tp(new j4b_tape());
  std::vector<GroupCode> codes;
  std::vector<std::vector<int64_t>> tables;
  std::vector<int> copy_outputs;
  int st = build_tape(tp.get(), words, nwords, codes, tables, copy_outputs);
  if (st) return st;
  std::string all;
  for (size_t g = 0; g < codes.size(); ++g) {
    std::vector<char> cubin;
    st = compile_source(codes[g].src, "j4b_tape.cu", cubin, true);
    if (st) return st;
    all += "// ---- group " + std::to_string(g) + " ----\n" + codes[g].src;
  }
  if (stats) {
    std::memset(stats, 0, sizeof *stats);
    stats->calls = (int)tp->ir.calls.size();
    for (const Step& s : tp->steps) {
      if (s.kind == S_GROUP) {
        stats->groups++;
        if (codes[(size_t)s.group].fold) stats->folds++;
      } else if (s.kind == S_EAGER) {
        stats->eager_steps++;
      }
    }
    stats->copies = (int)copy_outputs.size();
    stats->fills = (int)tp->fills.size();
    stats->arena_bytes = (int64_t)tp->arena_bytes;
  }
  if (len) *len = all.size();
  if (buf && cap) {
    size_t n = std::min(cap - 1, all.size());
    std::memcpy(buf, all.data(), n);
    buf[n] = 0;
  }
  return J4B_OK;
}

extern "C" int j4b_tape_compile(int dev, const int64_t* words, size_t nwords, j4b_tape** out) {
  J4B_REQUIRE(out != nullptr && words != nullptr, "null argument");
  *out = nullptr;
  int st = ensure_device(dev);
  if (st) return st;
  DeviceGuard guard(dev);
  std::unique_ptr<j4b_tape> tp(new j4b_tape());
  tp->dev = dev;
  std::vector<GroupCode> codes;
  std::vector<std::vector<int64_t>> tables;
  std::vector<int> copy_outputs;
  st = build_tape(tp.get(), words, nwords, codes, tables, copy_outputs);
  if (st) return st;
  std::string err;
  cudaFree(0);  // make the primary context current for the driver API
  if (!driver().ok) return set_error(J4B_ECUDA, "CUDA driver entry points are unavailable");

  // partial buffers and eager maps go after the value slots in the arena
  int64_t arena = (int64_t)tp->arena_bytes;
  DeviceCtx* ctx = device_ctx(dev);
  for (size_t g = 0; g < tp->groups.size(); ++g) {
    j4b_tape::GroupRun& run = tp->runs[g];
    std::vector<char> cubin;
    st = compile_source(codes[g].src, "j4b_tape.cu", cubin, true);
    if (st) return st;
    CUresult r = driver().ModuleLoadData(&run.mod, cubin.data());
    if (r != CUDA_SUCCESS) return cu_error(r, "cuModuleLoadData");
    r = driver().ModuleGetFunction(&run.row, run.mod, codes[g].row_name.c_str());
    if (r != CUDA_SUCCESS) return cu_error(r, "cuModuleGetFunction");
    if (codes[g].fold) {
      r = driver().ModuleGetFunction(&run.fold, run.mod, codes[g].fold_name.c_str());
      if (r != CUDA_SUCCESS) return cu_error(r, "cuModuleGetFunction");
    }
    run.NT = codes[g].NT;
    run.smem = codes[g].smem;
    if (run.smem > 48 * 1024) {
      if (run.smem > 227 * 1024) return set_error(J4B_EUNSUPPORTED, "tape group %zu stages too much data", g);
      r = driver().FuncSetAttribute(run.row, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, (int)run.smem);
      if (r != CUDA_SUCCESS) return cu_error(r, "cuFuncSetAttribute");
    }
    int per_sm = 1;
    r = driver().Occupancy(&per_sm, run.row, run.NT, run.smem);
    if (r != CUDA_SUCCESS) return cu_error(r, "cuOccupancyMaxActiveBlocksPerMultiprocessor");
    per_sm = std::max(per_sm, 1);
    const Group& G = tp->groups[g];
    run.R = G.has_rows ? G.R : 0;
    int64_t grid = G.has_rows ? std::min<int64_t>(G.R, (int64_t)ctx->sm_count * per_sm) : 1;
    run.grid = (int)std::max<int64_t>(grid, 1);
    run.fold_grid = (int)((codes[g].fold_len + 31) / 32);
    for (PtrRef& pr : run.ptrs) {
      if (pr.kind == 5) {
        pr.kind = 3;
        int64_t per = pr.bytes;
        pr.bytes = arena;
        arena = align_up(arena + per * run.grid * 8, 256);
      }
    }
  }
  // maps of eager reindex / scatterAdd calls
  tp->map_off.assign(tp->ir.calls.size(), -1);
  for (const Step& s : tp->steps) {
    if (s.kind != S_EAGER) continue;
    const TCall& c = tp->ir.calls[(size_t)s.call];
    if (c.op == T_REINDEX) {
      tp->map_off[(size_t)s.call] = arena;
      arena = align_up(arena + tp->ir.size[(size_t)c.out] * 4, 256);
    } else if (c.op == T_SCATTER) {
      // destination offsets (n_out + 1) then source indices (n_in), int64
      tp->map_off[(size_t)s.call] = arena;
      arena = align_up(arena + (tp->ir.size[(size_t)c.out] + 1 + tp->ir.size[(size_t)c.ins[0]]) * 8, 256);
    }
  }
  tp->arena_bytes = (size_t)arena;
  // table blob
  int64_t tb = 0;
  for (auto& tv : tables) {
    tp->tbl_off.push_back(tb);
    tb = align_up(tb + (int64_t)tv.size() * 8, 256);
  }
  tp->tblob_bytes = (size_t)tb;
  if (tp->arena_bytes) J4B_CUDA(cudaMalloc(&tp->arena, tp->arena_bytes), "cudaMalloc(tape arena)");
  if (tp->tblob_bytes) {
    J4B_CUDA(cudaMalloc(&tp->tblob, tp->tblob_bytes), "cudaMalloc(tape tables)");
    for (size_t i = 0; i < tables.size(); ++i)
      J4B_CUDA(cudaMemcpy((char*)tp->tblob + tp->tbl_off[i], tables[i].data(), tables[i].size() * 8,
                          cudaMemcpyHostToDevice), "cudaMemcpy(tape tables)");
  }
  // eager maps (int32, as the SPI kernels take them)
  for (size_t ci = 0; ci < tp->ir.calls.size(); ++ci) {
    if (tp->map_off[ci] < 0) continue;
    const TCall& c = tp->ir.calls[ci];
    IndexMap m;
    const Shape& side = c.op == T_REINDEX ? tp->ir.shape[(size_t)c.out] : tp->ir.shape[(size_t)c.ins[0]];
    int64_t limit = c.op == T_REINDEX ? tp->ir.size[(size_t)c.ins[0]] : tp->ir.size[(size_t)c.out];
    decode_map(c.at, side, limit, m, err);
    int64_t n = numel(side);
    if (c.op == T_REINDEX) {
      std::vector<int32_t> host((size_t)n);
      for (int64_t f = 0; f < n; ++f) host[(size_t)f] = (int32_t)m.at(f);
      J4B_CUDA(cudaMemcpy((char*)tp->arena + tp->map_off[ci], host.data(), (size_t)n * 4, cudaMemcpyHostToDevice),
               "cudaMemcpy(tape map)");
    } else {
      // sources grouped by destination, ascending (counting sort keeps the source order)
      const int64_t nd = tp->ir.size[(size_t)c.out];
      std::vector<int64_t> host((size_t)(nd + 1 + n), 0);
      int64_t* off = host.data();
      int64_t* src = host.data() + nd + 1;
      for (int64_t f = 0; f < n; ++f) {
        int64_t k = m.at(f);
        if (k >= 0) off[k + 1]++;
      }
      for (int64_t k = 0; k < nd; ++k) off[k + 1] += off[k];
      std::vector<int64_t> fillp(off, off + nd);
      for (int64_t f = 0; f < n; ++f) {
        int64_t k = m.at(f);
        if (k >= 0) src[fillp[(size_t)k]++] = f;
      }
      J4B_CUDA(cudaMemcpy((char*)tp->arena + tp->map_off[ci], host.data(), host.size() * 8, cudaMemcpyHostToDevice),
               "cudaMemcpy(tape map)");
    }
  }
  // output copies become steps at the end
  for (int k : copy_outputs) {
    Step s;
    s.kind = S_COPY;
    s.buf = tp->ir.outputs[(size_t)k];
    s.out_index = k;
    tp->steps.push_back(s);
  }
  int launches = (int)tp->fills.size();
  for (const Step& s : tp->steps) {
    if (s.kind == S_GROUP) launches += tp->runs[(size_t)s.group].fold ? 2 : 1;
    else launches += 1;
  }
  tp->launches_per_replay = launches;
  *out = tp.release();
  return J4B_OK;
}

namespace {

struct LaunchCtx {
  j4b_tape* tp;
  const j4b_buf* in;
  const j4b_buf* out;
};

uint64_t resolve(const LaunchCtx& L, const PtrRef& pr) {
  switch (pr.kind) {
    case 1: return L.in[pr.index];
    case 2: return L.out[pr.index];
    case 3: return (uint64_t)(uintptr_t)L.tp->arena + (uint64_t)pr.bytes;
    case 4: return (uint64_t)(uintptr_t)L.tp->tblob + (uint64_t)L.tp->tbl_off[(size_t)pr.index];
  }
  return 0;
}

// device address of a materialised value (its storage root + element offset)
uint64_t addr_of(const LaunchCtx& L, int b) {
  b = canon_of(L.tp->V, b);
  const Val& v = L.tp->V[(size_t)b];
  int root = b;
  int64_t off = 0;
  if (v.ctx == X_GLOBAL) {
    root = v.root;
    off = v.off;
  }
  return resolve(L, L.tp->loc[(size_t)root]) + (uint64_t)off * 4;
}

// A generated kernel launch with programmatic stream serialization (cuLaunchKernelEx); plain
// cuLaunchKernel where the driver lacks it (the kernels' griddepcontrol then return at once).
CUresult launch_pdl(CUfunction f, unsigned grid, unsigned threads, unsigned smem, cudaStream_t stream, void** params) {
  if (!driver().LaunchKernelEx)
    return driver().LaunchKernel(f, grid, 1, 1, threads, 1, 1, smem, (CUstream)stream, params, nullptr);
  CUlaunchConfig cfg = {};
  cfg.gridDimX = grid;
  cfg.gridDimY = cfg.gridDimZ = 1;
  cfg.blockDimX = threads;
  cfg.blockDimY = cfg.blockDimZ = 1;
  cfg.sharedMemBytes = smem;
  cfg.hStream = (CUstream)stream;
  CUlaunchAttribute attr[1];
  attr[0].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
  attr[0].value.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return driver().LaunchKernelEx(&cfg, f, params, nullptr);
}

int run_eager(const LaunchCtx& L, int ci, cudaStream_t stream) {
  const TapeIR& t = L.tp->ir;
  const TCall& c = t.calls[(size_t)ci];
  j4b_stream s = (j4b_stream)stream;
  auto A = [&](int i) { return (j4b_buf)addr_of(L, c.ins[(size_t)i]); };
  j4b_buf o = (j4b_buf)addr_of(L, c.out);
  const Shape& os = t.shape[(size_t)c.out];
  auto ishape = [&](int i) -> const Shape& { return t.shape[(size_t)c.ins[(size_t)i]]; };
  switch (c.op) {
    case T_MATMUL: {
      // an absorbed transpose operand is read from its source, transposed in place
      const int b0 = c.ins[0], b1 = c.ins[1];
      const int s0 = L.tp->tsrc[(size_t)b0], s1 = L.tp->tsrc[(size_t)b1];
      const float* pa = (const float*)addr_of(L, s0 >= 0 ? s0 : b0);
      const float* pb = (const float*)addr_of(L, s1 >= 0 ? s1 : b1);
      return matmul_strided(pa, pb, (float*)o, 1, ishape(0)[0], ishape(0)[1], ishape(1)[1], s0 >= 0, s1 >= 0, 0,
                            L.tp->dev, stream);
    }
    case T_BMM:
      return j4b_matmul(A(0), A(1), o, ishape(0)[0], ishape(0)[1], ishape(0)[2], ishape(1)[2], 0, s);
    case T_TRANSPOSE: return j4b_transpose(A(0), o, ishape(0)[0], ishape(0)[1], s);
    case T_STACK0: {
      int64_t each = t.size[(size_t)c.ins[0]];
      for (size_t i = 0; i < c.ins.size(); ++i) {
        int st = j4b_d2d(o + (j4b_buf)(i * each * 4), A((int)i), (size_t)each * 4, s);
        if (st) return st;
      }
      return J4B_OK;
    }
    case T_RSUM: return j4b_reduce_sum(A(0), t.size[(size_t)c.ins[0]], o, s);
    case T_RMAX: return j4b_reduce_max(A(0), t.size[(size_t)c.ins[0]], o, s);
    case T_SUMAX: case T_MAXAX: case T_ARGMAX: {
      int64_t outer, nn, inner;
      axis_split(ishape(0), (int)c.at[0], &outer, &nn, &inner);
      if (c.op == T_SUMAX) return j4b_sum_axis(A(0), outer, nn, inner, o, s);
      if (c.op == T_MAXAX) return j4b_max_axis(A(0), outer, nn, inner, o, s);
      return j4b_argmax_axis(A(0), outer, nn, inner, o, s);
    }
    case T_MAXBWD: {
      int64_t outer, nn, inner;
      axis_split(ishape(1), (int)c.at[0], &outer, &nn, &inner);
      return j4b_max_axis_backward(A(0), A(1), outer, nn, inner, o, s);
    }
    case T_BCAST:
      return j4b_broadcast_to(A(0), ishape(0).data(), (int)ishape(0).size(), os.data(), (int)os.size(), o, s);
    case T_REINDEX:
      return j4b_reindex(A(0), t.size[(size_t)c.ins[0]],
                         (j4b_buf)((uintptr_t)L.tp->arena + L.tp->map_off[(size_t)ci]), t.size[(size_t)c.out], o, s);
    case T_SCATTER: {
      const int64_t nd = t.size[(size_t)c.out];
      const int64_t* off = (const int64_t*)((char*)L.tp->arena + L.tp->map_off[(size_t)ci]);
      return launch_segment_sum((const float*)(uintptr_t)A(0), off, off + nd + 1, nd, (float*)(uintptr_t)o, s);
    }
    case T_RUNIF: return j4b_random_uniform(c.at[0], c.at[1], o, t.size[(size_t)c.out], s);
    case T_RNORM: return j4b_random_normal(c.at[0], c.at[1], o, t.size[(size_t)c.out], s);
    case T_BINARY: return j4b_binary((int)c.at[0], A(0), A(1), o, t.size[(size_t)c.out], s);
    case T_UNARY: return j4b_unary((int)c.at[0], A(0), o, t.size[(size_t)c.out], s);
    case T_SCALAR: {
      double d;
      std::memcpy(&d, &c.at[1], 8);
      return j4b_scalar((int)c.at[0], A(0), d, o, t.size[(size_t)c.out], s);
    }
    case T_RELUBWD: return j4b_relu_backward(A(0), A(1), o, t.size[(size_t)c.out], s);
  }
  return set_error(J4B_EUNSUPPORTED, "tape call %d (op %d) has no eager kernel", ci, c.op);
}

}  // namespace

extern "C" int j4b_tape_launch(j4b_tape* tp, const j4b_buf* inputs, int nin, const j4b_buf* outputs,
                               int nout, j4b_stream s) {
  J4B_REQUIRE(tp != nullptr, "null tape");
  J4B_REQUIRE(nin == (int)tp->ir.inputs.size(), "tape expects %zu inputs, got %d", tp->ir.inputs.size(), nin);
  J4B_REQUIRE(nout == (int)tp->ir.outputs.size(), "tape expects %zu outputs, got %d", tp->ir.outputs.size(), nout);
  for (int i = 0; i < nin; ++i)
    J4B_REQUIRE(inputs[i] % 16 == 0 || tp->ir.size[(size_t)tp->ir.inputs[(size_t)i]] == 0,
                "tape input %d must be 16-byte aligned", i);
  for (int i = 0; i < nout; ++i)
    J4B_REQUIRE(outputs[i] % 16 == 0 || tp->ir.size[(size_t)tp->ir.outputs[(size_t)i]] == 0,
                "tape output %d must be 16-byte aligned", i);
  std::lock_guard<std::mutex> lk(tp->mu);
  DeviceGuard guard(tp->dev);
  cudaStream_t stream = resolve_stream(tp->dev, s);
  LaunchCtx L{tp, inputs, outputs};
  // constants that must exist in memory
  for (int b : tp->fills) {
    int st = j4b_fill((j4b_buf)addr_of(L, b), tp->ir.size[(size_t)b], tp->V[(size_t)b].cval, (j4b_stream)stream);
    if (st) return st;
  }
  for (const Step& step : tp->steps) {
    if (step.kind == S_GROUP) {
      j4b_tape::GroupRun& run = tp->runs[(size_t)step.group];
      std::vector<uint64_t> args(std::max<size_t>(run.ptrs.size(), 1) + 2, 0);
      for (size_t k = 0; k < run.ptrs.size(); ++k) {
        const PtrRef& pr = run.ptrs[k];
        args[k] = pr.kind == 10 ? (uint64_t)addr_of(L, pr.index) : resolve(L, pr);
      }
      size_t np = std::max<size_t>(run.ptrs.size(), 1);
      args[np] = (uint64_t)run.R;
      args[np + 1] = (uint64_t)run.grid;
      void* params[] = {args.data()};
      CUresult r = launch_pdl(run.row, (unsigned)run.grid, (unsigned)run.NT, (unsigned)run.smem, stream, params);
      if (r != CUDA_SUCCESS) return cu_error(r, "cuLaunchKernel(tape group)");
      count_launch();
      if (run.fold) {
        r = launch_pdl(run.fold, (unsigned)run.fold_grid, kFoldThreads, 0, stream, params);
        if (r != CUDA_SUCCESS) return cu_error(r, "cuLaunchKernel(tape fold)");
        count_launch();
      }
    } else if (step.kind == S_EAGER) {
      int st = run_eager(L, step.call, stream);
      if (st) return st;
    } else if (step.kind == S_COPY) {
      int b = step.buf;
      const Val& v = tp->V[(size_t)b];
      j4b_buf dst = outputs[step.out_index];
      int st;
      if (v.ctx == X_CONST && !v.need_store)
        st = j4b_fill(dst, tp->ir.size[(size_t)b], v.cval, (j4b_stream)stream);
      else
        st = j4b_d2d(dst, (j4b_buf)addr_of(L, b), (size_t)tp->ir.size[(size_t)b] * 4, (j4b_stream)stream);
      if (st) return st;
    }
  }
  return J4B_OK;
}

extern "C" int j4b_tape_free(j4b_tape* tp) {
  if (!tp) return J4B_OK;
  {
    DeviceGuard guard(tp->dev);
    cudaDeviceSynchronize();
    for (auto& r : tp->runs)
      if (r.mod) driver().ModuleUnload(r.mod);
    if (tp->arena) cudaFree(tp->arena);
    if (tp->tblob) cudaFree(tp->tblob);
  }
  delete tp;
  return J4B_OK;
}

extern "C" int j4b_tape_info(j4b_tape* tp, j4b_tape_stats* st) {
  J4B_REQUIRE(tp != nullptr && st != nullptr, "null argument");
  std::memset(st, 0, sizeof *st);
  for (const Step& s : tp->steps) {
    if (s.kind == S_GROUP) {
      st->groups++;
      if (tp->runs[(size_t)s.group].fold) st->folds++;
    } else if (s.kind == S_EAGER) {
      st->eager_steps++;
    } else if (s.kind == S_COPY) {
      st->copies++;
    }
  }
  st->fills = (int)tp->fills.size();
  st->launches = tp->launches_per_replay;
  st->arena_bytes = (int64_t)tp->arena_bytes;
  st->calls = (int)tp->ir.calls.size();
  return J4B_OK;
}

extern "C" int j4b_tape_source(j4b_tape* tp, int group, char* buf, size_t cap, size_t* len) {
  J4B_REQUIRE(tp != nullptr, "null tape");
  J4B_REQUIRE(group >= 0 && group < (int)tp->runs.size(), "no group %d", group);
  const std::string& s = tp->runs[(size_t)group].src;
  if (len) *len = s.size();
  if (buf && cap) {
    size_t n = std::min(cap - 1, s.size());
    std::memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
  return J4B_OK;
}
