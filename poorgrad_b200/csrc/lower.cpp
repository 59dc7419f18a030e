// lower.cpp -- plan columns -> device program (value kinds, fusion groups,
// emitted kernel sources, buffer liveness and the arena layout).
//
// The node semantics restated here are those of topos's Function rules and
// Tensor arithmetic (function/*.rs `forward`, payload/tensor.rs); the device
// arithmetic uses IEEE round-to-nearest intrinsics without contraction so that
// every elementwise group without a transcendental reproduces the interpreter
// bit for bit.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <set>
#include <sstream>
#include <stdexcept>
#include <unordered_map>

#include "engine.h"
#include "kernels.h"

namespace tb {
namespace {

[[noreturn]] void fail(const std::string& m) { throw std::runtime_error(m); }

bool is_elementwise(int op) {
  switch (op) {
    case TB_OP_ADD: case TB_OP_SUB: case TB_OP_MUL: case TB_OP_DIV: case TB_OP_NEG:
    case TB_OP_TANH: case TB_OP_EXP: case TB_OP_LN: case TB_OP_SQRT: case TB_OP_POWF:
    case TB_OP_MAXIMUM: case TB_OP_RELU: case TB_OP_STEP:
      return true;
    default:
      return false;
  }
}

bool is_view(int op) {
  switch (op) {
    case TB_OP_TRANSPOSE: case TB_OP_BROADCAST: case TB_OP_BROADCAST_ALONG:
    case TB_OP_RESHAPE: case TB_OP_PERMUTE: case TB_OP_NARROW: case TB_OP_UNFOLD:
      return true;
    default:
      return false;
  }
}

bool is_transcendental(int op) {
  return op == TB_OP_TANH || op == TB_OP_EXP || op == TB_OP_LN || op == TB_OP_POWF;
}

// `f32::max` (payload/elementary.rs:137-139); ties keep the first argument.
float fmax_ref(float a, float b) {
  if (std::isnan(a)) return b;
  if (std::isnan(b)) return a;
  return (b > a) ? b : a;
}

// Host evaluation of one elementwise op on constants: the same IEEE f32
// operations (this file is compiled without contraction) and the host libm.
float fold_scalar(int op, float a, float b) {
  switch (op) {
    case TB_OP_ADD: return a + b;
    case TB_OP_SUB: return a - b;
    case TB_OP_MUL: return a * b;
    case TB_OP_DIV: return a / b;
    case TB_OP_NEG: return -a;
    case TB_OP_TANH: return tanhf(a);
    case TB_OP_EXP: return expf(a);
    case TB_OP_LN: return logf(a);
    case TB_OP_SQRT: return sqrtf(a);
    case TB_OP_POWF: return powf(a, b);
    case TB_OP_MAXIMUM: return fmax_ref(a, b);
    case TB_OP_RELU: return fmax_ref(a, 0.0f);
    case TB_OP_STEP: return a >= b ? 1.0f : 0.0f;
  }
  fail("fold_scalar: not elementwise");
}

Layout contiguous(const Node& n) {
  Layout l;
  l.rank = n.rank;
  int64_t s = 1;
  for (int i = n.rank - 1; i >= 0; --i) {
    l.shape[i] = n.shape[i];
    l.stride[i] = s;
    s *= n.shape[i];
  }
  return l;
}

// View-compatible strides for a reshape (the chunk-matching rule used by
// strided tensor libraries); false when the reshape needs a copy.
bool reshape_strides(const Layout& in, const Node& out, Layout& res) {
  res = Layout();
  res.rank = out.rank;
  res.offset = in.offset;
  for (int i = 0; i < out.rank; ++i) res.shape[i] = out.shape[i];
  if (in.rank == 0) {
    for (int i = 0; i < out.rank; ++i) res.stride[i] = 0;
    return true;
  }
  int view_d = out.rank - 1;
  int64_t chunk_base_stride = in.stride[in.rank - 1];
  int64_t tensor_numel = 1, view_numel = 1;
  for (int tensor_d = in.rank - 1; tensor_d >= 0; --tensor_d) {
    tensor_numel *= in.shape[tensor_d];
    if (tensor_d == 0 || (in.shape[tensor_d - 1] != 1 &&
                          in.stride[tensor_d - 1] != tensor_numel * chunk_base_stride)) {
      while (view_d >= 0 && (view_numel < tensor_numel || out.shape[view_d] == 1)) {
        res.stride[view_d] = view_numel * chunk_base_stride;
        view_numel *= out.shape[view_d];
        --view_d;
      }
      if (view_numel != tensor_numel) return false;
      if (tensor_d > 0) {
        chunk_base_stride = in.stride[tensor_d - 1];
        tensor_numel = 1;
        view_numel = 1;
      }
    }
  }
  return view_d == -1;
}

// The layout of view node `n` over its operand's layout `in`.
bool view_layout(const Node& n, const Node& operand, const Layout& in, Layout& out) {
  const int64_t* at = n.attrs;
  out = in;
  switch (n.op) {
    case TB_OP_TRANSPOSE:
      if (in.rank == 2) {
        std::swap(out.shape[0], out.shape[1]);
        std::swap(out.stride[0], out.stride[1]);
      }
      return true;
    case TB_OP_PERMUTE:
      for (int j = 0; j < n.rank; ++j) {
        out.shape[j] = in.shape[at[j]];
        out.stride[j] = in.stride[at[j]];
      }
      return true;
    case TB_OP_NARROW:
      out.offset = in.offset + at[1] * in.stride[at[0]];
      out.shape[at[0]] = at[2];
      return true;
    case TB_OP_BROADCAST_ALONG: {
      int axis = (int)at[0];
      out.rank = n.rank;
      for (int j = 0, s = 0; j < n.rank; ++j) {
        if (j == axis) {
          out.shape[j] = n.shape[j];
          out.stride[j] = 0;
        } else {
          out.shape[j] = in.shape[s];
          out.stride[j] = in.stride[s];
          ++s;
        }
      }
      return true;
    }
    case TB_OP_BROADCAST: {
      out.rank = n.rank;
      for (int j = 0; j < n.rank; ++j) {
        out.shape[j] = n.shape[j];
        out.stride[j] = 0;
      }
      return true;
    }
    case TB_OP_RESHAPE:
      return reshape_strides(in, n, out);
    case TB_OP_UNFOLD: {
      int axis = (int)at[0];
      out.rank = n.rank;
      for (int j = 0, s = 0; j < n.rank; ++j) {
        if (j == axis) {
          out.shape[j] = n.shape[j];
          out.stride[j] = in.stride[s] * at[2];
        } else if (j == axis + 1) {
          out.shape[j] = n.shape[j];
          out.stride[j] = in.stride[s] * at[3];
          ++s;
        } else {
          out.shape[j] = in.shape[s];
          out.stride[j] = in.stride[s];
          ++s;
        }
      }
      (void)operand;
      return true;
    }
  }
  return false;
}

// ------------------------------------------------------------ index strings
bool numeric(const std::string& s, int64_t& v) {
  if (s.empty()) return false;
  char* end = nullptr;
  long long x = strtoll(s.c_str(), &end, 10);
  if (*end) return false;
  v = x;
  return true;
}
std::string lit(int64_t v) {
  std::string s = std::to_string(v);
  if (v > 2147483647LL || v < -2147483647LL) s += "LL";
  return s;
}
std::string s_add(const std::string& a, const std::string& b) {
  int64_t x, y;
  bool na = numeric(a, x), nb = numeric(b, y);
  if (na && nb) return lit(x + y);
  if (na && x == 0) return b;
  if (nb && y == 0) return a;
  return "(" + a + "+" + b + ")";
}
std::string s_mul(const std::string& a, int64_t k) {
  int64_t x;
  if (k == 0) return "0";
  if (k == 1) return a;
  if (numeric(a, x)) return lit(x * k);
  return "(" + a + "*" + lit(k) + ")";
}
std::string s_div(const std::string& a, int64_t k) {
  int64_t x;
  if (k == 1) return a;
  if (numeric(a, x)) return lit(x / k);
  return "(" + a + "/" + lit(k) + ")";
}
std::string s_mod(const std::string& a, int64_t k) {
  int64_t x;
  if (k == 1) return "0";
  if (numeric(a, x)) return lit(x % k);
  return "(" + a + "%" + lit(k) + ")";
}
// Column sums over at most this many rows run as one serial fold per column
// (the REDUCE kernel) instead of per-block partials and a final.
constexpr int64_t kSerialColumnRows = 256;

std::string flit(float f) {
  uint32_t bits;
  memcpy(&bits, &f, 4);
  char buf[40];
  snprintf(buf, sizeof buf, "__int_as_float(0x%08x)", bits);
  return buf;
}

// The constant a flit() literal spells, if `s` is one.
static bool literal_value(const std::string& s, float& out) {
  unsigned bits = 0;
  int used = 0;
  if (sscanf(s.c_str(), "__int_as_float(0x%8x)%n", &bits, &used) != 1 || used != (int)s.size())
    return false;
  memcpy(&out, &bits, 4);
  return true;
}
// 1/c when c is a power of two, whose reciprocal is exact (a normal c's
// reciprocal is at least 2^-127, a representable subnormal): x / c and
// x * (1/c) are then the same real number, rounded once -- bit for bit the
// same result, NaN, infinity and signed zero included.
static bool exact_reciprocal(float c, float& r) {
  uint32_t bits;
  memcpy(&bits, &c, 4);
  const uint32_t e = (bits >> 23) & 0xff;
  if ((bits & 0x7fffff) != 0 || e == 0 || e == 0xff) return false;
  r = 1.0f / c;
  return true;
}

struct Idx {
  std::vector<std::string> c;
  int lane = -1;          // c.back() == lbase + lane
  std::string lbase;
};

}  // namespace

// ============================================================== lowering
class Lowerer {
 public:
  Program& P;
  explicit Lowerer(Program& p) : P(p) {}

  int add_node(const Node& n) {
    P.nodes.push_back(n);
    P.info.emplace_back();
    return (int)P.nodes.size() - 1;
  }

  int resolve(int n) const {
    while (n >= 0 && P.info[n].alias >= 0) n = P.info[n].alias;
    return n;
  }

  int new_buffer(Storage s, int64_t bytes, int node, int slot = -1) {
    Buffer b;
    b.storage = s;
    b.bytes = bytes;
    b.node = node;
    b.slot = slot;
    P.buffers.push_back(b);
    return (int)P.buffers.size() - 1;
  }

  // ---- pass 1: load columns, expand LogSumExp / LogSoftmax into primitives
  void load(const tb_plan_desc* d) {
    if (d->element != TB_ELEMENT_F32 && d->element != TB_ELEMENT_BF16)
      fail("unknown element type " + std::to_string(d->element));
    P.bf16 = d->element == TB_ELEMENT_BF16;
    const int64_t count = d->node_count;
    P.nodes.reserve(count * 2);
    for (int64_t i = 0; i < count; ++i) {
      const tb_node& s = d->nodes[i];
      Node n;
      n.op = s.op;
      n.rank = s.rank;
      if (s.rank < 0 || s.rank > TB_MAX_RANK) fail("node rank out of range");
      if (s.op < 0 || s.op >= TB_OP_COUNT) fail("unknown opcode " + std::to_string(s.op));
      for (int k = 0; k < s.rank; ++k) {
        // the reference has no empty values (payload/tensor.rs rejects them)
        if (s.shape[k] < 1) fail("node " + std::to_string(i) + " has an empty extent");
        n.shape[k] = s.shape[k];
      }
      if ((s.op == TB_OP_PARAMETER || s.op == TB_OP_INPUT) && s.slot < 0)
        fail("node " + std::to_string(i) + " has no slot");
      for (int k = 0; k < TB_MAX_RANK; ++k) n.attrs[k] = s.attrs[k];
      n.operands[0] = s.operands[0];
      n.operands[1] = s.operands[1];
      n.slot = s.slot;
      n.payload = s.payload;
      n.constant = s.constant;
      n.vocab = s.vocab;
      n.dense = s.dense;
      n.indices = s.indices;
      n.wanted = s.wanted;
      n.readable = s.readable;
      for (int k = 0; k < 2; ++k)
        if (n.operands[k] >= i) fail("operand links must point backwards");
      P.nodes.push_back(n);
      P.info.emplace_back();
      if (n.op == TB_OP_PARAMETER) {
        P.parameter_slots = std::max(P.parameter_slots, n.slot + 1);
        if ((int)P.parameter_shapes.size() <= n.slot) P.parameter_shapes.resize(n.slot + 1);
        P.parameter_shapes[n.slot] = n.dims();
      }
      if (n.op == TB_OP_INPUT) P.input_slots = std::max(P.input_slots, n.slot + 1);
    }
    P.input_buffer.assign(P.input_slots, -1);
    P.input_node.assign(P.input_slots, -1);
    for (int64_t i = 0; i < count; ++i) {
      Node& n = P.nodes[i];
      for (int k = 0; k < 2; ++k)
        if (n.operands[k] >= 0) n.operands[k] = resolve(n.operands[k]);
      if (n.op == TB_OP_INPUT) P.input_node[n.slot] = (int)i;
      if (!n.wanted) continue;
      if (n.op == TB_OP_LOG_SUM_EXP || n.op == TB_OP_LOG_SOFTMAX) {
        expand_log_domain((int)i);
      } else {
        P.order.push_back((int)i);
      }
    }
    if (d->backward) append_backward(d);
  }

  // ---- engine-backward plans (`Run::backward`, engine/run.rs:229-318)
  // For every scalar readable root, the reverse scan is appended as nodes: a
  // `one_like` seed, the derivative rules of function/*.rs in the engine's
  // order, and per slot a zero-seeded accumulation `g = g + c` in reverse-scan
  // order.  The gradient of every parameter becomes a readable value.
  int grad_node(int op, int a, int b, std::vector<int64_t> shape,
                std::vector<int64_t> attrs = {}) {
    Node n;
    n.op = op;
    n.operands[0] = a;
    n.operands[1] = b;
    n.rank = (int)shape.size();
    if (n.rank > TB_MAX_RANK) fail("rank above the ABI maximum in a gradient");
    for (int i = 0; i < n.rank; ++i) n.shape[i] = shape[i];
    for (size_t i = 0; i < attrs.size(); ++i) n.attrs[i] = attrs[i];
    n.wanted = true;
    int id = add_node(n);
    P.order.push_back(id);
    return id;
  }
  std::vector<int64_t> dims(int n) const { return P.nodes[n].dims(); }
  int constant_like(int n, float c) {
    int id = grad_node(TB_OP_LEAF, -1, -1, dims(n));
    P.nodes[id].payload = TB_PAYLOAD_CONSTANT;
    P.nodes[id].constant = c;
    return id;
  }
  int ew(int op, int a, int b = -1) { return grad_node(op, a, b, dims(a)); }
  int swapped(int v) {
    std::vector<int64_t> s = dims(v);
    int r = (int)s.size();
    if (r <= 2) {
      std::reverse(s.begin(), s.end());
      return grad_node(TB_OP_TRANSPOSE, v, -1, s);
    }
    std::vector<int64_t> order(r);
    for (int i = 0; i < r; ++i) order[i] = i;
    std::swap(order[r - 2], order[r - 1]);
    std::swap(s[r - 2], s[r - 1]);
    return grad_node(TB_OP_PERMUTE, v, -1, s, order);
  }
  int matmul(int a, int b) {
    std::vector<int64_t> s = dims(a);
    s.back() = P.nodes[b].shape[P.nodes[b].rank - 1];
    return grad_node(TB_OP_MATMUL, a, b, s);
  }
  int sum_along(int x, int64_t axis) {
    std::vector<int64_t> s = dims(x);
    s.erase(s.begin() + axis);
    return grad_node(TB_OP_SUM_ALONG, x, -1, s, {axis});
  }
  int bcast_along(int x, int64_t axis, int like) {
    return grad_node(TB_OP_BROADCAST_ALONG, x, like, dims(like), {axis});
  }

  // The cotangents of node i (original indices) given output value `out`,
  // operand values `x`, `y` and gradient `g` (function/*.rs `backward`).
  void rule(const Node& nd, int x, int y, int out, int g, int& cx, int& cy) {
    const int64_t* at = nd.attrs;
    cx = cy = -1;
    switch (nd.op) {
      case TB_OP_ADD: cx = g; cy = g; return;
      case TB_OP_SUB: cx = g; cy = ew(TB_OP_NEG, g); return;
      case TB_OP_MUL: cx = ew(TB_OP_MUL, g, y); cy = ew(TB_OP_MUL, g, x); return;
      case TB_OP_DIV: {
        cx = ew(TB_OP_DIV, g, y);
        int go = ew(TB_OP_MUL, g, out);
        cy = ew(TB_OP_NEG, ew(TB_OP_DIV, go, y));
        return;
      }
      case TB_OP_NEG: cx = ew(TB_OP_NEG, g); return;
      case TB_OP_TANH: {
        int one = constant_like(out, 1.0f);
        int d = ew(TB_OP_SUB, one, ew(TB_OP_MUL, out, out));
        cx = ew(TB_OP_MUL, g, d);
        return;
      }
      case TB_OP_EXP: cx = ew(TB_OP_MUL, g, out); return;
      case TB_OP_LN: cx = ew(TB_OP_DIV, g, x); return;
      case TB_OP_SQRT: cx = ew(TB_OP_DIV, g, ew(TB_OP_ADD, out, out)); return;
      case TB_OP_POWF: {
        int lowered = ew(TB_OP_SUB, y, constant_like(y, 1.0f));
        int ge = ew(TB_OP_MUL, g, y);
        cx = ew(TB_OP_MUL, ge, ew(TB_OP_POWF, x, lowered));
        int go = ew(TB_OP_MUL, g, out);
        cy = ew(TB_OP_MUL, go, ew(TB_OP_LN, x));
        return;
      }
      case TB_OP_MAXIMUM: {
        int w = ew(TB_OP_STEP, x, y);
        cx = ew(TB_OP_MUL, g, w);
        cy = ew(TB_OP_MUL, g, ew(TB_OP_SUB, constant_like(w, 1.0f), w));
        return;
      }
      case TB_OP_RELU: {
        int z = constant_like(x, 0.0f);
        cx = ew(TB_OP_MUL, g, ew(TB_OP_STEP, x, z));
        return;
      }
      case TB_OP_STEP: return;
      case TB_OP_MATMUL:
        cx = matmul(g, swapped(y));
        cy = matmul(swapped(x), g);
        return;
      case TB_OP_TRANSPOSE: {
        std::vector<int64_t> s = dims(g);
        std::reverse(s.begin(), s.end());
        cx = grad_node(TB_OP_TRANSPOSE, g, -1, s);
        return;
      }
      case TB_OP_SUM: cx = grad_node(TB_OP_BROADCAST, g, x, dims(x)); return;
      case TB_OP_SUM_ALONG: cx = bcast_along(g, at[0], x); return;
      case TB_OP_BROADCAST: {
        int total = grad_node(TB_OP_SUM, g, -1, {});
        cx = grad_node(TB_OP_BROADCAST, total, x, dims(x));
        return;
      }
      case TB_OP_BROADCAST_ALONG: cx = sum_along(g, at[0]); return;
      case TB_OP_RESHAPE: cx = grad_node(TB_OP_RESHAPE, g, -1, dims(x)); return;
      case TB_OP_PERMUTE: {
        std::vector<int64_t> inv(nd.rank);
        for (int j = 0; j < nd.rank; ++j) inv[at[j]] = j;
        cx = grad_node(TB_OP_PERMUTE, g, -1, dims(x), inv);
        return;
      }
      case TB_OP_NARROW:
        cx = grad_node(TB_OP_PAD, g, -1, dims(x), {at[0], at[1], P.nodes[x].shape[at[0]]});
        return;
      case TB_OP_PAD:
        cx = grad_node(TB_OP_NARROW, g, -1, dims(x), {at[0], at[1], P.nodes[x].shape[at[0]]});
        return;
      case TB_OP_UNFOLD:
        cx = grad_node(TB_OP_FOLD, g, -1, dims(x),
                       {at[0], at[1], at[2], at[3], P.nodes[x].shape[at[0]]});
        return;
      case TB_OP_FOLD:
        cx = grad_node(TB_OP_UNFOLD, g, -1, dims(x), {at[0], at[1], at[2], at[3]});
        return;
      case TB_OP_GATHER:
        cx = grad_node(TB_OP_SCATTER, g, y, dims(x), {P.nodes[x].shape[0]});
        return;
      case TB_OP_SCATTER: {
        std::vector<int64_t> s = dims(x);
        cx = grad_node(TB_OP_GATHER, g, y, s);
        return;
      }
      case TB_OP_LOG_SOFTMAX: {
        int total = bcast_along(sum_along(g, at[0]), at[0], g);
        cx = ew(TB_OP_SUB, g, ew(TB_OP_MUL, ew(TB_OP_EXP, out), total));
        return;
      }
      case TB_OP_LOG_SUM_EXP: {
        int prob = ew(TB_OP_EXP, ew(TB_OP_SUB, x, bcast_along(out, at[0], x)));
        cx = ew(TB_OP_MUL, bcast_along(g, at[0], x), prob);
        return;
      }
    }
    fail("no derivative rule for op " + std::to_string(nd.op));
  }

  void append_backward(const tb_plan_desc* d) {
    const int count = (int)d->node_count;
    for (int root = 0; root < count; ++root) {
      const tb_node& r = d->nodes[root];
      if (!r.readable || !r.wanted || r.rank != 0) continue;
      std::vector<int> grad(root + 1, -1);
      std::vector<char> ancestor(root + 1, 0);
      grad[root] = constant_like(resolve(root), 1.0f);
      ancestor[root] = 1;
      for (int i = root; i >= 0; --i) {
        if (!ancestor[i]) continue;
        const tb_node& src = d->nodes[i];
        if (src.op == TB_OP_LEAF || src.op == TB_OP_PARAMETER || src.op == TB_OP_INPUT) continue;
        Node nd = P.nodes[i];  // attributes; operands below are the original links
        const int lx = src.operands[0], ly = src.operands[1];
        const int x = lx >= 0 ? resolve(lx) : -1, y = ly >= 0 ? resolve(ly) : -1;
        int cx, cy;
        rule(nd, x, y, resolve(i), grad[i], cx, cy);
        const int links[2] = {lx, ly};
        const int cots[2] = {cx, cy};
        for (int k = 0; k < 2; ++k) {
          if (links[k] < 0 || cots[k] < 0) continue;
          const int slot = links[k];
          ancestor[slot] = 1;
          const int seed = grad[slot] >= 0 ? grad[slot] : constant_like(resolve(slot), 0.0f);
          grad[slot] = ew(TB_OP_ADD, seed, cots[k]);
        }
      }
      for (int i = 0; i <= root; ++i) {
        if (d->nodes[i].op != TB_OP_PARAMETER) continue;
        int gn = grad[i] >= 0 ? grad[i] : constant_like(i, 0.0f);
        P.nodes[gn].readable = true;
        P.gradient_of[{root, i}] = gn;
      }
    }
  }

  // function/log_sum_exp.rs:53-63 and function/log_softmax.rs:51-65 as
  // primitive nodes: peak, shifted, exp, row sum, ln, and the combination.
  void expand_log_domain(int i) {
    Node src = P.nodes[i];
    int x = src.operands[0];
    int axis = (int)src.attrs[0];
    const Node xn = P.nodes[x];
    auto mk = [&](int op, int a, int b, const Node& shape_of, bool drop_axis) {
      Node n;
      n.op = op;
      n.operands[0] = a;
      n.operands[1] = b;
      n.wanted = true;
      n.attrs[0] = axis;
      n.rank = 0;
      for (int k = 0; k < shape_of.rank; ++k)
        if (!(drop_axis && k == axis)) n.shape[n.rank++] = shape_of.shape[k];
      int id = add_node(n);
      P.order.push_back(id);
      return id;
    };
    int peak = mk(TB_OP_MAX_ALONG, x, -1, xn, true);
    int peak_b = mk(TB_OP_BROADCAST_ALONG, peak, x, xn, false);
    int shifted = mk(TB_OP_SUB, x, peak_b, xn, false);
    int e = mk(TB_OP_EXP, shifted, -1, xn, false);
    int total = mk(TB_OP_SUM_ALONG, e, -1, xn, true);
    int normalizer = mk(TB_OP_LN, total, -1, P.nodes[total], false);
    int out;
    if (src.op == TB_OP_LOG_SUM_EXP) {
      out = mk(TB_OP_ADD, peak, normalizer, P.nodes[peak], false);
    } else {
      int nb = mk(TB_OP_BROADCAST_ALONG, normalizer, shifted, xn, false);
      out = mk(TB_OP_SUB, shifted, nb, xn, false);
    }
    P.nodes[out].readable = src.readable;
    P.info[i].alias = out;
  }

  // ---- pass 2: consumer counts
  void count_consumers() {
    for (int n : P.order) {
      const Node& nd = P.nodes[n];
      if (nd.op == TB_OP_LEAF || nd.op == TB_OP_PARAMETER || nd.op == TB_OP_INPUT) continue;
      int a = nd.operands[0], b = nd.operands[1];
      if (nd.op == TB_OP_BROADCAST || nd.op == TB_OP_BROADCAST_ALONG) b = -1;
      if (a >= 0) P.info[a].consumers++;
      if (b >= 0 && b != a) P.info[b].consumers++;
    }
  }

  bool source_layout(int n) const {
    const Node& nd = P.nodes[n];
    return nd.op == TB_OP_LEAF || nd.op == TB_OP_PARAMETER || nd.op == TB_OP_INPUT;
  }

  void materialize(int n) {
    Info& f = P.info[n];
    f.materialized = true;
    if (f.kind == Kind::None) f.kind = Kind::Expr;
    f.buf = new_buffer(Storage::Arena, P.nodes[n].volume() * 4, n);
    f.lay = contiguous(P.nodes[n]);
    f.owner = n;
    f.heavy.clear();
    f.ops = 0;
  }

  // ---- pass 3: kinds, constant folding, view folding, materialization
  void classify() {
    for (int n : P.order) {
      Node& nd = P.nodes[n];
      Info& f = P.info[n];
      const int a = nd.operands[0], b = nd.operands[1];
      switch (nd.op) {
        case TB_OP_LEAF:
          if (nd.payload == TB_PAYLOAD_CONSTANT) {
            f.kind = Kind::Const;
            f.c = P.bf16 ? round_bf16(nd.constant) : nd.constant;
          } else if (nd.payload == TB_PAYLOAD_SELECTION) {
            f.kind = Kind::Sel;
            f.one = P.bf16 ? round_bf16(nd.constant) : nd.constant;
            f.buf = new_buffer(Storage::LeafIndices, nd.shape[0] * 4, n);
          } else if (nd.payload == TB_PAYLOAD_DENSE) {
            f.kind = Kind::Layout;
            f.buf = new_buffer(Storage::Leaf, nd.volume() * 4, n);
            f.lay = contiguous(nd);
            f.owner = n;
          } else {
            fail("leaf without payload");
          }
          break;
        case TB_OP_PARAMETER:
          f.kind = Kind::Layout;
          f.buf = new_buffer(Storage::Parameter, nd.volume() * 4, n, nd.slot);
          f.lay = contiguous(nd);
          f.owner = n;
          break;
        case TB_OP_INPUT:
          if (nd.payload == TB_PAYLOAD_SELECTION) {
            f.kind = Kind::Sel;
            f.one = P.bf16 ? round_bf16(nd.constant) : nd.constant;
            f.buf = new_buffer(Storage::InputIndices, nd.shape[0] * 4, n, nd.slot);
          } else {
            f.kind = Kind::Layout;
            f.buf = new_buffer(Storage::Input, nd.volume() * 4, n, nd.slot);
            f.lay = contiguous(nd);
            f.owner = n;
          }
          P.input_buffer[nd.slot] = f.buf;
          break;
        default:
          classify_computed(n, a, b);
      }
      if (nd.readable && !f.materialized && f.kind != Kind::Sel && fold_seed(n)) continue;
      if (nd.readable && !f.materialized && f.kind != Kind::Sel) materialize(n);
    }
  }

  // Whether node y's value is accumulated from +0 by its kernel, so that it
  // never holds -0: a GEMM (its epilogue and split-K sum add +0 on the way
  // out), a scatter-add (segment sums from zero), and the sums that become
  // row, column or full reductions of a fused group (their accumulators start
  // at zero).  The serial REDUCE kernel seeds with the first element: not.
  bool accumulated_from_zero(int y) const {
    const Node& nd = P.nodes[y];
    if (nd.op == TB_OP_MATMUL || nd.op == TB_OP_SCATTER) return true;
    if (nd.op != TB_OP_SUM && nd.op != TB_OP_SUM_ALONG) return false;
    const Node& x = P.nodes[nd.operands[0]];
    if (nd.op == TB_OP_SUM) return x.rank > 0;
    const int axis = (int)nd.attrs[0];
    if (axis == x.rank - 1) return true;
    if (x.rank == 2 && axis == 0 && x.shape[0] > kSerialColumnRows) {
      int64_t T, KC;
      int vec;
      row_shape(x.dims(), T, KC, vec);
      return KC * vec <= 32 && x.shape[1] <= 8192;
    }
    return false;
  }

  // A readable gradient seed `0 + y` (Tape::differentiate's first
  // contribution, graph/tape.rs:389-393) over such a y that nothing else
  // reads is y's buffer itself: no copy kernel, and y's buffer is kept as
  // a readable value.
  bool fold_seed(int n) {
    const Node& nd = P.nodes[n];
    if (P.bf16 || nd.op != TB_OP_ADD) return false;
    int y = -1;
    for (int o = 0; o < 2; ++o) {
      const Info& c = P.info[nd.operands[o]];
      if (c.kind == Kind::Const && c.c == 0.0f && !std::signbit(c.c)) y = nd.operands[1 - o];
    }
    if (y < 0) return false;
    const Info& fy = P.info[y];
    if (!fy.materialized || fy.owner != y || P.nodes[y].readable || fy.consumers != 1 ||
        fy.seed_of >= 0 || !accumulated_from_zero(y) || P.nodes[y].volume() != nd.volume())
      return false;
    Info& f = P.info[n];
    f.kind = Kind::Layout;
    f.materialized = true;
    f.buf = fy.buf;
    f.lay = contiguous(nd);
    f.owner = y;
    f.seed_of = y;
    P.buffers[fy.buf].keep = true;
    return true;
  }

  void classify_computed(int n, int a, int b) {
    Node& nd = P.nodes[n];
    Info& f = P.info[n];
    const Info* fa = a >= 0 ? &P.info[a] : nullptr;
    const Info* fb = b >= 0 ? &P.info[b] : nullptr;
    if (is_elementwise(nd.op)) {
      bool binary = nd.op == TB_OP_ADD || nd.op == TB_OP_SUB || nd.op == TB_OP_MUL ||
                    nd.op == TB_OP_DIV || nd.op == TB_OP_POWF || nd.op == TB_OP_MAXIMUM ||
                    nd.op == TB_OP_STEP;
      if (fa->kind == Kind::Const && (!binary || fb->kind == Kind::Const)) {
        f.kind = Kind::Const;
        f.c = fold_scalar(nd.op, fa->c, binary ? fb->c : 0.0f);
        if (P.bf16) f.c = round_bf16(f.c);
        return;
      }
      expression(n);
      return;
    }
    if (is_view(nd.op)) {
      if (fa->kind == Kind::Const) {
        f.kind = Kind::Const;
        f.c = fa->c;
        return;
      }
      if (fa->kind == Kind::Layout || fa->materialized) {
        Layout l;
        if (view_layout(nd, P.nodes[a], fa->lay, l)) {
          f.kind = Kind::Layout;
          f.lay = l;
          f.buf = fa->buf;
          f.owner = fa->owner;
          return;
        }
      }
      expression(n);
      return;
    }
    switch (nd.op) {
      case TB_OP_PAD:
        expression(n);
        return;
      case TB_OP_GATHER:
        if (fb->kind != Kind::Sel) fail("gather needs a selection operand");
        if (fa->kind == Kind::Const) {
          f.kind = Kind::Const;
          f.c = fa->c;
          return;
        }
        expression(n);
        return;
      case TB_OP_SUM:
      case TB_OP_SUM_ALONG:
      case TB_OP_MAX_ALONG:
        if (fa->kind == Kind::Const) {
          // a serial left fold of identical values (payload/tensor.rs:1055-1124)
          int64_t extent = nd.op == TB_OP_SUM ? P.nodes[a].volume()
                                              : P.nodes[a].shape[nd.attrs[0]];
          float acc = fa->c;
          for (int64_t s = 1; s < extent; ++s)
            acc = nd.op == TB_OP_MAX_ALONG ? fmax_ref(acc, fa->c) : acc + fa->c;
          f.kind = Kind::Const;
          f.c = P.bf16 ? round_bf16(acc) : acc;  // f32 accumulation, one rounding
          return;
        }
        f.kind = Kind::Expr;
        materialize(n);
        return;
      case TB_OP_MATMUL:
      case TB_OP_SCATTER:
      case TB_OP_FOLD:
        if (nd.op == TB_OP_SCATTER && fb->kind != Kind::Sel) fail("scatter needs a selection operand");
        f.kind = Kind::Expr;
        materialize(n);
        return;
      default:
        fail("unsupported op " + std::to_string(nd.op));
    }
  }

  // A computed elementwise or index-mapping value: recomputed by each consumer
  // unless it is shared and reads several large buffers, or grows too large.
  void expression(int n) {
    Node& nd = P.nodes[n];
    Info& f = P.info[n];
    f.kind = Kind::Expr;
    f.ops = 1;
    std::vector<int> heavy;
    const int64_t vol = nd.volume();
    for (int k = 0; k < 2; ++k) {
      int o = nd.operands[k];
      if (o < 0) continue;
      if (nd.op == TB_OP_GATHER && k == 1) continue;
      if ((nd.op == TB_OP_BROADCAST || nd.op == TB_OP_BROADCAST_ALONG) && k == 1) continue;
      const Info& fo = P.info[o];
      // a buffer is heavy for this value when it holds at least as many
      // elements as the value: a per-row vector broadcast over a matrix is not
      if (fo.materialized || fo.kind == Kind::Layout) {
        if (P.buffers[fo.buf].bytes / 4 >= vol) heavy.push_back(fo.buf);
      } else if (fo.kind == Kind::Expr) {
        f.ops += fo.ops;
        for (int hb : fo.heavy)
          if (P.buffers[hb].bytes / 4 >= vol) heavy.push_back(hb);
      }
    }
    std::sort(heavy.begin(), heavy.end());
    heavy.erase(std::unique(heavy.begin(), heavy.end()), heavy.end());
    if (heavy.size() > 4) heavy.resize(4);
    f.heavy = heavy;
    if ((f.consumers >= 2 && heavy.size() >= 2) || f.ops > 40) materialize(n);
  }

  // ---- pass 4: fusion groups
  enum Ctx { ID = 0, ROWB = 1, OTHER = 2 };
  struct Group {
    std::vector<int64_t> space;
    std::vector<Member> members;
    std::map<int, int> index;  // node -> member position
    std::set<int> after;       // open groups that must be emitted first
    bool open = true;
  };
  std::vector<Group> groups;
  std::map<std::vector<int64_t>, int> open_group;
  std::vector<int> group_of;  // node -> group id
  // materialized node -> the groups that read it (-1: a kernel of its own)
  std::map<int, std::set<int>> readers;
  void read_by(const std::vector<std::pair<int, int>>& r, int g) {
    for (auto& nc : r) readers[nc.first].insert(g);
  }

  void walk(int n, int ctx, std::set<std::pair<int, int>>& seen,
            std::vector<std::pair<int, int>>& out, bool is_root) {
    if (!seen.insert({n, ctx}).second) return;
    const Info& f = P.info[n];
    if (!is_root) {
      if (f.materialized) {
        out.push_back({n, ctx});
        return;
      }
      if (f.kind == Kind::Const || f.kind == Kind::Sel) return;
      if (f.kind == Kind::Layout && source_layout(n)) return;
    }
    const Node& nd = P.nodes[n];
    if (source_layout(n)) return;
    if (is_elementwise(nd.op)) {
      for (int k = 0; k < 2; ++k)
        if (nd.operands[k] >= 0) walk(nd.operands[k], ctx, seen, out, false);
      return;
    }
    if (nd.op == TB_OP_BROADCAST_ALONG) {
      int c = (ctx == ID && nd.attrs[0] == nd.rank - 1) ? ROWB : OTHER;
      walk(nd.operands[0], c, seen, out, false);
      return;
    }
    if (nd.op == TB_OP_SUM || nd.op == TB_OP_SUM_ALONG || nd.op == TB_OP_MAX_ALONG) {
      walk(nd.operands[0], ID, seen, out, false);  // the reduction's input space
      return;
    }
    if (nd.op == TB_OP_GATHER) {
      walk(nd.operands[0], OTHER, seen, out, false);
      return;
    }
    for (int k = 0; k < 2; ++k) {
      if (nd.operands[k] < 0) continue;
      if ((nd.op == TB_OP_BROADCAST || nd.op == TB_OP_BROADCAST_ALONG) && k == 1) continue;
      walk(nd.operands[k], OTHER, seen, out, false);
    }
  }

  std::vector<std::pair<int, int>> refs(int n) {
    std::set<std::pair<int, int>> seen;
    std::vector<std::pair<int, int>> out;
    walk(n, ID, seen, out, true);
    return out;
  }

  // whether open group `b` must run after open group `a` (transitively)
  bool runs_after(int b, int a) {
    std::vector<int> stack{b};
    std::set<int> seen;
    while (!stack.empty()) {
      int x = stack.back();
      stack.pop_back();
      if (x == a) return true;
      if (!seen.insert(x).second) continue;
      for (int y : groups[x].after)
        if (groups[y].open) stack.push_back(y);
    }
    return false;
  }

  void flush(int g) {
    Group& G0 = groups[g];
    if (!G0.open) return;
    G0.open = false;
    std::set<int> deps = G0.after;
    for (int d : deps) flush(d);
    Group& G = groups[g];
    open_group.erase(G.space);
    Kernel k;
    bool reductions = false;
    for (auto& m : G.members)
      if (m.type != MemberType::EW && m.type != MemberType::PREP) reductions = true;
    k.type = reductions ? KType::ROW : KType::EW;
    k.members = G.members;
    k.space = G.space;
    k.group = g;
    P.kernels.push_back(k);
  }

  void flush_refs(const std::vector<std::pair<int, int>>& r) {
    for (auto& [node, ctx] : r) {
      int g = group_of[node];
      if (g >= 0 && groups[g].open) flush(g);
    }
  }

  int row_vec(const std::vector<int64_t>& space) const {
    if (space.empty()) return 1;
    return space.back() % 4 == 0 ? 4 : 1;
  }

  // threads per row and chunks per thread of a row-space kernel; col_members
  // column sums each keep KC * vec register accumulators per thread
  void row_shape(const std::vector<int64_t>& space, int64_t& T, int64_t& KC, int& vec,
                 int col_members = 0) const {
    int64_t L = space.empty() ? 1 : space.back();
    vec = row_vec(space);
    int64_t chunks = (L + vec - 1) / vec;
    T = 32;
    // rows of up to 16 chunks per lane: one warp per row (shuffle-only
    // reductions, many rows in flight); longer rows: up to 256 threads
    if (chunks > 32 * 16)
      while (T * 2 <= chunks && T < 256) T *= 2;
    // column sums: widen the team until the accumulators fit in 24 registers
    // (occupancy, not the cross-warp row reductions, bounds such kernels)
    while (col_members > 0 && T < 256 && T * 2 <= chunks &&
           ((chunks + T - 1) / T) * vec * col_members > 24)
      T *= 2;
    KC = (chunks + T - 1) / T;
  }

  // Places a member in the open group of `space` (or a new one) at the phase
  // its reads allow.  A PREP member reads exactly its node's value (refs of
  // the node itself, or the node when it is materialized) and is not
  // registered as the node's producer; returns the group.
  int group_member(int n, MemberType type, const std::vector<int64_t>& space, int hi = -1,
                   int lo = -1) {
    const bool prep = type == MemberType::PREP;
    std::vector<std::pair<int, int>> r;
    if (prep && P.info[n].materialized) r.push_back({n, ID});
    else r = refs(n);
    // Members of open groups read in a way the group cannot serve are flushed.
    auto it = open_group.find(space);
    int g = it == open_group.end() ? -1 : it->second;
    int phase = 0;
    bool conflict = false;
    std::set<int> before;
    for (auto& [node, ctx] : r) {
      int og = group_of[node];
      if (og < 0 || !groups[og].open) continue;
      if (og != g) {
        before.insert(og);
        continue;
      }
      const Member& m = groups[g].members[groups[g].index[node]];
      if (ctx == ID && m.type == MemberType::EW) {
        phase = std::max(phase, m.phase);
      } else if (ctx == ROWB && (m.type == MemberType::ROW_SUM || m.type == MemberType::ROW_MAX)) {
        phase = std::max(phase, m.phase + 1);
      } else {
        conflict = true;
      }
    }
    if (g >= 0 && (conflict || groups[g].members.size() >= 48 || phase > 6)) {
      flush(g);
      g = -1;
      phase = 0;
    }
    // groups this member reads must run first; if one of them already has to
    // run after this member's group, that group is closed and a new one opens
    for (int og : before) {
      if (g >= 0 && groups[og].open && runs_after(og, g)) {
        flush(og);
        g = -1;
        phase = 0;
      }
    }
    if (g < 0) {
      Group G;
      G.space = space;
      groups.push_back(G);
      g = (int)groups.size() - 1;
      open_group[space] = g;
    }
    for (int og : before)
      if (groups[og].open && og != g) groups[g].after.insert(og);
    read_by(r, g);
    Member m{n, type, phase, hi, lo};
    if (!prep) {
      groups[g].index[n] = (int)groups[g].members.size();
      group_of[n] = g;
    }
    groups[g].members.push_back(m);
    return g;
  }

  void own_kernel(int n, KType type) {
    auto r = refs(n);
    read_by(r, -1);
    flush_refs(r);
    Kernel k;
    k.type = type;
    k.node = n;
    k.members.push_back(Member{n, MemberType::EW, 0});
    P.kernels.push_back(k);
  }

  void group_all() {
    group_of.assign(P.nodes.size(), -1);
    for (int n : P.order) {
      const Node& nd = P.nodes[n];
      const Info& f = P.info[n];
      if (!f.materialized || f.owner != n) continue;
      if (source_layout(n) && !nd.readable) continue;
      switch (nd.op) {
        case TB_OP_MATMUL: {
          // operands that open fusion groups compute get their tf32 pair from
          // those groups, before the operands' groups are closed below
          {
            const Node& A = P.nodes[nd.operands[0]];
            int64_t batch = 1;
            for (int i = 0; i < A.rank - 2; ++i) batch *= A.shape[i];
            for (int o = 0; o < 2; ++o) {
              bool flip = false;
              const int base = strip_transposes(nd.operands[o], flip);
              if (!prepared.count(base) && !raw_base.count(base) && fusable_prep(base))
                prepare(base, batch);
            }
          }
          // the GEMM reads only tf32 pairs; what a pair is made from is read by
          // the group or the prep kernel that writes it
          auto r = refs(n);
          flush_refs(r);
          matmul_kernels(n);
          break;
        }
        case TB_OP_SCATTER: {
          auto r = refs(n);
          read_by(r, -1);
          flush_refs(r);
          int sel = nd.operands[1];
          if (!P.sort_of.count(sel)) {
            Kernel s;
            s.type = KType::SORT;
            s.sel = sel;
            P.kernels.push_back(s);
            P.sort_of[sel] = (int)P.kernels.size() - 1;
          }
          own_kernel(n, KType::SCATTER);
          break;
        }
        case TB_OP_FOLD:
          own_kernel(n, KType::FOLD);
          break;
        case TB_OP_SUM:
        case TB_OP_SUM_ALONG:
        case TB_OP_MAX_ALONG: {
          const Node& x = P.nodes[nd.operands[0]];
          std::vector<int64_t> space = x.dims();
          bool max = nd.op == TB_OP_MAX_ALONG;
          if (nd.op == TB_OP_SUM) {
            if (x.rank == 0) {
              group_member(n, MemberType::EW, nd.dims());
            } else {
              group_member(n, MemberType::ALL_SUM, space);
            }
            break;
          }
          int axis = (int)nd.attrs[0];
          if (axis == x.rank - 1) {
            group_member(n, max ? MemberType::ROW_MAX : MemberType::ROW_SUM, space);
            break;
          }
          // A column sum over a short batch (batch-norm statistics over a
          // mini-batch, a small batch's bias gradients) is one serial fold
          // per column from the first row: the reference's own order, so
          // bit-identical, and no partials or final.
          if (!max && x.rank == 2 && axis == 0 && x.shape[0] > kSerialColumnRows) {
            int64_t T, KC;
            int vec;
            row_shape(space, T, KC, vec);
            if (KC * vec <= 32 && space[1] <= 8192) {
              group_member(n, MemberType::COL_SUM, space);
              break;
            }
          }
          own_kernel(n, KType::REDUCE);
          break;
        }
        default:
          group_member(n, MemberType::EW, nd.dims());
      }
    }
    for (size_t g = 0; g < groups.size(); ++g) flush((int)g);
    mark_register_members();
  }

  // An EW member of a row kernel read by no other kernel, not readable and
  // not a view's storage, can stay in registers across the kernel's phases.
  void mark_register_members() {
    std::set<int> viewed;  // buffers other values are views of
    for (size_t i = 0; i < P.nodes.size(); ++i) {
      const Info& f = P.info[i];
      if (f.kind == Kind::Layout && f.owner >= 0 && f.owner != (int)i) viewed.insert(f.owner);
    }
    for (Kernel& K : P.kernels) {
      if (K.type != KType::ROW || K.group < 0) continue;
      for (Member& m : K.members) {
        if (m.type != MemberType::EW || P.nodes[m.node].readable || viewed.count(m.node)) continue;
        if (P.info[m.node].owner != m.node) continue;
        auto it = readers.find(m.node);
        bool only_here = true;
        if (it != readers.end())
          for (int g : it->second)
            if (g != K.group) only_here = false;
        m.reg = only_here;
      }
    }
  }

  // A value prepared for the tensor cores: its tf32 hi/lo pairs in the value's
  // own row-major layout [batch][rows][cols rounded up to 32].  A GEMM reads it
  // K-major when the value is its operand as is, MN-major when the operand is
  // the value's transpose -- so a product and the weight gradient that reads
  // the same activation transposed share one prep.
  struct Prepared {
    int hi = -1, lo = -1;
    int64_t rows = 0, cols = 0, ld = 0;
  };
  std::map<int, Prepared> prepared;

  // The value under any transposes of the last two axes (TRANSPOSE, or a
  // PERMUTE that swaps only those); `flip` is set when their count is odd.
  int strip_transposes(int x, bool& flip) {
    flip = false;
    for (;;) {
      const Node& nd = P.nodes[x];
      bool swap = nd.op == TB_OP_TRANSPOSE && nd.rank == 2;
      if (nd.op == TB_OP_PERMUTE && nd.rank >= 2) {
        swap = nd.attrs[nd.rank - 2] == nd.rank - 1 && nd.attrs[nd.rank - 1] == nd.rank - 2;
        for (int i = 0; i < nd.rank - 2; ++i)
          if (nd.attrs[i] != i) swap = false;
      }
      if (!swap) return x;
      flip = !flip;
      x = nd.operands[0];
    }
  }

  // Whether a value's prep can ride in the fusion group that computes it: an
  // expression (virtual, or a member of a still open group of its own shape)
  // whose last axis needs no padding.
  bool fusable_prep(int base) const {
    const Node& b = P.nodes[base];
    const Info& f = P.info[base];
    if (b.rank < 2 || b.shape[b.rank - 1] % 32 != 0 || f.kind != Kind::Expr) return false;
    if (!f.materialized) return true;
    const int g = group_of[base];
    return g >= 0 && groups[g].open && groups[g].space == b.dims() &&
           groups[g].members[groups[g].index.at(base)].type == MemberType::EW;
  }

  Prepared prepare(int base, int64_t batch) {
    auto it = prepared.find(base);
    if (it != prepared.end()) return it->second;
    const Node& b = P.nodes[base];
    Prepared r;
    r.rows = b.shape[b.rank - 2];
    r.cols = b.shape[b.rank - 1];
    r.ld = (r.cols + 31) / 32 * 32;
    if (raw_base.count(base)) {
      // the GEMM reads the stored f32 values (no lo) and splits them itself
      r.hi = P.info[base].buf;
      readers[base].insert(-1);
      prepared[base] = r;
      return r;
    }
    r.hi = new_buffer(Storage::Arena, batch * r.rows * r.ld * 4, -1);
    r.lo = new_buffer(Storage::Arena, batch * r.rows * r.ld * 4, -1);
    if (fusable_prep(base)) {
      // the group that computes the value also writes its tf32 pair; it is
      // closed now, before the GEMM that reads the pair
      const int g = group_member(base, MemberType::PREP, b.dims(), r.hi, r.lo);
      flush(g);
      prepared[base] = r;
      return r;
    }
    if (P.info[base].materialized) readers[base].insert(-1);
    else read_by(refs(base), -1);
    Kernel k;
    k.type = KType::PREP;
    k.node = base;
    k.batch = batch;
    k.m = r.rows;
    k.k = r.cols;
    k.kp = r.ld;
    k.a_hi = r.hi;
    k.a_lo = r.lo;
    P.kernels.push_back(k);
    prepared[base] = r;
    return r;
  }

  void matmul_kernels(int n) {
    const Node& nd = P.nodes[n];
    const Node& A = P.nodes[nd.operands[0]];
    const Node& B = P.nodes[nd.operands[1]];
    int split = A.rank - 2;
    int64_t batch = 1;
    for (int i = 0; i < split; ++i) batch *= A.shape[i];
    int64_t M = A.shape[split], K = A.shape[split + 1], N = B.shape[split + 1];
    bool fa = false, fb = false;
    const int base_a = strip_transposes(nd.operands[0], fa);
    const int base_b = strip_transposes(nd.operands[1], fb);
    const Prepared pa = prepare(base_a, batch);
    const Prepared pb = prepare(base_b, batch);
    Kernel g;
    g.type = KType::GEMM;
    g.node = n;
    g.batch = batch;
    g.m = M;
    g.n = N;
    g.k = K;
    g.kp = (K + 31) / 32 * 32;
    // A (M x K) is its base as is ([M, K]: K-major) or transposed ([K, M]:
    // MN-major); B (K x N) as is is [K, N]: MN-major for the N x K convention.
    g.a_hi = pa.hi;
    g.a_lo = pa.lo;
    g.a_mn = fa ? 1 : 0;
    g.a_ld = pa.ld;
    g.a_rows = pa.rows;
    g.b_hi = pb.hi;
    g.b_lo = pb.lo;
    g.b_mn = fb ? 0 : 1;
    g.b_ld = pb.ld;
    g.b_rows = pb.rows;
    g.out = P.info[n].buf;
    g.exact = false;
    g.passes = gemm_splits(batch, M, N, g.kp);  // split-K factor
    if (g.passes > 1) g.partial = new_buffer(Storage::Arena, g.passes * batch * M * N * 4, -1);
    P.kernels.push_back(g);
    P.gemms++;
  }

  // ---- raw GEMM operands
  // A value every product reads as its A operand and as a memory-bound one --
  // the product is at most 64 wide, so each element meets at most 64 others
  // -- is stored once in f32 and split into its tf32 pair inside the GEMM:
  // half the bytes of a prepared pair are written and read.  The value
  // must be a dense [batch][rows][cols] buffer with cols a multiple of 32 (no
  // padding, 16-byte rows); an expression that is not yet stored is
  // materialized for it.  Products wide enough to be bound by the tensor cores
  // keep prepared pairs.  A bf16 network keeps them too: its prep kernels
  // round what they load to bf16 (a GEMM's f32 result included), which a raw
  // operand read by the GEMM itself would skip.
  std::set<int> raw_base;
  static constexpr int64_t kRawOperandReuse = 64;

  bool dense_view(int n) const {
    const Info& f = P.info[n];
    const Node& nd = P.nodes[n];
    if (f.kind == Kind::Expr && !f.materialized) return true;  // materialized below
    if (!(f.kind == Kind::Layout || (f.kind == Kind::Expr && f.materialized)) || f.buf < 0)
      return false;
    if (f.lay.offset != 0 || f.lay.rank != nd.rank) return false;
    int64_t s = 1;
    for (int i = nd.rank - 1; i >= 0; --i) {
      if (nd.shape[i] != 1 && f.lay.stride[i] != s) return false;
      s *= nd.shape[i];
    }
    return P.buffers[f.buf].bytes >= nd.volume() * 4;
  }

  void choose_raw_operands() {
    if (P.bf16) return;
    if (const char* e = getenv("TB_RAW_OPERANDS"))
      if (atoi(e) == 0) return;
    std::map<int, bool> ok;
    for (int n : P.order) {
      const Node& nd = P.nodes[n];
      const Info& f = P.info[n];
      if (nd.op != TB_OP_MATMUL || !f.materialized || f.owner != n) continue;
      const Node& A = P.nodes[nd.operands[0]];
      const Node& B = P.nodes[nd.operands[1]];
      const int split = A.rank - 2;
      int64_t batch = 1;
      for (int i = 0; i < split; ++i) batch *= A.shape[i];
      const int64_t N = B.shape[split + 1];
      for (int o = 0; o < 2; ++o) {
        bool flip = false;
        const int base = strip_transposes(nd.operands[o], flip);
        const Node& b = P.nodes[base];
        bool fit = o == 0 && N <= kRawOperandReuse && b.rank >= 2 &&
                   b.shape[b.rank - 1] % 32 == 0 && b.volume() == batch * b.shape[b.rank - 2] *
                   b.shape[b.rank - 1] && dense_view(base);
        auto it = ok.find(base);
        ok[base] = (it == ok.end() ? true : it->second) && fit;
      }
    }
    for (auto& [base, fit] : ok) {
      if (!fit) continue;
      const Info& f = P.info[base];
      if (f.kind == Kind::Expr && !f.materialized) materialize(base);
      raw_base.insert(base);
    }
  }

  void run(const tb_plan_desc* d) {
    load(d);
    count_consumers();
    classify();
    choose_raw_operands();
    group_all();
  }
};

// ============================================================== codegen
class Emitter {
 public:
  Program& P;
  Kernel& K;
  int kid;
  std::ostringstream body;
  std::vector<std::unordered_map<std::string, std::string>> memo;
  std::map<int, int> param_of;   // buffer -> parameter position
  std::map<int, int> member_of;  // node -> member index (current kernel)
  std::set<int> in_registers;    // member indices held in `kr<m>[kc * vec + lane]`
  int phase = 0;
  int tmp = 0;
  int indent = 2;
  bool exact = true;
  // Set for a kernel already known to carry a tolerance (a transcendental or a
  // reassociated reduction): its divisions multiply by tb_rcp (about 2 ulp instead of
  // correctly rounded) and `0 + x` gradient seeds are dropped (they differ
  // from x only in the sign of a zero).  Exact kernels never set it.
  bool relaxed = false;
  // Values that already carry a tolerance: results of transcendentals, row
  // reductions, and anything computed from them.  A kernel whose every member
  // is such a value (or a reduction) may be emitted relaxed: no exact output
  // can observe the relaxation.
  std::set<std::string> tainted;
  std::set<int> tainted_members;
  bool exact_member_seen = false;
  bool is_tainted(const std::string& v) const { return tainted.count(v) || v.rfind("rv", 0) == 0; }
  void note_member_value(const std::string& v) {
    if (!is_tainted(v)) exact_member_seen = true;
  }
  bool wide = false;             // 64-bit indices
  int vec = 1;

  Emitter(Program& p, Kernel& k, int id) : P(p), K(k), kid(id) {
    memo.emplace_back();
    for (size_t i = 0; i < K.members.size(); ++i)
      if (K.members[i].type != MemberType::PREP) member_of[K.members[i].node] = (int)i;
  }

  // a bf16 network holds bf16 values: a loaded value (a source, or a
  // library kernel's f32 accumulation) and each operation's result round once;
  // rounding is idempotent, so values already rounded pass unchanged
  // Variables known never to hold -0 (results of a sum with a +0 literal), and
  // the operand of each emitted negation.
  std::set<std::string> no_negative_zero;
  std::map<std::string, std::string> negation_of;
  bool never_negative_zero(const std::string& v) const {
    if (no_negative_zero.count(v)) return true;
    // a literal other than -0
    return v.rfind("__int_as_float(0x", 0) == 0 && v != flit(-0.0f);
  }

  std::string rounded(const std::string& v) {
    if (!P.bf16) return v;
    const std::string k = "rb|" + v;
    if (const std::string* hit = find(k)) return *hit;
    std::string r = var("b");
    line("const float " + r + " = tb_rb(" + v + ");");
    memo.back()[k] = r;
    return r;
  }

  std::string pad() const { return std::string(indent, ' '); }
  void line(const std::string& s) { body << pad() << s << "\n"; }
  std::string var(const char* p = "v") { return std::string(p) + std::to_string(tmp++); }

  int param(int buf) {
    auto it = param_of.find(buf);
    if (it != param_of.end()) return it->second;
    int k = (int)K.params.size();
    K.params.push_back(buf);
    param_of[buf] = k;
    return k;
  }
  std::string fptr(int buf) { return "((float*)prm.p[" + std::to_string(param(buf)) + "])"; }
  std::string iptr(int buf) { return "((const int*)prm.p[" + std::to_string(param(buf)) + "])"; }

  const std::string* find(const std::string& key) const {
    for (auto it = memo.rbegin(); it != memo.rend(); ++it) {
      auto f = it->find(key);
      if (f != it->end()) return &f->second;
    }
    return nullptr;
  }
  void push() { memo.emplace_back(); }
  void pop() { memo.pop_back(); }

  static std::string key(int n, const Idx& idx) {
    std::string k = std::to_string(n) + "@";
    for (auto& c : idx.c) k += c + ",";
    return k;
  }

  std::string load(int buf, const Layout& lay, const Idx& idx) {
    if ((int)idx.c.size() != lay.rank) fail("index rank mismatch in load");
    bool aligned = lay.offset % 4 == 0;
    for (int d = 0; d + 1 < lay.rank; ++d)
      if (lay.stride[d] % 4 != 0) aligned = false;
    if (idx.lane >= 0 && vec == 4 && lay.rank > 0 && lay.stride[lay.rank - 1] == 1 && aligned) {
      std::string off = lit(lay.offset);
      for (int d = 0; d < lay.rank; ++d) {
        const std::string& c = d == lay.rank - 1 ? idx.lbase : idx.c[d];
        off = s_add(off, s_mul(c, lay.stride[d]));
      }
      std::string k = "vec|" + std::to_string(buf) + "|" + off;
      const std::string* hit = find(k);
      std::string v;
      if (hit) {
        v = *hit;
      } else {
        v = var("q");
        line("const float4 " + v + " = *(const float4*)(" + fptr(buf) + " + " + off + ");");
        memo.back()[k] = v;
      }
      static const char* comp[4] = {".x", ".y", ".z", ".w"};
      return v + comp[idx.lane];
    }
    std::string off = lit(lay.offset);
    for (int d = 0; d < lay.rank; ++d) off = s_add(off, s_mul(idx.c[d], lay.stride[d]));
    std::string k = "ld|" + std::to_string(buf) + "|" + off;
    const std::string* hit = find(k);
    if (hit) return *hit;
    std::string v = var();
    line("const float " + v + " = " + fptr(buf) + "[" + off + "];");
    memo.back()[k] = v;
    return v;
  }

  // The value of node n at idx, as seen by a consumer.
  std::string ref(int n, const Idx& idx) {
    const Info& f = P.info[n];
    if (f.kind == Kind::Const && !f.materialized) return flit(f.c);
    std::string k = key(n, idx);
    if (const std::string* hit = find(k)) return *hit;
    auto mit = member_of.find(n);
    if (mit != member_of.end()) {
      const Member& m = K.members[mit->second];
      if ((m.type == MemberType::ROW_SUM || m.type == MemberType::ROW_MAX) && m.phase < phase)
        return "rv" + std::to_string(mit->second);
      if (in_registers.count(mit->second) && m.phase < phase) {
        const std::string r = "kr" + std::to_string(mit->second) + "[kc * " +
                              std::to_string(vec) + " + " +
                              std::to_string(idx.lane >= 0 ? idx.lane : 0) + "]";
        if (tainted_members.count(mit->second)) tainted.insert(r);
        return r;
      }
    }
    if (f.kind == Kind::Sel && !f.materialized) {
      std::string v = var();
      line("const float " + v + " = (" + iptr(f.buf) + "[" + idx.c[0] + "] == (int)(" + idx.c[1] +
           ")) ? " + flit(f.one) + " : 0.0f;");
      memo.back()[k] = v;
      return v;
    }
    if (f.kind == Kind::Layout && !f.materialized && f.owner >= 0 && f.owner != n &&
        member_of.count(f.owner)) {
      // a view of a value this kernel computes: follow the view to the value
      // (registers or this thread's own stores), never the half-written buffer
      std::string v = def(n, idx);
      memo.back()[k] = v;
      return v;
    }
    if (f.materialized || f.kind == Kind::Layout) {
      std::string v = rounded(load(f.buf, f.lay, idx));
      // a stored value that an earlier kernel computed with a tolerance
      // carries it into this kernel too
      if (P.tolerance_nodes.count(n) || (f.owner >= 0 && P.tolerance_nodes.count(f.owner)))
        tainted.insert(v);
      return v;
    }
    std::string v = def(n, idx);
    memo.back()[k] = v;
    return v;
  }

  Idx keep_lane(const Idx& from, std::vector<std::string> c) {
    Idx r;
    r.c = std::move(c);
    if (from.lane >= 0 && !r.c.empty() && !from.c.empty() && r.c.back() == from.c.back()) {
      r.lane = from.lane;
      r.lbase = from.lbase;
    }
    return r;
  }

  // The defining computation of node n at idx.
  std::string def(int n, const Idx& idx) {
    const Node& nd = P.nodes[n];
    const int64_t* at = nd.attrs;
    const int a = nd.operands[0], b = nd.operands[1];
    if (P.info[n].kind == Kind::Const) return flit(P.info[n].c);
    if (nd.op == TB_OP_LEAF || nd.op == TB_OP_PARAMETER || nd.op == TB_OP_INPUT) {
      const Info& f = P.info[n];
      if (f.kind == Kind::Sel) {
        std::string v = var();
        line("const float " + v + " = (" + iptr(f.buf) + "[" + idx.c[0] + "] == (int)(" +
             idx.c[1] + ")) ? " + flit(f.one) + " : 0.0f;");
        return v;
      }
      // readable source: its original layout over its own storage
      Layout l = contiguous(nd);
      int src = -1;
      for (size_t i = 0; i < P.buffers.size(); ++i)
        if (P.buffers[i].node == n && P.buffers[i].storage != Storage::Arena) src = (int)i;
      return rounded(load(src, l, idx));
    }
    if (is_elementwise(nd.op)) {
      std::string x = ref(a, idx);
      std::string y = b >= 0 ? ref(b, idx) : "";
      // Exact identities (f32 only): 1*y is y; 0+y is y when y is never -0
      // (the sum of anything and +0 is never -0, so only the first of a chain
      // of `0 + ...` seeds is kept); -(-y) is y.
      if (!P.bf16 && relaxed && nd.op == TB_OP_ADD && (x == flit(0.0f) || y == flit(0.0f)))
        return x == flit(0.0f) ? y : x;
      if (!P.bf16) {
        const std::string one = flit(1.0f), zero = flit(0.0f);
        if (nd.op == TB_OP_MUL && (x == one || y == one)) return x == one ? y : x;
        if (nd.op == TB_OP_ADD && ((x == zero && never_negative_zero(y)) ||
                                   (y == zero && never_negative_zero(x))))
          return x == zero ? y : x;
        if (nd.op == TB_OP_NEG) {
          auto it = negation_of.find(x);
          if (it != negation_of.end()) return it->second;
        }
      }
      std::string e;
      switch (nd.op) {
        case TB_OP_ADD: e = "__fadd_rn(" + x + ", " + y + ")"; break;
        case TB_OP_SUB: e = "__fsub_rn(" + x + ", " + y + ")"; break;
        case TB_OP_MUL: e = "__fmul_rn(" + x + ", " + y + ")"; break;
        case TB_OP_DIV: {
          float c = 0.0f, r = 0.0f;
          if (literal_value(y, c) && exact_reciprocal(c, r))
            e = "__fmul_rn(" + x + ", " + flit(r) + ")";  // a power-of-two divisor
          else if (x == flit(1.0f) && relaxed && !P.bf16)
            e = "tb_rcp(" + y + ")";  // 1 * r is r
          else
            e = relaxed && !P.bf16 ? "__fmul_rn(" + x + ", tb_rcp(" + y + "))"
                                   : "__fdiv_rn(" + x + ", " + y + ")";
          break;
        }
        case TB_OP_NEG: e = "(-" + x + ")"; break;
        case TB_OP_TANH: e = "tanhf(" + x + ")"; break;
        case TB_OP_EXP: e = "expf(" + x + ")"; break;
        case TB_OP_LN: e = "logf(" + x + ")"; break;
        case TB_OP_SQRT: e = "__fsqrt_rn(" + x + ")"; break;
        case TB_OP_POWF: e = "powf(" + x + ", " + y + ")"; break;
        case TB_OP_MAXIMUM: e = "tb_max(" + x + ", " + y + ")"; break;
        case TB_OP_RELU: e = "tb_max(" + x + ", 0.0f)"; break;
        case TB_OP_STEP: e = "((" + x + " >= " + y + ") ? 1.0f : 0.0f)"; break;
      }
      if (is_transcendental(nd.op)) exact = false;
      std::string v = var();
      if (is_transcendental(nd.op) || is_tainted(x) || (!y.empty() && is_tainted(y)))
        tainted.insert(v);
      line("const float " + v + " = " + (P.bf16 ? "tb_rb(" + e + ")" : e) + ";");
      if (!P.bf16) {
        if (nd.op == TB_OP_ADD && (x == flit(0.0f) || y == flit(0.0f))) no_negative_zero.insert(v);
        if (nd.op == TB_OP_NEG) negation_of[v] = x;
      }
      return v;
    }
    const Node& on = P.nodes[a >= 0 ? a : n];
    std::vector<std::string> c;
    switch (nd.op) {
      case TB_OP_TRANSPOSE:
        c = idx.c;
        if (nd.rank == 2) std::swap(c[0], c[1]);
        return ref(a, keep_lane(idx, c));
      case TB_OP_PERMUTE:
        c.assign(nd.rank, "0");
        for (int j = 0; j < nd.rank; ++j) c[at[j]] = idx.c[j];
        return ref(a, keep_lane(idx, c));
      case TB_OP_NARROW:
        c = idx.c;
        c[at[0]] = s_add(c[at[0]], lit(at[1]));
        return ref(a, keep_lane(idx, c));
      case TB_OP_BROADCAST_ALONG:
        for (int j = 0; j < nd.rank; ++j)
          if (j != at[0]) c.push_back(idx.c[j]);
        return ref(a, keep_lane(idx, c));
      case TB_OP_BROADCAST:
        c.assign(on.rank, "0");
        return ref(a, keep_lane(idx, c));
      case TB_OP_RESHAPE: {
        std::string lin = "0";
        int64_t s = 1;
        for (int j = nd.rank - 1; j >= 0; --j) {
          lin = s_add(s_mul(idx.c[j], s), lin);
          s *= nd.shape[j];
        }
        // align trailing equal extents directly
        c.assign(on.rank, "");
        int64_t st = 1;
        for (int j = on.rank - 1; j >= 0; --j) {
          std::string q = s_div(lin, st);
          c[j] = j == 0 ? q : s_mod(q, on.shape[j]);
          st *= on.shape[j];
        }
        // equal trailing extents: the last index passes through unchanged
        if (on.rank > 0 && nd.rank > 0 && on.shape[on.rank - 1] == nd.shape[nd.rank - 1])
          c[on.rank - 1] = idx.c[nd.rank - 1];
        return ref(a, keep_lane(idx, c));
      }
      case TB_OP_UNFOLD: {
        int axis = (int)at[0];
        for (int j = 0; j < nd.rank; ++j) {
          if (j == axis) {
            c.push_back(s_add(s_mul(idx.c[j], at[2]), s_mul(idx.c[j + 1], at[3])));
          } else if (j == axis + 1) {
            continue;
          } else {
            c.push_back(idx.c[j]);
          }
        }
        return ref(a, keep_lane(idx, c));
      }
      case TB_OP_PAD: {
        int axis = (int)at[0];
        int64_t start = at[1], len = on.shape[axis];
        std::string v = var();
        line("float " + v + " = 0.0f;");
        line("if (" + idx.c[axis] + " >= " + lit(start) + " && " + idx.c[axis] + " < " +
             lit(start + len) + ") {");
        indent += 2;
        push();
        c = idx.c;
        c[axis] = s_add(c[axis], lit(-start));
        std::string x = ref(a, keep_lane(idx, c));
        line(v + " = " + x + ";");
        pop();
        indent -= 2;
        line("}");
        return v;
      }
      case TB_OP_SUM:
        if (on.rank == 0) return ref(a, idx);  // the sum of one element is itself
        break;
      case TB_OP_GATHER: {
        const Info& s = P.info[b];
        std::string r = var("r");
        line("const I " + r + " = (I)" + iptr(s.buf) + "[" + idx.c[0] + "];");
        c = idx.c;
        c[0] = r;
        return ref(a, keep_lane(idx, c));
      }
    }
    fail("codegen: node " + std::to_string(n) + " op " + std::to_string(nd.op) +
         " must be materialized");
  }

  // unravel a linear index string into shape components
  std::vector<std::string> unravel(const std::string& lin, const std::vector<int64_t>& shape,
                                   const std::string& prefix) {
    std::vector<std::string> c(shape.size());
    std::string rest = lin;
    for (int j = (int)shape.size() - 1; j >= 0; --j) {
      std::string name = prefix + std::to_string(j);
      if (j == 0) {
        line("const I " + name + " = " + rest + ";");
      } else {
        line("const I " + name + " = " + s_mod(rest, shape[j]) + ";");
        std::string r2 = var("u");
        line("const I " + r2 + " = " + s_div(rest, shape[j]) + ";");
        rest = r2;
      }
      c[j] = name;
    }
    return c;
  }
};

namespace {

std::string prelude() {
  return R"(
#define TB_INF __int_as_float(0x7f800000)
__device__ __forceinline__ float tb_max(float a, float b) {
  if (isnan(a)) return b;
  if (isnan(b)) return a;
  return (b > a) ? b : a;
}
// Online log-sum-exp state (m = running max, s = sum of exp(x - m)).  Branch
// free, so a row loop's loads are not held behind a divergent branch: one
// e = exp(-|x - m|) serves both cases -- a new maximum rescales the sum by
// exp(m - x) and adds 1, otherwise exp(x - m) is added (nothing for -inf);
// s * 1 is exact, so the result equals the branching form bit for bit.
__device__ __forceinline__ void tb_lse_push(float& m, float& s, float x) {
  const bool up = x > m;
  const float e = expf(-fabsf(x - m));
  const float scale = up ? e : 1.0f;
  const float add = up ? 1.0f : (x != -TB_INF ? e : 0.0f);
  s = s * scale + add;
  m = up ? x : m;
}
__device__ __forceinline__ void tb_lse_merge(float& m, float& s, float m2, float s2) {
  if (s2 == 0.0f && m2 == -TB_INF) return;
  if (s == 0.0f && m == -TB_INF) { m = m2; s = s2; return; }
  if (m2 > m) { s = s * expf(m - m2) + s2; m = m2; }
  else s = s + s2 * expf(m2 - m);
}
// 1 / y for kernels that carry a tolerance: the hardware reciprocal estimate
// with one Newton-Raphson correction (the residual 1 - y*r taken exactly by an
// FMA), within about 1 ulp of the correctly rounded reciprocal.  Such kernels
// divide as x * tb_rcp(y) (within about 2 ulp of x / y): a divisor shared by
// a row's elements then costs one reciprocal per row, not one per element.
// Zero, infinite and NaN operands take the estimate, whose special values are
// already IEEE's.
__device__ __forceinline__ float tb_rcp(float y) {
  float r;
  asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(y));
  const float e = __fmaf_rn(-y, r, 1.0f);
  return isfinite(e) ? __fmaf_rn(e, r, r) : r;
}
__device__ __forceinline__ float tb_tf32(float x) {
  unsigned r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
// the nearest bf16 as an f32 (ties to even; a NaN keeps its top half with a
// mantissa bit forced on): a bf16 network's rounding of every result
__device__ __forceinline__ float tb_rb(float x) {
  const unsigned b = __float_as_uint(x);
  return __uint_as_float(isnan(x) ? ((b >> 16) | 0x40u) << 16
                                  : ((b + 0x7fffu + ((b >> 16) & 1u)) >> 16) << 16);
}
)";
}

int64_t volume_of(const std::vector<int64_t>& s) {
  int64_t v = 1;
  for (auto e : s) v *= e;
  return v;
}

bool needs_wide(const Program& P, const Kernel& K) {
  int64_t big = volume_of(K.space);
  for (int b : K.params) big = std::max(big, P.buffers[b].bytes / 4);
  if (K.node >= 0) big = std::max(big, P.nodes[K.node].volume());
  big = std::max(big, K.batch * std::max(K.m, K.n) * std::max<int64_t>(K.kp, 1));
  return big >= (1LL << 31) - 1;
}

const int SMS = 148;

}  // namespace

// ---- flat elementwise group
// Evaluates once, before a kernel's element loop, every rank-0 value its
// members read that does not depend on the element: constants, scalars other
// kernels wrote, and expressions of those (a loss scale, a 1 / count).  The
// loop body then finds them in the outer memo scope instead of recomputing
// them per element.
static void hoist_uniform_scalars(Program& P, Kernel& K, Emitter& E) {
  std::map<int, bool> uniform;
  std::function<bool(int)> is_uniform = [&](int n) -> bool {
    auto it = uniform.find(n);
    if (it != uniform.end()) return it->second;
    const Node& nd = P.nodes[n];
    const Info& f = P.info[n];
    bool u = false;
    if (nd.rank == 0 && !E.member_of.count(n)) {
      if (f.kind == Kind::Const) u = true;
      else if (f.materialized && f.owner == n) u = true;  // read from its buffer
      else if (f.kind == Kind::Expr && !f.materialized && is_elementwise(nd.op)) {
        u = true;
        for (int o : {nd.operands[0], nd.operands[1]})
          if (o >= 0 && !is_uniform(o)) u = false;
      }
    }
    uniform[n] = u;
    return u;
  };
  std::set<int> seen;
  std::vector<int> order;
  std::function<void(int)> visit = [&](int n) {
    if (!seen.insert(n).second) return;
    const Info& f = P.info[n];
    if (is_uniform(n)) {
      if (f.kind != Kind::Const) order.push_back(n);
      return;
    }
    // a value read from a buffer (other than this kernel's members) ends the walk
    if ((f.materialized || f.kind == Kind::Layout) && !E.member_of.count(n)) return;
    const Node& nd = P.nodes[n];
    for (int o : {nd.operands[0], nd.operands[1]})
      if (o >= 0) visit(o);
  };
  for (auto& m : K.members) {
    const Node& nd = P.nodes[m.node];
    if (m.type == MemberType::EW || m.type == MemberType::PREP) {
      if (m.type == MemberType::PREP && !E.member_of.count(m.node) && P.info[m.node].materialized)
        continue;
      for (int o : {nd.operands[0], nd.operands[1]})
        if (o >= 0) visit(o);
    } else if (nd.operands[0] >= 0) {
      visit(nd.operands[0]);
    }
  }
  for (int n : order) E.ref(n, Idx{});
}

// In a row kernel, evaluates once per row (before the passes over its
// elements) every row-shaped value the members read that depends only on
// buffers other kernels wrote and constants -- per-row statistics such as
// sqrt(variance + eps) -- so the passes find it in the row's memo scope.
// Only when every team row is in range (R a multiple of the rows per block):
// the hoisted loads are not behind the `act` guard.
static void hoist_row_uniform(Program& P, Kernel& K, Emitter& E,
                              const std::vector<int64_t>& lead,
                              const std::vector<std::string>& rc) {
  std::map<int, bool> memo;
  std::function<bool(int)> row_uniform = [&](int n) -> bool {
    auto it = memo.find(n);
    if (it != memo.end()) return it->second;
    const Node& nd = P.nodes[n];
    const Info& f = P.info[n];
    bool u = false;
    if (!E.member_of.count(n)) {
      if (f.kind == Kind::Const) u = true;
      else if (nd.rank == 0 && f.materialized && f.owner == n) u = true;
      else if (nd.dims() == lead && f.materialized && f.owner == n) u = true;
      else if ((nd.rank == 0 || nd.dims() == lead) && f.kind == Kind::Expr && !f.materialized &&
               is_elementwise(nd.op)) {
        u = true;
        for (int o : {nd.operands[0], nd.operands[1]})
          if (o >= 0 && !row_uniform(o)) u = false;
      }
    }
    memo[n] = u;
    return u;
  };
  std::set<int> seen;
  std::vector<int> order;
  std::function<void(int)> visit = [&](int n) {
    if (!seen.insert(n).second) return;
    const Node& nd = P.nodes[n];
    const Info& f = P.info[n];
    if (nd.dims() == lead && !lead.empty() && row_uniform(n)) {
      if (f.kind != Kind::Const) order.push_back(n);
      return;
    }
    if ((f.materialized || f.kind == Kind::Layout) && !E.member_of.count(n)) return;
    for (int o : {nd.operands[0], nd.operands[1]})
      if (o >= 0) visit(o);
  };
  for (auto& m : K.members) {
    const Node& nd = P.nodes[m.node];
    if (m.type == MemberType::EW || m.type == MemberType::PREP) {
      if (m.type == MemberType::PREP && !E.member_of.count(m.node) && P.info[m.node].materialized)
        continue;
      for (int o : {nd.operands[0], nd.operands[1]})
        if (o >= 0) visit(o);
    } else if (nd.operands[0] >= 0) {
      visit(nd.operands[0]);
    }
  }
  Idx idx;
  idx.c = rc;
  for (int n : order) E.ref(n, idx);
}

// Stores a PREP member's values (one or four consecutive elements at `off`)
// as their tf32 pairs.
static void emit_prep_store(Emitter& E, const Member& mm, const std::string& off,
                            const std::vector<std::string>& x) {
  const std::string hi = E.fptr(mm.hi), lo = E.fptr(mm.lo);
  E.line("{");
  E.indent += 2;
  for (size_t v = 0; v < x.size(); ++v)
    E.line("const float h" + std::to_string(v) + " = tb_tf32(" + x[v] + ");");
  if (x.size() == 4) {
    E.line("*(float4*)(" + hi + " + " + off + ") = make_float4(h0, h1, h2, h3);");
    E.line("*(float4*)(" + lo + " + " + off + ") = make_float4(__fsub_rn(" + x[0] + ", h0), __fsub_rn(" +
           x[1] + ", h1), __fsub_rn(" + x[2] + ", h2), __fsub_rn(" + x[3] + ", h3));");
  } else {
    E.line(hi + "[" + off + "] = h0;");
    E.line(lo + "[" + off + "] = __fsub_rn(" + x[0] + ", h0);");
  }
  E.indent -= 2;
  E.line("}");
}

static void emit_ew(Program& P, Kernel& K, Emitter& E) {
  const std::vector<int64_t>& S = K.space;
  int64_t total = volume_of(S);
  E.vec = (!S.empty() && S.back() % 4 == 0) ? 4 : 1;
  int64_t units = total / E.vec;
  K.block = 256;
  K.grid = std::max<int64_t>(1, std::min<int64_t>((units + 255) / 256, SMS * 8));
  // one unit of work: the element(s) at lin = t * vec, in its own scope
  auto emit_unit = [&](const std::string& t) {
  E.line("{");
  E.indent += 2;
  E.push();
  E.line("const I lin = " + t + " * " + std::to_string(E.vec) + ";");
  std::vector<std::string> base = E.unravel("lin", S, "i");
  std::vector<std::vector<std::string>> vals(K.members.size());
  for (int v = 0; v < E.vec; ++v) {
    Idx idx;
    idx.c = base;
    if (!S.empty() && E.vec > 1) {
      idx.c.back() = s_add(base.back(), std::to_string(v));
      idx.lane = v;
      idx.lbase = base.back();
    }
    for (size_t m = 0; m < K.members.size(); ++m) {
      int n = K.members[m].node;
      if (K.members[m].type == MemberType::PREP) {
        vals[m].push_back(E.ref(n, idx));
        continue;
      }
      std::string x = E.def(n, idx);
      E.memo.back()[Emitter::key(n, idx)] = x;
      vals[m].push_back(x);
    }
  }
  for (size_t m = 0; m < K.members.size(); ++m)
    for (const std::string& x : vals[m]) E.note_member_value(x);
  for (size_t m = 0; m < K.members.size(); ++m) {
    if (K.members[m].type == MemberType::PREP) {
      emit_prep_store(E, K.members[m], "lin", vals[m]);
      continue;
    }
    int buf = P.info[K.members[m].node].buf;
    if (E.vec == 4) {
      E.line("*(float4*)(" + E.fptr(buf) + " + lin) = make_float4(" + vals[m][0] + ", " +
             vals[m][1] + ", " + vals[m][2] + ", " + vals[m][3] + ");");
    } else {
      E.line(E.fptr(buf) + "[lin] = " + vals[m][0] + ";");
    }
  }
  E.pop();
  E.indent -= 2;
  E.line("}");
  };
  hoist_uniform_scalars(P, K, E);
  E.line("const I stride = (I)gridDim.x * 256;");
  E.line("I t = (I)blockIdx.x * 256 + threadIdx.x;");
  // (the unrolled trip's index t + 3 * stride must not overflow a 32-bit I)
  if (E.vec == 1 && units >= 4 * K.grid * 256 && units + 4 * K.grid * 256 < (int64_t(1) << 31)) {
    // scalar elements: four strides per trip with no bounds test between
    // them, so each thread has four loads of each operand in flight
    E.line("for (; t + 3 * stride < " + lit(units) + "; t += 4 * stride) {");
    E.indent += 2;
    for (int u = 0; u < 4; ++u) emit_unit(u == 0 ? "t" : "(t + " + std::to_string(u) + " * stride)");
    E.indent -= 2;
    E.line("}");
  }
  E.line("for (; t < " + lit(units) + "; t += stride) {");
  E.indent += 2;
  emit_unit("t");
  E.indent -= 2;
  E.line("}");
}

// ---- row-space group: phases of elementwise work separated by row reductions
static void emit_row(Program& P, Kernel& K, Emitter& E, Lowerer& Lw,
                     std::vector<Kernel>& finals) {
  const std::vector<int64_t>& space = K.space;
  // A one-dimensional space with no row or column reductions (elementwise
  // members and full sums only) is cut into virtual rows of 128, so that
  // many blocks share it instead of one team walking all of it; members still
  // index the flat position row * 128 + j.
  bool virtual_rows = space.size() == 1 && space[0] >= 4096 && space[0] % 128 == 0;
  for (auto& m : K.members)
    if (m.type == MemberType::ROW_SUM || m.type == MemberType::ROW_MAX ||
        m.type == MemberType::COL_SUM)
      virtual_rows = false;
  const std::vector<int64_t> S =
      virtual_rows ? std::vector<int64_t>{space[0] / 128, 128} : space;
  int64_t L = S.back();
  int64_t R = volume_of(S) / L;
  int64_t T, KC;
  int vec;
  int col_members = 0;
  for (auto& m : K.members) col_members += m.type == MemberType::COL_SUM;
  Lw.row_shape(S, T, KC, vec, col_members);
  E.vec = vec;
  int64_t teams = 256 / T;
  // One-pass log-sum-exp: a row sum of exp(x - bcast(row max of x)) whose max
  // is a member here is accumulated in the max's own pass, online (running
  // max and rescaled sum), instead of a second pass over the row.
  std::vector<int> partner(K.members.size(), -1), partner_of(K.members.size(), -1);
  {
    std::map<int, int> max_member;
    for (size_t m = 0; m < K.members.size(); ++m)
      if (K.members[m].type == MemberType::ROW_MAX) max_member[K.members[m].node] = (int)m;
    auto virt = [&](int n) { return !P.info[n].materialized; };
    // a bf16 network rounds exp(x - max) per element against the final max,
    // which the online update cannot: its rows keep the two-pass form
    for (size_t m = 0; m < K.members.size() && !P.bf16; ++m) {
      if (K.members[m].type != MemberType::ROW_SUM) continue;
      const int e = P.nodes[K.members[m].node].operands[0];
      if (P.nodes[e].op != TB_OP_EXP || !virt(e)) continue;
      const int sh = P.nodes[e].operands[0];
      if (P.nodes[sh].op != TB_OP_SUB || !virt(sh)) continue;
      const int x = P.nodes[sh].operands[0], pb = P.nodes[sh].operands[1];
      if (P.nodes[pb].op != TB_OP_BROADCAST_ALONG || P.info[pb].materialized) continue;
      auto it = max_member.find(P.nodes[pb].operands[0]);
      if (it == max_member.end() || partner[it->second] >= 0) continue;
      if (P.nodes[K.members[it->second].node].operands[0] != x) continue;
      partner[it->second] = (int)m;
      partner_of[m] = it->second;
      K.members[m].phase = K.members[it->second].phase;
    }
    std::set<int> used;
    for (auto& mm : K.members) used.insert(mm.phase);
    std::map<int, int> rank;
    for (int ph : used) rank[ph] = (int)rank.size();
    for (auto& mm : K.members) mm.phase = rank[mm.phase];
  }
  bool has_col = false, has_all = false;
  int maxphase = 0;
  for (auto& m : K.members) {
    if (m.type == MemberType::COL_SUM) has_col = true;
    if (m.type == MemberType::ALL_SUM) has_all = true;
    maxphase = std::max(maxphase, m.phase);
  }
  K.block = 256;
  // per-block column partials cost blocks * L floats: fewer blocks for wide rows
  // four blocks per SM (the launch bound): for C2's 8192-wide rows, 592 blocks
  // ran the kernel 8% faster than 444 for 5 MB more partials
  int64_t cap = SMS * 4;
  K.grid = std::max<int64_t>(1, std::min<int64_t>((R + teams - 1) / teams, cap));
  if (has_col || has_all) E.exact = false;
  // A team's reduction waits only for its own warps (a named barrier per
  // team), so the teams of a block move through their rows independently.
  const std::string team_sync =
      teams > 1 ? "asm volatile(\"bar.sync %0, " + std::to_string(T) +
                      ";\" :: \"r\"(team + 1) : \"memory\");"
                : "__syncthreads();";
  E.line("__shared__ float sred[8], sred2[8];");
  if (has_col) E.line("__shared__ float scol[" + lit(L) + "];");
  E.line("const int tid = threadIdx.x, team = tid / " + std::to_string(T) + ", tl = tid % " +
         std::to_string(T) + ";");
  (void)teams;
  for (size_t m = 0; m < K.members.size(); ++m) {
    if (K.members[m].type == MemberType::COL_SUM)
      E.line("float ca" + std::to_string(m) + "[" + std::to_string(KC * vec) + "] = {0};");
    if (K.members[m].type == MemberType::ALL_SUM) E.line("float fa" + std::to_string(m) + " = 0.0f;");
  }
  // EW members no other kernel reads and that a later phase uses stay in
  // registers (fully unrolled passes index the arrays with constants)
  for (size_t m = 0; m < K.members.size(); ++m) {
    Member& mm = K.members[m];
    if (KC * vec > 32) mm.reg = false;
    if (!mm.reg) continue;
    E.in_registers.insert((int)m);
    E.line("float kr" + std::to_string(m) + "[" + std::to_string(KC * vec) + "];");
  }
  hoist_uniform_scalars(P, K, E);
  E.line("for (I base = (I)blockIdx.x * " + std::to_string(teams) + "; base < " + lit(R) +
         "; base += (I)gridDim.x * " + std::to_string(teams) + ") {");
  E.indent += 2;
  E.line("const I row = base + team;");
  E.line("const bool act = row < " + lit(R) + ";");
  std::vector<int64_t> lead(S.begin(), S.end() - 1);
  if (virtual_rows) lead.clear();  // the row is part of the flat position, not a coordinate
  const std::string jbase = virtual_rows ? "(row * " + lit(L) + " + j0)" : "j0";
  std::vector<std::string> rc = lead.empty() ? std::vector<std::string>{}
                                             : E.unravel("row", lead, "i");
  if (R % teams == 0) hoist_row_uniform(P, K, E, lead, rc);
  for (int ph = 0; ph <= maxphase; ++ph) {
    E.phase = ph;
    E.line("// phase " + std::to_string(ph));
    for (size_t m = 0; m < K.members.size(); ++m) {
      const Member& mm = K.members[m];
      if (mm.phase != ph) continue;
      if (mm.type == MemberType::ROW_SUM) E.line("float ra" + std::to_string(m) + " = 0.0f;");
      if (mm.type == MemberType::ROW_MAX)
        E.line("float ra" + std::to_string(m) + " = " +
               (partner[m] >= 0 ? "-TB_INF;" : "__int_as_float(0x7fc00000);"));
    }
    // Full passes over the row need no bounds test, so the unrolled loads of
    // several passes are issued before their results are used; only a last
    // partial pass (row length not a multiple of the team's stride) is guarded.
    const int64_t kc_full = L / (T * vec);
    auto emit_pass = [&]() {
    E.push();
    std::vector<std::vector<std::string>> vals(K.members.size());
    for (int v = 0; v < vec; ++v) {
      Idx idx;
      idx.c = rc;
      idx.c.push_back(vec > 1 ? s_add(jbase, std::to_string(v)) : jbase);
      if (vec > 1) {
        idx.lane = v;
        idx.lbase = jbase;
      }
      for (size_t m = 0; m < K.members.size(); ++m) {
        const Member& mm = K.members[m];
        if (mm.phase != ph) continue;
        int n = mm.node;
        if (partner_of[m] >= 0) continue;  // accumulated with its max
        std::string x;
        if (mm.type == MemberType::EW) {
          x = E.def(n, idx);
          E.memo.back()[Emitter::key(n, idx)] = x;
        } else if (mm.type == MemberType::PREP) {
          x = E.ref(n, idx);
        } else {
          x = E.ref(P.nodes[n].operands[0], idx);
        }
        vals[m].push_back(x);
        if (mm.type == MemberType::EW || mm.type == MemberType::PREP) {
          E.note_member_value(x);
          if (E.is_tainted(x)) E.tainted_members.insert((int)m);
        }
        std::string ms = std::to_string(m);
        switch (mm.type) {
          case MemberType::ROW_SUM: E.line("ra" + ms + " = __fadd_rn(ra" + ms + ", " + x + ");"); break;
          case MemberType::ROW_MAX:
            if (partner[m] >= 0)
              E.line("tb_lse_push(ra" + ms + ", ra" + std::to_string(partner[m]) + ", " + x + ");");
            else
              E.line("ra" + ms + " = tb_max(ra" + ms + ", " + x + ");");
            break;
          case MemberType::COL_SUM:
            E.line("ca" + ms + "[kc * " + std::to_string(vec) + " + " + std::to_string(v) +
                   "] = __fadd_rn(ca" + ms + "[kc * " + std::to_string(vec) + " + " +
                   std::to_string(v) + "], " + x + ");");
            break;
          case MemberType::ALL_SUM: E.line("fa" + ms + " = __fadd_rn(fa" + ms + ", " + x + ");"); break;
          default: break;
        }
      }
    }
    for (size_t m = 0; m < K.members.size(); ++m) {
      const Member& mm = K.members[m];
      if (mm.phase != ph || mm.type != MemberType::PREP) continue;
      emit_prep_store(E, mm, "row * " + lit(L) + " + j0", vals[m]);
    }
    for (size_t m = 0; m < K.members.size(); ++m) {
      const Member& mm = K.members[m];
      if (mm.phase != ph || mm.type != MemberType::EW) continue;
      if (E.in_registers.count((int)m)) {
        for (int v = 0; v < vec; ++v)
          E.line("kr" + std::to_string(m) + "[kc * " + std::to_string(vec) + " + " +
                 std::to_string(v) + "] = " + vals[m][v] + ";");
        continue;
      }
      int buf = P.info[mm.node].buf;
      if (vec == 4) {
        E.line("*(float4*)(" + E.fptr(buf) + " + row * " + lit(L) + " + j0) = make_float4(" +
               vals[m][0] + ", " + vals[m][1] + ", " + vals[m][2] + ", " + vals[m][3] + ");");
      } else {
        E.line(E.fptr(buf) + "[row * " + lit(L) + " + j0] = " + vals[m][0] + ";");
      }
    }
    E.pop();
    };
    if (kc_full > 0) {
      E.line("if (act) {");
      E.indent += 2;
      E.line(has_col || !E.in_registers.empty() ? "#pragma unroll"
                                                 : (vec == 1 ? "#pragma unroll 8" : "#pragma unroll 4"));
      E.line("for (int kc = 0; kc < " + std::to_string(kc_full) + "; ++kc) {");
      E.indent += 2;
      E.line("const I j0 = ((I)kc * " + std::to_string(T) + " + tl) * " + std::to_string(vec) + ";");
      emit_pass();
      E.indent -= 2;
      E.line("}");
      E.indent -= 2;
      E.line("}");
    }
    if (kc_full < KC) {
      E.line("{");
      E.indent += 2;
      E.line("const int kc = " + std::to_string(kc_full) + ";");
      E.line("const I j0 = ((I)kc * " + std::to_string(T) + " + tl) * " + std::to_string(vec) + ";");
      E.line("if (act && j0 < " + lit(L) + ") {");
      E.indent += 2;
      emit_pass();
      E.indent -= 2;
      E.line("}");
      E.indent -= 2;
      E.line("}");
    }
    // team reductions of this phase
    for (size_t m = 0; m < K.members.size(); ++m) {
      const Member& mm = K.members[m];
      if (mm.phase != ph || (mm.type != MemberType::ROW_SUM && mm.type != MemberType::ROW_MAX))
        continue;
      E.exact = false;
      if (partner_of[m] >= 0) continue;  // reduced with its max
      std::string ms = std::to_string(m);
      if (partner[m] >= 0) {
        const std::string ts = std::to_string(partner[m]);
        E.line("float rv" + ms + " = ra" + ms + ", rv" + ts + " = ra" + ts + ";");
        int64_t width = std::min<int64_t>(T, 32);
        for (int64_t o = width / 2; o > 0; o /= 2)
          E.line("{ const float m2 = __shfl_xor_sync(0xffffffffu, rv" + ms + ", " +
                 std::to_string(o) + "), s2 = __shfl_xor_sync(0xffffffffu, rv" + ts + ", " +
                 std::to_string(o) + "); tb_lse_merge(rv" + ms + ", rv" + ts + ", m2, s2); }");
        if (T > 32) {
          E.line("if ((tid & 31) == 0) { sred[tid >> 5] = rv" + ms + "; sred2[tid >> 5] = rv" + ts + "; }");
          E.line(team_sync);
          int64_t w = T / 32;
          E.line("{ const int w0 = team * " + std::to_string(w) + "; rv" + ms + " = sred[w0]; rv" +
                 ts + " = sred2[w0];");
          for (int64_t q = 1; q < w; ++q)
            E.line("  tb_lse_merge(rv" + ms + ", rv" + ts + ", sred[w0 + " + std::to_string(q) +
                   "], sred2[w0 + " + std::to_string(q) + "]);");
          E.line("}");
          E.line(team_sync);
        }
        E.line("if (act && tl == 0) { " + E.fptr(P.info[mm.node].buf) + "[row] = rv" + ms + "; " +
               E.fptr(P.info[K.members[partner[m]].node].buf) + "[row] = rv" + ts + "; }");
        continue;
      }
      std::string op = mm.type == MemberType::ROW_SUM ? "__fadd_rn" : "tb_max";
      E.line("float rv" + ms + " = ra" + ms + ";");
      int64_t width = std::min<int64_t>(T, 32);
      for (int64_t o = width / 2; o > 0; o /= 2)
        E.line("rv" + ms + " = " + op + "(rv" + ms + ", __shfl_xor_sync(0xffffffffu, rv" + ms +
               ", " + std::to_string(o) + "));");
      if (T > 32) {
        E.line("if ((tid & 31) == 0) sred[tid >> 5] = rv" + ms + ";");
        E.line(team_sync);
        int64_t w = T / 32;
        E.line("{ const int w0 = team * " + std::to_string(w) + "; rv" + ms + " = sred[w0];");
        for (int64_t q = 1; q < w; ++q)
          E.line("  rv" + ms + " = " + op + "(rv" + ms + ", sred[w0 + " + std::to_string(q) + "]);");
        E.line("}");
        E.line(team_sync);
      }
      // f32 accumulation, one rounding (payload/tensor.rs:1085-1089)
      if (P.bf16 && mm.type == MemberType::ROW_SUM) E.line("rv" + ms + " = tb_rb(rv" + ms + ");");
      E.line("if (act && tl == 0) " + E.fptr(P.info[mm.node].buf) + "[row] = rv" + ms + ";");
    }
  }
  E.indent -= 2;
  E.line("}");
  // column and full sums: per-block partials, combined by a FINAL kernel
  for (size_t m = 0; m < K.members.size(); ++m) {
    const Member& mm = K.members[m];
    std::string ms = std::to_string(m);
    if (mm.type == MemberType::COL_SUM) {
      int part = Lw.new_buffer(Storage::Arena, K.grid * L * 4, -1);
      E.line("{");
      E.line("  for (int tm = 0; tm < " + std::to_string(teams) + "; ++tm) {");
      E.line("    if (team == tm) {");
      E.line("#pragma unroll");
      E.line("      for (int kc = 0; kc < " + std::to_string(KC) + "; ++kc) {");
      for (int v = 0; v < vec; ++v) {
        E.line("        { const I j = ((I)kc * " + std::to_string(T) + " + tl) * " +
               std::to_string(vec) + " + " + std::to_string(v) + "; if (j < " + lit(L) +
               ") scol[j] = tm == 0 ? ca" + ms + "[kc * " + std::to_string(vec) + " + " +
               std::to_string(v) + "] : __fadd_rn(scol[j], ca" + ms + "[kc * " +
               std::to_string(vec) + " + " + std::to_string(v) + "]); }");
      }
      E.line("      }");
      E.line("    }");
      E.line("    __syncthreads();");
      E.line("  }");
      E.line("  for (I j = tid; j < " + lit(L) + "; j += 256) " + E.fptr(part) +
             "[(I)blockIdx.x * " + lit(L) + " + j] = scol[j];");
      E.line("  __syncthreads();");
      E.line("}");
      Kernel f;
      f.type = KType::FINAL;
      f.partial = part;
      f.final_out = P.info[mm.node].buf;
      f.final_blocks = K.grid;
      f.final_width = L;
      f.exact = false;
      finals.push_back(f);
    }
    if (mm.type == MemberType::ALL_SUM) {
      int part = Lw.new_buffer(Storage::Arena, K.grid * 4, -1);
      E.line("{");
      E.line("  float s = fa" + ms + ";");
      for (int o = 16; o > 0; o /= 2)
        E.line("  s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, " + std::to_string(o) + "));");
      E.line("  if ((tid & 31) == 0) sred[tid >> 5] = s;");
      E.line("  __syncthreads();");
      E.line("  if (tid == 0) { float t = sred[0]; for (int w = 1; w < 8; ++w) t = __fadd_rn(t, sred[w]); " +
             E.fptr(part) + "[blockIdx.x] = t; }");
      E.line("  __syncthreads();");
      E.line("}");
      Kernel f;
      f.type = KType::FINAL;
      f.partial = part;
      f.final_out = P.info[mm.node].buf;
      f.final_blocks = K.grid;
      f.final_width = 1;
      f.exact = false;
      finals.push_back(f);
    }
  }
}

// ---- generic serial reduction: one thread per output, ascending order
static void emit_reduce(Program& P, Kernel& K, Emitter& E) {
  int n = K.node;
  const Node& nd = P.nodes[n];
  const Node& x = P.nodes[nd.operands[0]];
  int axis = (int)nd.attrs[0];
  bool max = nd.op == TB_OP_MAX_ALONG;
  int64_t outs = nd.volume();
  K.grid = std::max<int64_t>(1, std::min<int64_t>((outs + 255) / 256, SMS * 8));
  E.line("for (I t = (I)blockIdx.x * 256 + threadIdx.x; t < " + lit(outs) +
         "; t += (I)gridDim.x * 256) {");
  E.indent += 2;
  std::vector<std::string> oc = E.unravel("t", nd.dims(), "o");
  std::vector<std::string> c;
  for (int j = 0, s = 0; j < x.rank; ++j) c.push_back(j == axis ? "0" : oc[s++]);
  Idx first;
  first.c = c;
  E.push();
  std::string x0 = E.ref(nd.operands[0], first);
  E.line("float acc = " + x0 + ";");
  E.pop();
  E.line("for (I s = 1; s < " + lit(x.shape[axis]) + "; ++s) {");
  E.indent += 2;
  E.push();
  Idx at;
  at.c = c;
  at.c[axis] = "s";
  std::string xv = E.ref(nd.operands[0], at);
  E.line(std::string("acc = ") + (max ? "tb_max" : "__fadd_rn") + "(acc, " + xv + ");");
  E.pop();
  E.indent -= 2;
  E.line("}");
  E.line(E.fptr(P.info[n].buf) + (P.bf16 ? "[t] = tb_rb(acc);" : "[t] = acc;"));
  E.indent -= 2;
  E.line("}");
}

// ---- scatter-add over the stably sorted selection (payload/tensor.rs:1582-1618)
// This kernel writes the scatter source rows in target order (perm[q] =
// g[vals[q]]), a fully parallel copy; a SEGSUM kernel then sums each target's
// contiguous rows from zero in ascending source order -- the reference's
// serial order, so the result is bit-identical.
static void emit_scatter(Program& P, Kernel& K, Emitter& E, const Kernel& sort) {
  int n = K.node;
  const Node& nd = P.nodes[n];
  const Node& g = P.nodes[nd.operands[0]];
  int64_t count = g.shape[0];
  int64_t width = nd.volume() / nd.shape[0];
  std::vector<int64_t> rest(nd.shape + 1, nd.shape + nd.rank);
  int64_t total = count * width;
  K.grid = std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, SMS * 8));
  E.line("for (I t = (I)blockIdx.x * 256 + threadIdx.x; t < " + lit(total) +
         "; t += (I)gridDim.x * 256) {");
  E.indent += 2;
  E.line("const I q = t / " + lit(width) + ";");
  E.line("const I o = t % " + lit(width) + ";");
  std::vector<std::string> oc = rest.empty() ? std::vector<std::string>{} : E.unravel("o", rest, "c");
  E.line("const I s = (I)" + E.iptr(sort.vals) + "[q];");
  Idx at;
  at.c.push_back("s");
  for (auto& c : oc) at.c.push_back(c);
  std::string v = E.ref(nd.operands[0], at);
  E.line(E.fptr(K.partial) + "[t] = " + v + ";");
  E.indent -= 2;
  E.line("}");
}

// ---- fold (payload/tensor.rs:1392-1463)
static void emit_fold(Program& P, Kernel& K, Emitter& E) {
  int n = K.node;
  const Node& nd = P.nodes[n];
  const Node& x = P.nodes[nd.operands[0]];
  int axis = (int)nd.attrs[0];
  int64_t size = nd.attrs[1], step = nd.attrs[2], dil = nd.attrs[3];
  int64_t count = x.shape[axis];
  int64_t outs = nd.volume();
  K.grid = std::max<int64_t>(1, std::min<int64_t>((outs + 255) / 256, SMS * 8));
  E.line("for (I t = (I)blockIdx.x * 256 + threadIdx.x; t < " + lit(outs) +
         "; t += (I)gridDim.x * 256) {");
  E.indent += 2;
  std::vector<std::string> oc = E.unravel("t", nd.dims(), "o");
  E.line("float acc = 0.0f;");
  E.line("for (I k = 0; k < " + lit(size) + "; ++k) {");
  E.indent += 2;
  E.line("const I reach = k * " + lit(dil) + ";");
  E.line("if (reach > " + oc[axis] + ") break;");
  E.line("const I rest = " + oc[axis] + " - reach;");
  E.line("if (rest % " + lit(step) + " != 0) continue;");
  E.line("const I w = rest / " + lit(step) + ";");
  E.line("if (w >= " + lit(count) + ") continue;");
  E.push();
  Idx at;
  for (int j = 0; j < nd.rank; ++j) {
    if (j == axis) {
      at.c.push_back("w");
      at.c.push_back("k");
    } else {
      at.c.push_back(oc[j]);
    }
  }
  std::string v = E.ref(nd.operands[0], at);
  E.line("acc = __fadd_rn(acc, " + v + ");");
  E.pop();
  E.indent -= 2;
  E.line("}");
  E.line(E.fptr(P.info[n].buf) + (P.bf16 ? "[t] = tb_rb(acc);" : "[t] = acc;"));
  E.indent -= 2;
  E.line("}");
}

// The logical axis of node n along which consecutive elements sit next to
// each other in the memory the expression ultimately reads (the axis a
// coalesced reader should walk).
static int fast_axis(const Program& P, int n, int depth = 0) {
  const Node& nd = P.nodes[n];
  const Info& f = P.info[n];
  const int last = nd.rank - 1;
  if (nd.rank <= 1 || depth > 64) return last;
  if (f.materialized || f.kind == Kind::Layout) {
    for (int d = nd.rank - 1; d >= 0; --d)
      if (f.lay.stride[d] == 1 && f.lay.shape[d] > 1) return d;
    return last;
  }
  const int a = nd.operands[0];
  const int64_t* at = nd.attrs;
  if (is_elementwise(nd.op)) {
    // follow the operand that reads a full-size buffer rather than a broadcast
    for (int k = 0; k < 2; ++k) {
      int o = nd.operands[k];
      if (o < 0) continue;
      const Info& fo = P.info[o];
      if (fo.kind == Kind::Const || fo.kind == Kind::Sel) continue;
      if ((fo.materialized || fo.kind == Kind::Layout)) {
        bool broadcast = false;
        for (int d = 0; d < fo.lay.rank; ++d)
          if (fo.lay.stride[d] == 0 && fo.lay.shape[d] > 1) broadcast = true;
        if (broadcast) continue;
      }
      return fast_axis(P, o, depth + 1);
    }
    return last;
  }
  switch (nd.op) {
    case TB_OP_TRANSPOSE: return fast_axis(P, a, depth + 1) == 0 ? 1 : 0;
    case TB_OP_PERMUTE: {
      int fa = fast_axis(P, a, depth + 1);
      for (int j = 0; j < nd.rank; ++j)
        if (at[j] == fa) return j;
      return last;
    }
    case TB_OP_NARROW:
    case TB_OP_PAD:
      return fast_axis(P, a, depth + 1);
    case TB_OP_BROADCAST_ALONG: {
      int fa = fast_axis(P, a, depth + 1);
      return fa >= at[0] ? fa + 1 : fa;
    }
    case TB_OP_RESHAPE:
    case TB_OP_GATHER: {
      const Node& on = P.nodes[a];
      (void)on;  // row-major results of a reshape or a row gather run along the last axis
      return last;
    }
  }
  return last;
}

// ---- GEMM operand preparation: tf32 hi/lo split of a value [batch, R, Kd]
// into its own row-major layout [batch, R, Kp], the last axis zero-padded to
// Kp (a multiple of 32)
static void emit_prep(Program& P, Kernel& K, Emitter& E) {
  const int x = K.node;
  const Node& xn = P.nodes[x];
  int split = xn.rank - 2;
  std::vector<int64_t> bshape(xn.shape, xn.shape + split);
  int64_t R = K.m, Kd = K.k, Kp = K.kp;
  const bool is_b = false;  // the value's own axes: R then Kd
  // transpose through shared memory when the value is contiguous along R
  const int fa = fast_axis(P, x);
  const bool tile = fa == (is_b ? split + 1 : split);
  auto operand_idx = [&](const std::vector<std::string>& bc, const std::string& r,
                         const std::string& k) {
    Idx idx;
    idx.c = bc;
    if (is_b) {
      idx.c.push_back(k);
      idx.c.push_back(r);
    } else {
      idx.c.push_back(r);
      idx.c.push_back(k);
    }
    return idx;
  };
  std::string hi = E.fptr(K.a_hi), lo = E.fptr(K.a_lo);
  if (!tile) {
    int64_t quads = K.batch * R * (Kp / 4);
    K.grid = std::max<int64_t>(1, std::min<int64_t>((quads + 255) / 256, SMS * 8));
    E.vec = (!is_b && Kd % 4 == 0) ? 4 : 1;
    E.line("for (I t = (I)blockIdx.x * 256 + threadIdx.x; t < " + lit(quads) +
           "; t += (I)gridDim.x * 256) {");
    E.indent += 2;
    E.line("const I kq = t % " + lit(Kp / 4) + ";");
    E.line("const I rest = t / " + lit(Kp / 4) + ";");
    E.line("const I r = rest % " + lit(R) + ";");
    E.line("const I b = rest / " + lit(R) + ";");
    E.line("const I k0 = kq * 4;");
    std::vector<std::string> bc = bshape.empty() ? std::vector<std::string>{}
                                                 : E.unravel("b", bshape, "bb");
    E.line("float x0 = 0.0f, x1 = 0.0f, x2 = 0.0f, x3 = 0.0f;");
    if (Kd % 4 == 0) {
      E.line("if (k0 < " + lit(Kd) + ") {");
      E.indent += 2;
      E.push();
      for (int v = 0; v < 4; ++v) {
        Idx idx = operand_idx(bc, "r", s_add("k0", std::to_string(v)));
        if (E.vec == 4) {
          idx.lane = v;
          idx.lbase = "k0";
        }
        std::string xv = E.ref(x, idx);
        E.line("x" + std::to_string(v) + " = " + xv + ";");
      }
      E.pop();
      E.indent -= 2;
      E.line("}");
    } else {
      for (int v = 0; v < 4; ++v) {
        E.line("if (k0 + " + std::to_string(v) + " < " + lit(Kd) + ") {");
        E.indent += 2;
        E.push();
        Idx idx = operand_idx(bc, "r", s_add("k0", std::to_string(v)));
        std::string xv = E.ref(x, idx);
        E.line("x" + std::to_string(v) + " = " + xv + ";");
        E.pop();
        E.indent -= 2;
        E.line("}");
      }
    }
    E.line("const float h0 = tb_tf32(x0), h1 = tb_tf32(x1), h2 = tb_tf32(x2), h3 = tb_tf32(x3);");
    E.line("const I o = (b * " + lit(R) + " + r) * " + lit(Kp) + " + k0;");
    E.line("*(float4*)(" + hi + " + o) = make_float4(h0, h1, h2, h3);");
    E.line("*(float4*)(" + lo + " + o) = make_float4(__fsub_rn(x0, h0), __fsub_rn(x1, h1), "
           "__fsub_rn(x2, h2), __fsub_rn(x3, h3));");
    E.indent -= 2;
    E.line("}");
    return;
  }
  int64_t rt = (R + 31) / 32, kt = Kp / 32;
  int64_t tiles = K.batch * rt * kt;
  K.grid = std::max<int64_t>(1, std::min<int64_t>(tiles, SMS * 16));
  E.vec = 1;
  E.line("__shared__ float sm[32][33];");
  E.line("const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;");
  E.line("for (I t = blockIdx.x; t < " + lit(tiles) + "; t += gridDim.x) {");
  E.indent += 2;
  E.line("const I kt = t % " + lit(kt) + ";");
  E.line("const I rest = t / " + lit(kt) + ";");
  E.line("const I r0 = (rest % " + lit(rt) + ") * 32;");
  E.line("const I b = rest / " + lit(rt) + ";");
  E.line("const I k0 = kt * 32;");
  std::vector<std::string> bc = bshape.empty() ? std::vector<std::string>{}
                                               : E.unravel("b", bshape, "bb");
  E.line("#pragma unroll");
  E.line("for (int q = 0; q < 4; ++q) {");
  E.indent += 2;
  E.line("const I r = r0 + tx, k = k0 + ty + 8 * q;");
  E.line("float xv = 0.0f;");
  E.line("if (r < " + lit(R) + " && k < " + lit(Kd) + ") {");
  E.indent += 2;
  E.push();
  Idx idx = operand_idx(bc, "r", "k");
  std::string xv = E.ref(x, idx);
  E.line("xv = " + xv + ";");
  E.pop();
  E.indent -= 2;
  E.line("}");
  E.line("sm[ty + 8 * q][tx] = xv;");
  E.indent -= 2;
  E.line("}");
  E.line("__syncthreads();");
  E.line("#pragma unroll");
  E.line("for (int q = 0; q < 4; ++q) {");
  E.line("  const I r = r0 + ty + 8 * q;");
  E.line("  const float xv = sm[tx][ty + 8 * q];");
  E.line("  const float h = tb_tf32(xv);");
  E.line("  if (r < " + lit(R) + ") { const I o = (b * " + lit(R) + " + r) * " + lit(Kp) +
         " + k0 + tx; " + hi + "[o] = h; " + lo + "[o] = __fsub_rn(xv, h); }");
  E.line("}");
  E.line("__syncthreads();");
  E.indent -= 2;
  E.line("}");
}

// ---- buffer liveness and the arena layout
// Arena invariants, checked after placement (a violation is a lowering bug
// and fails the compile): buffers whose kernel intervals intersect do not
// share bytes, and every buffer of a side kernel stays allocated until the
// side stream joins.
// A row member held in registers has no storage: no kernel, its own
// included, may name its buffer.  Checked before any device memory exists.
static void check_register_members(const Program& P) {
  std::set<int> held;
  for (const Kernel& K : P.kernels)
    for (const Member& m : K.members)
      if (m.reg) held.insert(P.info[m.node].buf);
  if (held.empty()) return;
  for (const Kernel& K : P.kernels)
    for (const std::vector<int>* list : {&K.reads, &K.writes})
      for (int b : *list)
        if (held.count(b))
          fail("internal: the buffer of a register-held value is named by kernel " + K.name);
}

static void check_arena(const Program& P) {
  std::vector<int> placed;
  for (size_t i = 0; i < P.buffers.size(); ++i) {
    const Buffer& b = P.buffers[i];
    if (b.storage == Storage::Arena && b.first >= 0) placed.push_back((int)i);
  }
  std::sort(placed.begin(), placed.end(),
            [&](int x, int y) { return P.buffers[x].offset < P.buffers[y].offset; });
  for (size_t i = 0; i < placed.size(); ++i) {
    const Buffer& a = P.buffers[placed[i]];
    for (size_t j = i + 1; j < placed.size(); ++j) {
      const Buffer& b = P.buffers[placed[j]];
      if (b.offset >= a.offset + a.bytes) break;
      if (a.first <= b.last && b.first <= a.last)
        fail("arena: buffers " + std::to_string(placed[i]) + " and " + std::to_string(placed[j]) +
             " overlap while both are live");
    }
  }
  for (const Kernel& K : P.kernels) {
    if (!K.side) continue;
    for (const std::vector<int>* list : {&K.reads, &K.writes})
      for (int b : *list)
        if (P.buffers[b].storage == Storage::Arena && P.buffers[b].last < P.side_join)
          fail("arena: a side-stream buffer is released before the join");
  }
}

// The main kernel at which the side stream joins: the first that reads or
// writes a buffer a side kernel wrote (the last kernel when none does).
static int side_join(const Program& P) {
  std::set<int> written;
  bool any = false;
  for (const Kernel& K : P.kernels)
    if (K.side) {
      any = true;
      written.insert(K.writes.begin(), K.writes.end());
    }
  if (!any) return -1;
  for (size_t k = 0; k < P.kernels.size(); ++k) {
    const Kernel& K = P.kernels[k];
    if (K.side) continue;
    for (int b : K.reads)
      if (written.count(b)) return (int)k;
    for (int b : K.writes)
      if (written.count(b)) return (int)k;
  }
  return (int)P.kernels.size() - 1;
}

static void plan_arena(Program& P) {
  const int never = -1;
  for (auto& b : P.buffers) {
    b.first = never;
    b.last = never;
  }
  P.side_join = side_join(P);
  for (size_t k = 0; k < P.kernels.size(); ++k) {
    const Kernel& K = P.kernels[k];
    auto touch = [&](int buf) {
      if (buf < 0) return;
      Buffer& b = P.buffers[buf];
      if (b.first == never) b.first = (int)k;
      b.first = std::min(b.first, (int)k);
      b.last = std::max(b.last, (int)k);
    };
    for (int b : K.reads) touch(b);
    for (int b : K.writes) touch(b);
  }
  // a side kernel's buffers (its scratch included) stay allocated until the
  // join: every main kernel before it runs concurrently with the side stream
  for (const Kernel& K : P.kernels) {
    if (!K.side) continue;
    for (int b : K.reads) P.buffers[b].last = std::max(P.buffers[b].last, P.side_join);
    for (int b : K.writes) P.buffers[b].last = std::max(P.buffers[b].last, P.side_join);
  }
  const int end = (int)P.kernels.size();
  std::vector<int> ids;
  for (size_t i = 0; i < P.buffers.size(); ++i) {
    Buffer& b = P.buffers[i];
    if (b.storage != Storage::Arena) continue;
    if (b.node >= 0 && P.nodes[b.node].readable) b.keep = true;
    if (b.first == never) continue;
    if (b.keep) b.last = end;
    ids.push_back((int)i);
  }
  // Readable values (the plan's results, gradients among them) live past the
  // program: they are packed first, contiguously in the order they are
  // written, so gradient exchange can move them in few large ranges.
  std::vector<int> kept, rest;
  for (int id : ids) (P.buffers[id].keep ? kept : rest).push_back(id);
  std::sort(kept.begin(), kept.end(), [&](int x, int y) {
    if (P.buffers[x].first != P.buffers[y].first) return P.buffers[x].first < P.buffers[y].first;
    return x < y;
  });
  int64_t base = 0;
  P.unplanned_bytes = 0;
  for (int id : kept) {
    Buffer& b = P.buffers[id];
    b.offset = base;
    base += (b.bytes + 255) / 256 * 256;
  }
  P.unplanned_bytes = base;
  ids = rest;
  std::sort(ids.begin(), ids.end(), [&](int x, int y) {
    if (P.buffers[x].bytes != P.buffers[y].bytes) return P.buffers[x].bytes > P.buffers[y].bytes;
    return x < y;
  });
  std::vector<int> placed;
  int64_t top = base;
  for (int id : ids) {
    Buffer& b = P.buffers[id];
    int64_t size = (b.bytes + 255) / 256 * 256;
    P.unplanned_bytes += size;
    std::vector<std::pair<int64_t, int64_t>> busy;
    for (int o : placed) {
      const Buffer& q = P.buffers[o];
      if (q.first <= b.last && b.first <= q.last)
        busy.push_back({q.offset, q.offset + (q.bytes + 255) / 256 * 256});
    }
    std::sort(busy.begin(), busy.end());
    int64_t at = base;
    for (auto& [s, e] : busy) {
      if (at + size <= s) break;
      at = std::max(at, e);
    }
    b.offset = at;
    top = std::max(top, at + size);
    placed.push_back(id);
  }
  P.arena_bytes = top;
}

std::unique_ptr<Program> lower(const tb_plan_desc* desc) {
  if (!desc || desc->node_count <= 0 || !desc->nodes) fail("empty plan");
  auto prog = std::make_unique<Program>();
  Program& P = *prog;
  Lowerer Lw(P);
  Lw.run(desc);

  // codegen; FINAL kernels are inserted right after their row kernel
  std::vector<Kernel> kernels;
  kernels.swap(P.kernels);
  // Selection sorts read only input or leaf indices: they move to the front
  // and run on a side stream, overlapping the forward program (their buffers
  // then live from the program's start, so the arena keeps them apart from
  // everything that runs meanwhile).
  {
    std::vector<Kernel> order;
    std::vector<int> moved(kernels.size(), -1);
    for (size_t i = 0; i < kernels.size(); ++i)
      if (kernels[i].type == KType::SORT) {
        moved[i] = (int)order.size();
        order.push_back(kernels[i]);
        order.back().side = true;
      }
    for (size_t i = 0; i < kernels.size(); ++i)
      if (kernels[i].type != KType::SORT) {
        moved[i] = (int)order.size();
        order.push_back(kernels[i]);
      }
    for (auto& [sel, k] : P.sort_of) k = moved[k];
    kernels.swap(order);
  }
  std::map<std::string, std::string> dedupe;  // body -> function name
  std::ostringstream all;
  all << prelude();
  std::map<int, int> sort_index;  // old SORT kernel index -> new index
  for (size_t i = 0; i < kernels.size(); ++i) {
    Kernel K = kernels[i];
    std::vector<Kernel> finals;
    if (K.type == KType::GEMM) {
      K.reads.clear();
      for (int b : {K.a_hi, K.a_lo, K.b_hi, K.b_lo})
        if (b >= 0) K.reads.push_back(b);
      K.writes = {K.out};
      if (K.partial >= 0) K.writes.push_back(K.partial);
      K.exact = false;
      K.describe = "gemm3xtf32 batch=" + std::to_string(K.batch) + " m=" + std::to_string(K.m) +
                   " n=" + std::to_string(K.n) + " k=" + std::to_string(K.k) +
                   " splits=" + std::to_string(K.passes) + " a=" + (K.a_mn ? "mn" : "k") +
                   (K.a_lo < 0 ? ":raw" : "") + " b=" + (K.b_mn ? "mn" : "k") +
                   (K.b_lo < 0 ? ":raw" : "");
      P.kernels.push_back(K);
      continue;
    }
    if (K.type == KType::SORT) {
      const Node& s = P.nodes[K.sel];
      K.count = s.shape[0];
      K.rows = s.shape[1];
      int bits = 0;
      while ((1LL << bits) < K.rows) ++bits;
      K.passes = std::max(1, (bits + 7) / 8);
      K.tiles = (K.count + 1023) / 1024;
      K.keys = Lw.new_buffer(Storage::Arena, K.count * 4, -1);
      K.vals = Lw.new_buffer(Storage::Arena, K.count * 4, -1);
      K.tmp_keys = Lw.new_buffer(Storage::Arena, K.count * 4, -1);
      K.tmp_vals = Lw.new_buffer(Storage::Arena, K.count * 4, -1);
      K.counts = Lw.new_buffer(Storage::Arena, 256 * (K.tiles + 1) * 4, -1);
      K.rstart = Lw.new_buffer(Storage::Arena, K.rows * 4, -1);
      K.rend = Lw.new_buffer(Storage::Arena, K.rows * 4, -1);
      K.out = P.info[K.sel].buf;  // the index buffer
      K.reads = {K.out};
      K.writes = {K.keys, K.vals, K.tmp_keys, K.tmp_vals, K.counts, K.rstart, K.rend};
      K.describe = "sort selection node " + std::to_string(K.sel) + " count=" +
                   std::to_string(K.count) + " rows=" + std::to_string(K.rows);
      sort_index[(int)i] = (int)P.kernels.size();
      P.kernels.push_back(K);
      continue;
    }
    // A first, discarded emission learns whether the kernel carries a
    // tolerance; it is then emitted for real, relaxed if it does.
    bool carries_tolerance = false;
    if (K.type == KType::EW || K.type == KType::ROW) {
      const Kernel saved = K;
      const size_t buffers = P.buffers.size(), nfinals = finals.size();
      Emitter probe(P, K, (int)P.kernels.size());
      if (K.type == KType::EW) emit_ew(P, K, probe);
      else emit_row(P, K, probe, Lw, finals);
      carries_tolerance = !probe.exact && !probe.exact_member_seen && !P.bf16;
      K = saved;
      P.buffers.resize(buffers);
      finals.resize(nfinals);
    }
    Emitter E(P, K, (int)P.kernels.size());
    E.relaxed = carries_tolerance;
    // after the emission: which of the kernel's stored values carry a tolerance
    auto note_tolerance = [&](const Emitter& done) {
      for (size_t m = 0; m < K.members.size(); ++m) {
        const Member& mm = K.members[m];
        const bool reduction = mm.type == MemberType::ROW_SUM || mm.type == MemberType::ROW_MAX ||
                               mm.type == MemberType::COL_SUM || mm.type == MemberType::ALL_SUM;
        if (reduction || done.tainted_members.count((int)m)) P.tolerance_nodes.insert(mm.node);
      }
    };
    switch (K.type) {
      case KType::EW: emit_ew(P, K, E); break;
      case KType::ROW: emit_row(P, K, E, Lw, finals); break;
      case KType::REDUCE: emit_reduce(P, K, E); break;
      case KType::SCATTER: {
        int sk = sort_index.at(P.sort_of.at(P.nodes[K.node].operands[1]));
        K.sel = sk;
        const Node& sn = P.nodes[K.node];
        const Node& gn = P.nodes[sn.operands[0]];
        const int64_t width = sn.volume() / sn.shape[0];
        K.partial = Lw.new_buffer(Storage::Arena, gn.shape[0] * width * 4, -1);
        emit_scatter(P, K, E, P.kernels[sk]);
        Kernel seg;
        seg.type = KType::SEGSUM;
        seg.node = K.node;
        seg.partial = K.partial;
        seg.final_out = P.info[K.node].buf;
        seg.rstart = P.kernels[sk].rstart;
        seg.rend = P.kernels[sk].rend;
        seg.rows = sn.shape[0];
        seg.final_width = width;
        seg.count = gn.shape[0];
        seg.exact = true;
        finals.push_back(seg);
        break;
      }
      case KType::FOLD: emit_fold(P, K, E); break;
      case KType::PREP: emit_prep(P, K, E); break;
      default: fail("codegen: unexpected kernel type");
    }
    K.exact = E.exact;
    if (K.type == KType::EW || K.type == KType::ROW) note_tolerance(E);
    E.wide = needs_wide(P, K);
    std::ostringstream fn;
    fn << "struct PRM_NAME { void* p[" << std::max<size_t>(1, K.params.size()) << "]; };\n";
    // row kernels run at most four blocks per SM (their grid cap): ask for
    // registers that let all four be resident
    fn << "extern \"C\" __global__ void __launch_bounds__(256"
       << (K.type == KType::ROW ? ", 4" : "") << ") NAME(const PRM_NAME prm) {\n";
    fn << "  typedef " << (E.wide ? "long long" : "int") << " I;\n";
    // launched with programmatic stream serialization: wait for the previous
    // kernels (and their memory) before any access, then let the next launch
    fn << "  asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n";
    fn << "  asm volatile(\"griddepcontrol.launch_dependents;\" ::: \"memory\");\n";
    fn << E.body.str() << "}\n";
    std::string text = fn.str();
    auto it = dedupe.find(text);
    if (it == dedupe.end()) {
      std::string name = "tbk" + std::to_string(dedupe.size());
      std::string src = text;
      for (size_t p; (p = src.find("PRM_NAME")) != std::string::npos;)
        src.replace(p, 8, "P_" + name);
      for (size_t p; (p = src.find("NAME(")) != std::string::npos;) src.replace(p, 4, name);
      all << src << "\n";
      it = dedupe.emplace(text, name).first;
    }
    K.name = it->second;
    K.source.clear();
    for (int b : K.params) {
      const Buffer& bf = P.buffers[b];
      bool written = false;
      for (auto& m : K.members) {
        if (m.type == MemberType::PREP) {
          if (b == m.hi || b == m.lo) written = true;
          continue;
        }
        if (P.info[m.node].buf == b && P.info[m.node].owner == m.node) written = true;
      }
      if (b == K.a_hi || b == K.a_lo) written = true;
      if (bf.storage == Storage::Arena && bf.node < 0 &&
          (K.type == KType::ROW || K.type == KType::SCATTER))
        written = true;
      (written ? K.writes : K.reads).push_back(b);
    }
    if (K.type == KType::SCATTER) K.reads.push_back(P.kernels[K.sel].vals);
    std::ostringstream d;
    static const char* names[] = {"ew", "row", "reduce", "prep", "gemm", "sort", "scatter", "fold", "final", "segsum"};
    d << names[(int)K.type] << " " << K.name << " grid=" << K.grid;
    if (!K.space.empty()) {
      d << " space=[";
      for (size_t j = 0; j < K.space.size(); ++j) d << (j ? "," : "") << K.space[j];
      d << "]";
    }
    d << " members=";
    for (auto& m : K.members)
      d << m.node << (m.type == MemberType::PREP ? "prep" : "")
        << (m.phase ? "p" + std::to_string(m.phase) : "") << (m.reg ? "reg" : "") << " ";
    d << (K.exact ? "exact" : "tolerance");
    if (K.type == KType::PREP)
      d << " value=" << K.node << " [" << K.batch << "," << K.m << "," << K.kp << "]";
    K.describe = d.str();
    P.kernels.push_back(K);
    for (auto& f : finals) {
      f.reads = {f.partial};
      f.writes = {f.final_out};
      if (f.type == KType::SEGSUM) {
        f.reads.push_back(f.rstart);
        f.reads.push_back(f.rend);
        f.describe = "segsum rows=" + std::to_string(f.rows) + " width=" +
                     std::to_string(f.final_width) + " exact";
        P.kernels.push_back(f);
        continue;
      }
      // narrow finals of this row kernel share one launch (8-column blocks)
      Kernel* prev = P.kernels.empty() ? nullptr : &P.kernels.back();
      const bool narrow = (f.final_width + 31) / 32 < SMS;
      if (narrow && prev && prev->type == KType::FINAL && !prev->final_parts.empty() &&
          prev->final_blocks == f.final_blocks && prev->final_parts.size() < 8) {
        prev->final_parts.push_back(f.partial);
        prev->final_outs.push_back(f.final_out);
        prev->final_widths.push_back(f.final_width);
        prev->reads.push_back(f.partial);
        prev->writes.push_back(f.final_out);
        prev->describe += "," + std::to_string(f.final_width);
        continue;
      }
      if (narrow) {
        f.final_parts = {f.partial};
        f.final_outs = {f.final_out};
        f.final_widths = {f.final_width};
      }
      f.describe = "final partials=" + std::to_string(f.final_blocks) + "x" +
                   std::to_string(f.final_width);
      P.kernels.push_back(f);
    }
  }
  P.source = all.str();
  P.exact = true;
  for (auto& k : P.kernels) P.exact = P.exact && k.exact;
  P.fused_nodes = 0;
  for (int n : P.order)
    if (P.info[n].kind == Kind::Expr && !P.info[n].materialized) P.fused_nodes++;
  check_register_members(P);
  plan_arena(P);
  check_arena(P);
  return prog;
}

// payload/bf16.rs:39-55: the nearest bf16 (ties to even, carried into the
// exponent), as an f32; a NaN keeps its top half with a mantissa bit forced on.
float round_bf16(float v) {
  uint32_t bits;
  std::memcpy(&bits, &v, 4);
  const uint32_t out = std::isnan(v) ? ((bits >> 16) | 0x0040u) << 16
                                     : ((bits + 0x7FFFu + ((bits >> 16) & 1u)) >> 16) << 16;
  float r;
  std::memcpy(&r, &out, 4);
  return r;
}

}  // namespace tb
