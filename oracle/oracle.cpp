// oracle.cpp -- CPU restatement of the topos interpreter's arithmetic.
//
// TEST INFRASTRUCTURE ONLY.  This file is the parity oracle for the B200
// backend: tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
// it as the checker or as the timed reference-CPU path.  The product
// (poorgrad_b200/, libtopos_b200.so) never links, loads or calls it.
//
// It restates, for f32 payloads, what topos computes when a compiled plan runs
// on its default build (no backend features):
//   * the plan/interpreter node loop (engine/plan.rs:566-622, engine/run.rs:417-526),
//   * each Function's forward (function/*.rs `forward`),
//   * the Tensor arithmetic those forwards call (payload/tensor.rs):
//     elementwise map/zip in logical row-major order (365-510),
//     serial left-fold reductions seeded with the first element (1055-1124),
//     the slice-path GEMM seeded with the first product term, inner steps in
//     ascending order (payload/gemm.rs:140-211),
//     gather / scatter-add from zero in source order (1554-1618),
//     pad / unfold / fold (1292-1463),
//   * scalar semantics of payload/elementary.rs:116-143 (libm expf/logf/tanhf/
//     powf, sqrtf, `f32::max` for maximum, `x >= t` for step).
//   * bf16 networks (payload/bf16.rs): every payload operation rounds its f32
//     result once to bf16; products, sums, folds and scatters accumulate in
//     f32 and round once (tensor.rs:1015-1022, 1055-1093, 1431-1451,
//     1605-1616; gemm.rs:149-161).
// Compiled with -O2 -ffp-contract=off and without fast-math: no contraction,
// no reassociation, exactly as the Rust source is evaluated.
//
// Values are independent of storage representation (payload/tests/
// tensor_tests.rs:1209-1240), so every value is held densely except constants
// (one scalar) and selections (indices), which gather/scatter need.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "../include/topos_b200.h"

namespace {

struct Val {
  int kind = TB_PAYLOAD_DENSE;  // DENSE, CONSTANT or SELECTION
  std::vector<int64_t> shape;
  std::vector<float> data;      // DENSE
  float c = 0.0f;               // CONSTANT value / SELECTION one
  std::vector<int32_t> idx;     // SELECTION
  int64_t vocab = 0;

  int64_t volume() const {
    int64_t v = 1;
    for (auto e : shape) v *= e;
    return v;
  }
  float get(int64_t i) const {
    switch (kind) {
      case TB_PAYLOAD_CONSTANT: return c;
      case TB_PAYLOAD_SELECTION: return (i % vocab) == idx[i / vocab] ? c : 0.0f;
      default: return data[i];
    }
  }
};

// `f32::max` (elementary.rs:137-139): the non-NaN argument when one is NaN;
// otherwise the larger, the first argument on ties.
inline float fmax_ref(float a, float b) {
  if (std::isnan(a)) return b;
  if (std::isnan(b)) return a;
  return (b > a) ? b : a;
}

// Element type of the running plan: a bf16 network rounds each payload
// operation's f32 result once (payload/bf16.rs:131-170, 206-257) and each
// accumulation (sums, folds, scatters, products) once at its end.
thread_local bool g_bf16 = false;

// payload/bf16.rs:39-55: the nearest bf16 with ties to even, carried into the
// exponent; a NaN keeps its top half with a mantissa bit forced on.
inline float round_bf16(float v) {
  uint32_t bits;
  std::memcpy(&bits, &v, 4);
  uint32_t out;
  if (std::isnan(v)) {
    out = ((bits >> 16) | 0x0040u) << 16;
  } else {
    out = ((bits + 0x7FFFu + ((bits >> 16) & 1u)) >> 16) << 16;
  }
  float r;
  std::memcpy(&r, &out, 4);
  return r;
}

// One payload result in the running element type.
inline float el(float v) { return g_bf16 ? round_bf16(v) : v; }

Val dense(std::vector<int64_t> shape) {
  Val v;
  v.kind = TB_PAYLOAD_DENSE;
  v.shape = std::move(shape);
  v.data.assign(v.volume(), 0.0f);
  return v;
}

Val constant(std::vector<int64_t> shape, float c) {
  Val v;
  v.kind = TB_PAYLOAD_CONSTANT;
  v.shape = std::move(shape);
  v.c = c;
  return v;
}

std::vector<int64_t> node_shape(const tb_node& n) {
  return std::vector<int64_t>(n.shape, n.shape + n.rank);
}

template <class F>
Val map1(const Val& a, F f) {
  if (a.kind == TB_PAYLOAD_CONSTANT) return constant(a.shape, el(f(a.c)));
  Val out = dense(a.shape);
  for (int64_t i = 0; i < out.volume(); ++i) out.data[i] = el(f(a.get(i)));
  return out;
}

template <class F>
Val zip(const Val& a, const Val& b, F f) {
  if (a.shape != b.shape) throw std::runtime_error("tensors have different shapes");
  if (a.kind == TB_PAYLOAD_CONSTANT && b.kind == TB_PAYLOAD_CONSTANT)
    return constant(a.shape, el(f(a.c, b.c)));
  Val out = dense(a.shape);
  for (int64_t i = 0; i < out.volume(); ++i) out.data[i] = el(f(a.get(i), b.get(i)));
  return out;
}

void split3(const std::vector<int64_t>& shape, int axis, int64_t& outer, int64_t& extent,
            int64_t& inner) {
  outer = 1;
  inner = 1;
  for (int i = 0; i < axis; ++i) outer *= shape[i];
  extent = shape[axis];
  for (size_t i = axis + 1; i < shape.size(); ++i) inner *= shape[i];
}

std::vector<int64_t> without(const std::vector<int64_t>& s, int axis) {
  std::vector<int64_t> r;
  for (int i = 0; i < (int)s.size(); ++i)
    if (i != axis) r.push_back(s[i]);
  return r;
}

// payload/tensor.rs:1073-1093
Val sum_along(const Val& a, int axis) {
  int64_t outer, extent, inner;
  split3(a.shape, axis, outer, extent, inner);
  Val out = dense(without(a.shape, axis));
  for (int64_t o = 0; o < outer; ++o)
    for (int64_t in = 0; in < inner; ++in) {
      float total = a.get((o * extent + 0) * inner + in);
      for (int64_t s = 1; s < extent; ++s) total = total + a.get((o * extent + s) * inner + in);
      out.data[o * inner + in] = el(total);
    }
  return out;
}

// payload/tensor.rs:1104-1124
Val max_along(const Val& a, int axis) {
  int64_t outer, extent, inner;
  split3(a.shape, axis, outer, extent, inner);
  Val out = dense(without(a.shape, axis));
  for (int64_t o = 0; o < outer; ++o)
    for (int64_t in = 0; in < inner; ++in) {
      float largest = a.get((o * extent + 0) * inner + in);
      for (int64_t s = 1; s < extent; ++s)
        largest = fmax_ref(largest, a.get((o * extent + s) * inner + in));
      out.data[o * inner + in] = largest;
    }
  return out;
}

// payload/tensor.rs:1147-1171 (a view; materialized here)
Val broadcast_along(const Val& a, int axis, const std::vector<int64_t>& ref) {
  if (a.kind == TB_PAYLOAD_CONSTANT) return constant(ref, a.c);
  int64_t outer, extent, inner;
  split3(ref, axis, outer, extent, inner);
  Val out = dense(ref);
  for (int64_t o = 0; o < outer; ++o)
    for (int64_t s = 0; s < extent; ++s)
      for (int64_t in = 0; in < inner; ++in)
        out.data[(o * extent + s) * inner + in] = a.get(o * inner + in);
  return out;
}

// row-major strides of a shape
std::vector<int64_t> strides_of(const std::vector<int64_t>& s) {
  std::vector<int64_t> st(s.size(), 1);
  for (int i = (int)s.size() - 2; i >= 0; --i) st[i] = st[i + 1] * s[i + 1];
  return st;
}

// Materializes a strided reading of `a`: output element at multi-index `m`
// reads a.get(offset + sum m[i]*strides[i]).
Val strided(const Val& a, const std::vector<int64_t>& shape, int64_t offset,
            const std::vector<int64_t>& strides) {
  Val out = dense(shape);
  int64_t vol = out.volume();
  int rank = (int)shape.size();
  std::vector<int64_t> m(rank, 0);
  for (int64_t i = 0; i < vol; ++i) {
    int64_t src = offset;
    for (int d = 0; d < rank; ++d) src += m[d] * strides[d];
    out.data[i] = a.get(src);
    for (int d = rank - 1; d >= 0; --d) {
      if (++m[d] < shape[d]) break;
      m[d] = 0;
    }
  }
  return out;
}

// Worker threads for the row-parallel GEMM (1 = the interpreter's single
// thread).  Set by oracle_set_threads; the test harness may use every core.
int g_threads = 1;

template <class F>
void parallel_rows(int64_t total_rows, int64_t work, F&& body) {
  const int64_t t = std::min<int64_t>(g_threads, total_rows);
  if (t <= 1 || work * total_rows < (int64_t(1) << 22)) {
    body(0, total_rows);
    return;
  }
  std::vector<std::thread> pool;
  const int64_t per = (total_rows + t - 1) / t;
  for (int64_t i = 0; i < t; ++i) {
    const int64_t a = i * per, b = std::min(total_rows, a + per);
    if (a < b) pool.emplace_back([=, &body]() { body(a, b); });
  }
  for (auto& th : pool) th.join();
}

// payload/tensor.rs:921-1027 and payload/gemm.rs:140-211
Val matmul(const Val& a, const Val& b) {
  int rank = (int)a.shape.size();
  int split = rank - 2;
  int64_t rows = a.shape[split], inner = a.shape[split + 1], cols = b.shape[split + 1];
  int64_t batches = 1;
  std::vector<int64_t> shape;
  for (int i = 0; i < split; ++i) {
    batches *= a.shape[i];
    shape.push_back(a.shape[i]);
  }
  shape.push_back(rows);
  shape.push_back(cols);
  Val out = dense(shape);
  // dense copies make the inner loops plain slices
  std::vector<float> A(a.volume()), B(b.volume());
  for (int64_t i = 0; i < a.volume(); ++i) A[i] = a.get(i);
  for (int64_t i = 0; i < b.volume(); ++i) B[i] = b.get(i);
  // Every output row is its own serial chain, so rows may be computed on
  // several threads (oracle_set_threads) with bit-identical results.
  auto rows_of = [&](int64_t first_row, int64_t last_row) {
    for (int64_t q = first_row; q < last_row; ++q) {
      const int64_t bt = q / rows, r = q % rows;
      const float* Ab = A.data() + bt * rows * inner;
      const float* Bb = B.data() + bt * inner * cols;
      float* acc = out.data.data() + bt * rows * cols + r * cols;
      const float first = Ab[r * inner];
      for (int64_t c = 0; c < cols; ++c) acc[c] = first * Bb[c];
      for (int64_t s = 1; s < inner; ++s) {
        const float av = Ab[r * inner + s];
        const float* brow = Bb + s * cols;
        for (int64_t c = 0; c < cols; ++c) acc[c] = acc[c] + av * brow[c];
      }
    }
  };
  parallel_rows(batches * rows, rows * inner * cols, rows_of);
  for (float& v : out.data) v = el(v);  // f32 accumulators, one rounding
  return out;
}

struct Oracle {
  const tb_plan_desc* desc;
  std::vector<Val> values;
};

Val source_payload(const tb_node& n, const float* dense_ptr, const int32_t* idx_ptr) {
  Val v;
  v.shape = node_shape(n);
  if (n.payload == TB_PAYLOAD_CONSTANT) {
    v.kind = TB_PAYLOAD_CONSTANT;
    v.c = el(n.constant);
  } else if (n.payload == TB_PAYLOAD_SELECTION) {
    v.kind = TB_PAYLOAD_SELECTION;
    v.c = el(n.constant);
    v.vocab = n.shape[1];
    if (!idx_ptr) throw std::runtime_error("selection without indices");
    v.idx.assign(idx_ptr, idx_ptr + n.shape[0]);
  } else {
    v.kind = TB_PAYLOAD_DENSE;
    if (!dense_ptr) throw std::runtime_error("dense source without elements");
    v.data.assign(dense_ptr, dense_ptr + v.volume());
    for (float& e : v.data) e = el(e);  // a bf16 network holds bf16 sources
  }
  return v;
}

Val forward(const tb_node& n, const Val* x, const Val* y) {
  const int64_t* at = n.attrs;
  std::vector<int64_t> shape = node_shape(n);
  switch (n.op) {
    case TB_OP_ADD: return zip(*x, *y, [](float l, float r) { return l + r; });
    case TB_OP_SUB: return zip(*x, *y, [](float l, float r) { return l - r; });
    case TB_OP_MUL: return zip(*x, *y, [](float l, float r) { return l * r; });
    case TB_OP_DIV: return zip(*x, *y, [](float l, float r) { return l / r; });
    case TB_OP_NEG: return map1(*x, [](float v) { return -v; });
    case TB_OP_TANH: return map1(*x, [](float v) { return tanhf(v); });
    case TB_OP_EXP: return map1(*x, [](float v) { return expf(v); });
    case TB_OP_LN: return map1(*x, [](float v) { return logf(v); });
    case TB_OP_SQRT: return map1(*x, [](float v) { return sqrtf(v); });
    case TB_OP_POWF: return zip(*x, *y, [](float l, float r) { return powf(l, r); });
    case TB_OP_MAXIMUM: return zip(*x, *y, [](float l, float r) { return fmax_ref(l, r); });
    case TB_OP_RELU: return map1(*x, [](float v) { return fmax_ref(v, 0.0f); });
    case TB_OP_STEP:
      return zip(*x, *y, [](float l, float r) { return l >= r ? 1.0f : 0.0f; });
    case TB_OP_MATMUL: return matmul(*x, *y);
    case TB_OP_TRANSPOSE: {
      if (x->shape.size() < 2) {
        Val v = *x;
        v.shape = shape;
        return v;
      }
      if (x->kind == TB_PAYLOAD_CONSTANT) return constant(shape, x->c);
      return strided(*x, shape, 0, {1, x->shape[1]});
    }
    case TB_OP_SUM: {  // payload/tensor.rs:1055-1063
      float total = x->get(0);
      for (int64_t i = 1; i < x->volume(); ++i) total = total + x->get(i);
      return constant({}, el(total));
    }
    case TB_OP_SUM_ALONG: return sum_along(*x, (int)at[0]);
    case TB_OP_BROADCAST: return constant(shape, x->get(0));
    case TB_OP_BROADCAST_ALONG: return broadcast_along(*x, (int)at[0], shape);
    case TB_OP_RESHAPE: {
      Val v = *x;
      v.shape = shape;
      if (v.kind == TB_PAYLOAD_SELECTION) {  // a reshaped selection is dense
        Val d = dense(shape);
        for (int64_t i = 0; i < d.volume(); ++i) d.data[i] = x->get(i);
        return d;
      }
      return v;
    }
    case TB_OP_PERMUTE: {
      if (x->kind == TB_PAYLOAD_CONSTANT) return constant(shape, x->c);
      std::vector<int64_t> src = strides_of(x->shape), st(shape.size());
      for (size_t j = 0; j < shape.size(); ++j) st[j] = src[at[j]];
      return strided(*x, shape, 0, st);
    }
    case TB_OP_NARROW: {
      if (x->kind == TB_PAYLOAD_CONSTANT) return constant(shape, x->c);
      std::vector<int64_t> st = strides_of(x->shape);
      return strided(*x, shape, at[1] * st[at[0]], st);
    }
    case TB_OP_UNFOLD: {  // layout.unfold: (count, size) pair at axis
      if (x->kind == TB_PAYLOAD_CONSTANT) return constant(shape, x->c);
      int axis = (int)at[0];
      std::vector<int64_t> src = strides_of(x->shape), st;
      for (int i = 0; i < (int)x->shape.size(); ++i) {
        if (i == axis) {
          st.push_back(src[i] * at[2]);
          st.push_back(src[i] * at[3]);
        } else {
          st.push_back(src[i]);
        }
      }
      return strided(*x, shape, 0, st);
    }
    case TB_OP_PAD: {  // payload/tensor.rs:1292-1330
      int axis = (int)at[0];
      int64_t start = at[1], full = at[2];
      int64_t outer, len, inner;
      split3(x->shape, axis, outer, len, inner);
      Val out = dense(shape);
      int64_t w = 0;
      for (int64_t o = 0; o < outer; ++o)
        for (int64_t p = 0; p < full; ++p)
          for (int64_t in = 0; in < inner; ++in)
            out.data[w++] = (p >= start && p < start + len)
                                ? x->get((o * len + (p - start)) * inner + in)
                                : 0.0f;
      return out;
    }
    case TB_OP_FOLD: {  // payload/tensor.rs:1392-1463
      int axis = (int)at[0];
      int64_t size = at[1], step = at[2], dilation = at[3], extent = at[4];
      int64_t count = x->shape[axis];
      int64_t outer = 1, inner = 1;
      for (int i = 0; i < axis; ++i) outer *= x->shape[i];
      for (size_t i = axis + 2; i < x->shape.size(); ++i) inner *= x->shape[i];
      Val out = dense(shape);
      int64_t w = 0;
      for (int64_t o = 0; o < outer; ++o)
        for (int64_t p = 0; p < extent; ++p)
          for (int64_t in = 0; in < inner; ++in) {
            float total = 0.0f;
            for (int64_t k = 0; k < size; ++k) {
              int64_t reach = k * dilation;
              if (reach > p) break;
              int64_t rest = p - reach;
              if (rest % step != 0) continue;
              int64_t window = rest / step;
              if (window >= count) continue;
              total = total + x->get(((o * count + window) * size + k) * inner + in);
            }
            out.data[w++] = el(total);
          }
      return out;
    }
    case TB_OP_GATHER: {  // payload/tensor.rs:1554-1576
      if (y->kind != TB_PAYLOAD_SELECTION) throw std::runtime_error("gather needs a selection");
      int64_t row = 1;
      for (size_t i = 1; i < x->shape.size(); ++i) row *= x->shape[i];
      Val out = dense(shape);
      for (size_t s = 0; s < y->idx.size(); ++s)
        for (int64_t o = 0; o < row; ++o) out.data[s * row + o] = x->get(y->idx[s] * row + o);
      return out;
    }
    case TB_OP_SCATTER: {  // payload/tensor.rs:1582-1618
      if (y->kind != TB_PAYLOAD_SELECTION) throw std::runtime_error("scatter needs a selection");
      int64_t row = 1;
      for (size_t i = 1; i < x->shape.size(); ++i) row *= x->shape[i];
      Val out = dense(shape);  // zeros
      for (size_t s = 0; s < y->idx.size(); ++s)
        for (int64_t o = 0; o < row; ++o) {
          int64_t p = (int64_t)y->idx[s] * row + o;
          out.data[p] = out.data[p] + x->get(s * row + o);
        }
      for (float& v : out.data) v = el(v);  // f32 accumulators, one rounding
      return out;
    }
    case TB_OP_LOG_SOFTMAX: {  // function/log_softmax.rs:51-65
      int axis = (int)at[0];
      Val peak = broadcast_along(max_along(*x, axis), axis, x->shape);
      Val shifted = zip(*x, peak, [](float l, float r) { return l - r; });
      Val e = map1(shifted, [](float v) { return expf(v); });
      Val normalizer = map1(sum_along(e, axis), [](float v) { return logf(v); });
      Val nb = broadcast_along(normalizer, axis, shifted.shape);
      return zip(shifted, nb, [](float l, float r) { return l - r; });
    }
    case TB_OP_LOG_SUM_EXP: {  // function/log_sum_exp.rs:53-63
      int axis = (int)at[0];
      Val peak = max_along(*x, axis);
      Val shifted = zip(*x, broadcast_along(peak, axis, x->shape),
                        [](float l, float r) { return l - r; });
      Val e = map1(shifted, [](float v) { return expf(v); });
      Val lse = map1(sum_along(e, axis), [](float v) { return logf(v); });
      return zip(peak, lse, [](float l, float r) { return l + r; });
    }
    default: throw std::runtime_error("oracle: unsupported op " + std::to_string(n.op));
  }
}

// Evaluates every wanted node of a plan in index order (`Plan::forward`,
// engine/plan.rs:514-640) in the plan's element type and returns all values.
std::vector<Val> evaluate(const tb_plan_desc* desc, const float* const* params,
                          int32_t param_count, int32_t feed_count, const tb_feed* feeds) {
  if (desc->element != TB_ELEMENT_F32 && desc->element != TB_ELEMENT_BF16)
    throw std::runtime_error("unknown element type");
  g_bf16 = desc->element == TB_ELEMENT_BF16;
  const int64_t n = desc->node_count;
  std::vector<Val> values(n);
  std::vector<const tb_feed*> feed_of;
  for (int32_t f = 0; f < feed_count; ++f) {
    if ((int32_t)feed_of.size() <= feeds[f].slot) feed_of.resize(feeds[f].slot + 1, nullptr);
    feed_of[feeds[f].slot] = &feeds[f];
  }
  // release bookkeeping of forward-only plans is irrelevant to values; the
  // oracle keeps everything so any readable value can be read back.
  for (int64_t i = 0; i < n; ++i) {
    const tb_node& node = desc->nodes[i];
    if (!node.wanted) continue;
    switch (node.op) {
      case TB_OP_LEAF: values[i] = source_payload(node, node.dense, node.indices); break;
      case TB_OP_PARAMETER:
        if (node.slot >= param_count) throw std::runtime_error("missing parameter slot");
        values[i] = source_payload(node, params[node.slot], nullptr);
        values[i].kind = TB_PAYLOAD_DENSE;
        break;
      case TB_OP_INPUT: {
        const tb_feed* f =
            node.slot < (int32_t)feed_of.size() ? feed_of[node.slot] : nullptr;
        tb_node copy = node;
        // a feed replaces the initial payload whole, its kind included
        if (f) copy.payload = f->indices ? TB_PAYLOAD_SELECTION : TB_PAYLOAD_DENSE;
        if (copy.payload == TB_PAYLOAD_NONE) copy.payload = TB_PAYLOAD_DENSE;
        values[i] = source_payload(copy, f ? f->dense : node.dense,
                                   f ? f->indices : node.indices);
        break;
      }
      default: {
        const Val* x = node.operands[0] >= 0 ? &values[node.operands[0]] : nullptr;
        const Val* y = node.operands[1] >= 0 ? &values[node.operands[1]] : nullptr;
        values[i] = forward(node, x, y);
      }
    }
  }
  return values;
}

// ---- the engine's reverse scan (`Run::backward`, engine/run.rs:229-318)

// One forward operation applied to computed values, as the derivative rules
// compose payload methods.
Val apply(int op, const Val* x, const Val* y, const std::vector<int64_t>& shape,
          std::initializer_list<int64_t> attrs = {}) {
  tb_node n{};
  n.op = op;
  n.rank = (int32_t)shape.size();
  for (int i = 0; i < n.rank; ++i) n.shape[i] = shape[i];
  int k = 0;
  for (int64_t a : attrs) n.attrs[k++] = a;
  return forward(n, x, y);
}
Val add(const Val& a, const Val& b) { return apply(TB_OP_ADD, &a, &b, a.shape); }
Val sub(const Val& a, const Val& b) { return apply(TB_OP_SUB, &a, &b, a.shape); }
Val mul(const Val& a, const Val& b) { return apply(TB_OP_MUL, &a, &b, a.shape); }
Val div(const Val& a, const Val& b) { return apply(TB_OP_DIV, &a, &b, a.shape); }
Val neg(const Val& a) { return apply(TB_OP_NEG, &a, nullptr, a.shape); }
Val un(int op, const Val& a) { return apply(op, &a, nullptr, a.shape); }

// function/matmul.rs:89-97: the last two axes exchanged
Val swapped(const Val& v) {
  std::vector<int64_t> s = v.shape;
  const int r = (int)s.size();
  if (r <= 2) {
    std::reverse(s.begin(), s.end());
    return apply(TB_OP_TRANSPOSE, &v, nullptr, s);
  }
  std::swap(s[r - 2], s[r - 1]);
  tb_node n{};
  n.op = TB_OP_PERMUTE;
  n.rank = r;
  for (int i = 0; i < r; ++i) {
    n.shape[i] = s[i];
    n.attrs[i] = i;
  }
  std::swap(n.attrs[r - 2], n.attrs[r - 1]);
  return forward(n, &v, nullptr);
}

Val matmul_of(const Val& a, const Val& b) {
  std::vector<int64_t> s = a.shape;
  s.back() = b.shape.back();
  return apply(TB_OP_MATMUL, &a, &b, s);
}

// The cotangents of one node (function/*.rs `backward`); an absent
// cotangent (a shape-only or selection operand, `Step`) is `present = false`.
void cotangents(const tb_node& n, const Val* x, const Val* y, const Val& out, const Val& g,
                Val c[2], bool present[2]) {
  const int64_t* at = n.attrs;
  present[0] = present[1] = false;
  auto one = [](const Val& v) { return constant(v.shape, 1.0f); };
  auto give = [&](int k, Val v) {
    c[k] = std::move(v);
    present[k] = true;
  };
  switch (n.op) {
    case TB_OP_ADD: give(0, g); give(1, g); return;                     // add.rs
    case TB_OP_SUB: give(0, g); give(1, neg(g)); return;                // sub.rs
    case TB_OP_MUL: give(0, mul(g, *y)); give(1, mul(g, *x)); return;   // mul.rs
    case TB_OP_DIV:                                                     // div.rs:46-52
      give(0, div(g, *y));
      give(1, neg(div(mul(g, out), *y)));
      return;
    case TB_OP_NEG: give(0, neg(g)); return;
    case TB_OP_TANH: give(0, mul(g, sub(one(out), mul(out, out)))); return;  // tanh.rs:41-44
    case TB_OP_EXP: give(0, mul(g, out)); return;
    case TB_OP_LN: give(0, div(g, *x)); return;
    case TB_OP_SQRT: give(0, div(g, add(out, out))); return;           // sqrt.rs:43-45
    case TB_OP_POWF: {                                                 // powf.rs:48-54
      Val lowered = sub(*y, one(*y));
      give(0, mul(mul(g, *y), apply(TB_OP_POWF, x, &lowered, x->shape)));
      give(1, mul(mul(g, out), un(TB_OP_LN, *x)));
      return;
    }
    case TB_OP_MAXIMUM: {                                              // maximum.rs:45-51
      Val winners = apply(TB_OP_STEP, x, y, x->shape);
      give(0, mul(g, winners));
      give(1, mul(g, sub(one(winners), winners)));
      return;
    }
    case TB_OP_RELU: {                                                 // relu.rs
      Val zero = constant(x->shape, 0.0f);
      give(0, mul(g, apply(TB_OP_STEP, x, &zero, x->shape)));
      return;
    }
    case TB_OP_STEP: return;
    case TB_OP_MATMUL:                                                 // matmul.rs
      give(0, matmul_of(g, swapped(*y)));
      give(1, matmul_of(swapped(*x), g));
      return;
    case TB_OP_TRANSPOSE: give(0, apply(TB_OP_TRANSPOSE, &g, nullptr, x->shape)); return;
    case TB_OP_SUM: give(0, apply(TB_OP_BROADCAST, &g, x, x->shape)); return;
    case TB_OP_SUM_ALONG: give(0, apply(TB_OP_BROADCAST_ALONG, &g, x, x->shape, {at[0]})); return;
    case TB_OP_BROADCAST: {                                            // broadcast.rs
      Val total = apply(TB_OP_SUM, &g, nullptr, {});
      give(0, apply(TB_OP_BROADCAST, &total, x, x->shape));
      return;
    }
    case TB_OP_BROADCAST_ALONG: give(0, apply(TB_OP_SUM_ALONG, &g, nullptr, x->shape, {at[0]})); return;
    case TB_OP_RESHAPE: give(0, apply(TB_OP_RESHAPE, &g, nullptr, x->shape)); return;
    case TB_OP_PERMUTE: {                                              // permute.rs:53-60
      tb_node p{};
      p.op = TB_OP_PERMUTE;
      p.rank = n.rank;
      for (int i = 0; i < n.rank; ++i) {
        p.shape[i] = x->shape[i];
        p.attrs[at[i]] = i;
      }
      give(0, forward(p, &g, nullptr));
      return;
    }
    case TB_OP_NARROW:
      give(0, apply(TB_OP_PAD, &g, nullptr, x->shape, {at[0], at[1], x->shape[at[0]]}));
      return;
    case TB_OP_PAD:
      give(0, apply(TB_OP_NARROW, &g, nullptr, x->shape, {at[0], at[1], x->shape[at[0]]}));
      return;
    case TB_OP_UNFOLD:
      give(0, apply(TB_OP_FOLD, &g, nullptr, x->shape, {at[0], at[1], at[2], at[3], x->shape[at[0]]}));
      return;
    case TB_OP_FOLD:
      give(0, apply(TB_OP_UNFOLD, &g, nullptr, x->shape, {at[0], at[1], at[2], at[3]}));
      return;
    case TB_OP_GATHER: give(0, apply(TB_OP_SCATTER, &g, y, x->shape, {x->shape[0]})); return;
    case TB_OP_SCATTER: give(0, apply(TB_OP_GATHER, &g, y, x->shape)); return;
    case TB_OP_LOG_SOFTMAX: {                                          // log_softmax.rs
      std::vector<int64_t> reduced = without(g.shape, (int)at[0]);
      Val rows = apply(TB_OP_SUM_ALONG, &g, nullptr, reduced, {at[0]});
      Val total = apply(TB_OP_BROADCAST_ALONG, &rows, &g, g.shape, {at[0]});
      give(0, sub(g, mul(un(TB_OP_EXP, out), total)));
      return;
    }
    case TB_OP_LOG_SUM_EXP: {                                          // log_sum_exp.rs
      Val spread = apply(TB_OP_BROADCAST_ALONG, &out, x, x->shape, {at[0]});
      Val probabilities = un(TB_OP_EXP, sub(*x, spread));
      give(0, mul(apply(TB_OP_BROADCAST_ALONG, &g, x, x->shape, {at[0]}), probabilities));
      return;
    }
  }
  throw std::runtime_error("oracle: no derivative rule for op " + std::to_string(n.op));
}

// engine/run.rs:264-317: zero gradients, a `one_like` seed at the scalar
// root, one reverse scan that marks ancestors as it goes, and `g = g + c`
// per present cotangent.
std::vector<Val> reverse_scan(const tb_plan_desc* desc, const std::vector<Val>& values,
                              int64_t root) {
  if (root < 0 || root >= desc->node_count || desc->nodes[root].rank != 0)
    throw std::runtime_error("backward requires a scalar target; reduce it with `sum` first");
  std::vector<Val> grads(root + 1);
  for (int64_t i = 0; i <= root; ++i) grads[i] = constant(node_shape(desc->nodes[i]), 0.0f);
  grads[root] = constant({}, 1.0f);
  std::vector<char> ancestor(root + 1, 0);
  ancestor[root] = 1;
  for (int64_t i = root; i >= 0; --i) {
    if (!ancestor[i]) continue;
    const tb_node& n = desc->nodes[i];
    if (n.op == TB_OP_LEAF || n.op == TB_OP_PARAMETER || n.op == TB_OP_INPUT) continue;
    const int64_t lx = n.operands[0], ly = n.operands[1];
    Val c[2];
    bool present[2];
    cotangents(n, lx >= 0 ? &values[lx] : nullptr, ly >= 0 ? &values[ly] : nullptr, values[i],
               grads[i], c, present);
    const int64_t links[2] = {lx, ly};
    for (int k = 0; k < 2; ++k) {
      if (!present[k] || links[k] < 0) continue;
      ancestor[links[k]] = 1;
      grads[links[k]] = add(grads[links[k]], c[k]);
    }
  }
  return grads;
}

thread_local std::string g_error;

}  // namespace

extern "C" {

const char* oracle_last_error(void) { return g_error.c_str(); }

// Runs a compiled plan on the CPU (`Plan::forward`, engine/plan.rs:514-640).
// params[slot] are host f32 arrays; feeds override Input payloads; the values of
// `read_nodes` are written row-major into `outputs[i]`.
int oracle_run(const tb_plan_desc* desc, const float* const* params, int32_t param_count,
               int32_t feed_count, const tb_feed* feeds, int32_t read_count,
               const int64_t* read_nodes, float* const* outputs) {
  try {
    std::vector<Val> values = evaluate(desc, params, param_count, feed_count, feeds);
    for (int32_t r = 0; r < read_count; ++r) {
      const Val& v = values[read_nodes[r]];
      for (int64_t i = 0; i < v.volume(); ++i) outputs[r][i] = v.get(i);
    }
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
}

// `Run::backward(root)` then `Gradients::of(node)` for each of `nodes`
// (engine/run.rs:229-318) over the plan's forward values: the engine's own
// reverse scan, against which recorded-gradient plans close bitwise.
int oracle_backward(const tb_plan_desc* desc, const float* const* params, int32_t param_count,
                    int32_t feed_count, const tb_feed* feeds, int64_t root, int32_t count,
                    const int64_t* nodes, float* const* outputs) {
  try {
    std::vector<Val> values = evaluate(desc, params, param_count, feed_count, feeds);
    std::vector<Val> grads = reverse_scan(desc, values, root);
    for (int32_t r = 0; r < count; ++r) {
      if (nodes[r] < 0 || nodes[r] >= desc->node_count)
        throw std::runtime_error("gradient of a node outside the plan");
      const Val v = nodes[r] <= root ? grads[nodes[r]]
                                     : constant(node_shape(desc->nodes[nodes[r]]), 0.0f);
      for (int64_t i = 0; i < v.volume(); ++i) outputs[r][i] = v.get(i);
    }
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
}

// The interpreter's serial-order GEMM alone (payload/gemm.rs:140-211) over
// dense row-major operands: the CPU baseline of the GEMM configs.
void oracle_set_threads(int threads) { g_threads = threads < 1 ? 1 : threads; }

void oracle_gemm(const float* a, const float* b, float* c, int64_t m, int64_t k, int64_t n) {
  parallel_rows(m, k * n, [&](int64_t r0, int64_t r1) {
  for (int64_t r = r0; r < r1; ++r) {
    float* acc = c + r * n;
    const float first = a[r * k];
    for (int64_t j = 0; j < n; ++j) acc[j] = first * b[j];
    for (int64_t s = 1; s < k; ++s) {
      const float av = a[r * k + s];
      const float* brow = b + s * n;
      for (int64_t j = 0; j < n; ++j) acc[j] = acc[j] + av * brow[j];
    }
  }
  });
}

// libm scalar maps of payload/elementary.rs:116-143, for ulp measurements.
// `Bf16::from_f32(x).to_f32()` per element (payload/bf16.rs:39-55).
void oracle_round_bf16(const float* in, int64_t count, float* out) {
  for (int64_t i = 0; i < count; ++i) out[i] = round_bf16(in[i]);
}

void oracle_map(int32_t op, const float* in, int64_t count, float* out) {
  for (int64_t i = 0; i < count; ++i) {
    float v = in[i];
    switch (op) {
      case TB_OP_EXP: out[i] = expf(v); break;
      case TB_OP_LN: out[i] = logf(v); break;
      case TB_OP_SQRT: out[i] = sqrtf(v); break;
      case TB_OP_TANH: out[i] = tanhf(v); break;
      default: out[i] = v;
    }
  }
}

}  // extern "C"
