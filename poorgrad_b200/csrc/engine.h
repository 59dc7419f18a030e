// engine.h -- lowering of a topos compiled plan into a B200 device program.
//
// A plan arrives as node columns (`tb_plan_desc`).  Lowering decides, per
// wanted node, how its value exists on the device:
//   CONST   one scalar known at compile time (constant leaves, `counted`
//           literals, and everything computed only from constants);
//   SEL     a one-hot selection held as an int32 index buffer;
//   LAYOUT  a strided view of a buffer (parameters, inputs, dense leaves,
//           materialized values) -- transpose/permute/narrow/broadcast/
//           reshape/unfold cost nothing;
//   EXPR    an elementwise or index-mapping expression that is either
//           recomputed inside each consuming kernel (virtual) or materialized.
// Materialized values are produced by kernels: fused elementwise groups,
// row-space groups (elementwise + row/column/full reductions in phases),
// GEMM operand preparation + GEMM, scatter-add and fold.  Every kernel body
// except the GEMM core and the index sort is emitted as CUDA C from the
// expression DAG and compiled with NVRTC for sm_100a.
#pragma once

#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "../../include/topos_b200.h"

namespace tb {

constexpr int TB_OP_MAX_ALONG = 100;  // internal: row maximum of LogSumExp/LogSoftmax

struct Node {
  int op = 0;
  int rank = 0;
  int64_t shape[TB_MAX_RANK] = {};
  int operands[2] = {-1, -1};
  int64_t attrs[TB_MAX_RANK] = {};
  int slot = -1;
  int payload = TB_PAYLOAD_NONE;
  float constant = 0.0f;
  int64_t vocab = 0;
  const float* dense = nullptr;
  const int32_t* indices = nullptr;
  bool wanted = false, readable = false;
  int64_t volume() const {
    int64_t v = 1;
    for (int i = 0; i < rank; ++i) v *= shape[i];
    return v;
  }
  std::vector<int64_t> dims() const { return std::vector<int64_t>(shape, shape + rank); }
};

struct Layout {
  int rank = 0;
  int64_t shape[TB_MAX_RANK] = {};
  int64_t stride[TB_MAX_RANK] = {};
  int64_t offset = 0;
};

enum class Kind { None, Const, Sel, Layout, Expr };

// Where a buffer's storage comes from.
enum class Storage { Arena, Parameter, Input, Leaf, InputIndices, LeafIndices };

struct Buffer {
  Storage storage = Storage::Arena;
  int64_t bytes = 0;
  int slot = -1;       // Parameter/Input slot
  int node = -1;       // owning node (materialized value) or source node
  int first = -1;      // first kernel that touches it (arena)
  int last = -1;       // last kernel that touches it (arena)
  bool keep = false;   // readable: lives past the program
  int64_t offset = 0;  // arena offset
};

// PREP: the member's value also written as the tf32 pair of a GEMM operand
// (hi = rna_tf32(x), lo = x - hi) into `hi`/`lo`, in the value's own
// row-major layout (its last axis a multiple of 32, so no padding).
enum class MemberType { EW, ROW_SUM, ROW_MAX, COL_SUM, ALL_SUM, PREP };

struct Member {
  int node;
  MemberType type;
  int phase = 0;
  int hi = -1, lo = -1;  // PREP: operand buffers
  // EW member of a row kernel that no other kernel reads: later phases take
  // it from the thread's registers instead of a store and a reload
  bool reg = false;
};

enum class KType {
  EW,         // flat elementwise group
  ROW,        // row-space group with reductions
  REDUCE,     // generic serial reduction (thread per output)
  PREP,       // a GEMM operand value split into tf32 hi/lo, in its own row-major layout
  GEMM,       // 3xTF32 GEMM over prepared operands
  SORT,       // stable index sort of a selection (scatter)
  SCATTER,    // serial-order scatter-add
  FOLD,       // window fold
  FINAL,      // sum of per-block partials
  SEGSUM      // serial segment sums of a target-ordered scatter source
};

struct Kernel {
  KType type = KType::EW;
  std::vector<Member> members;  // EW / ROW / REDUCE / SCATTER / FOLD
  std::vector<int64_t> space;   // iteration shape (EW/ROW)
  int node = -1;                // REDUCE/SCATTER/FOLD/GEMM: the node computed
  int group = -1;               // EW/ROW: the fusion group it was flushed from
  // generated kernels
  std::string name, source;
  std::vector<int> params;      // buffer ids, in kernel parameter order
  int64_t grid = 1, block = 256;
  int smem = 0;
  bool exact = true;
  // static kernels
  int a_hi = -1, a_lo = -1, b_hi = -1, b_lo = -1, out = -1;  // GEMM buffers
  int64_t batch = 1, m = 0, n = 0, k = 0, kp = 0;
  // GEMM operand layouts (1 = MN-major), row strides and rows per batch entry
  int a_mn = 0, b_mn = 0;
  int64_t a_ld = 0, b_ld = 0, a_rows = 0, b_rows = 0;
  int sel = -1;                 // SORT: selection node; SCATTER: sorted buffers via sort_of
  int keys = -1, vals = -1, tmp_keys = -1, tmp_vals = -1, counts = -1, rstart = -1, rend = -1;
  int64_t count = 0, rows = 0, passes = 0, tiles = 0;
  int partial = -1, final_out = -1;  // FINAL
  int64_t final_blocks = 0, final_width = 0;
  // FINAL of several outputs in one launch (same partial-row count): per entry
  // its partials, output and width
  std::vector<int> final_parts, final_outs;
  std::vector<int64_t> final_widths;
  std::vector<int> reads, writes;    // buffer ids touched (liveness)
  bool side = false;                 // runs on the side stream from the program's start
  std::string describe;
};

struct Info {
  Kind kind = Kind::None;
  float c = 0.0f;          // Const
  int buf = -1;            // Sel: index buffer; Layout: underlying buffer
  Layout lay;              // Layout
  float one = 1.0f;        // Sel
  bool materialized = false;
  int owner = -1;          // node whose buffer `buf` is (Layout views)
  int group = -1;          // open/closed group id that computes it
  int alias = -1;          // LogSumExp/LogSoftmax: value of this synthetic node
  // A readable `0 + y` gradient seed whose value is y's buffer as it stands:
  // y is accumulated from +0 (a product, a scatter-add, a row, column or full
  // sum), so it never holds -0 and adding +0 would change no bit.
  int seed_of = -1;
  int consumers = 0;
  int ops = 0;             // expression size bound for virtual nodes
  std::vector<int> heavy;  // big buffers a virtual expression reads
};

struct Program {
  std::vector<Node> nodes;
  std::vector<Info> info;
  std::vector<Buffer> buffers;
  std::vector<Kernel> kernels;
  std::vector<int> order;  // processing order (synthetic nodes included)
  int64_t arena_bytes = 0, unplanned_bytes = 0, fused_nodes = 0;
  bool exact = true;
  // a bf16 network (payload/bf16.rs): values are bf16 numbers held in f32
  // storage; every operation rounds its result once, accumulations round once
  bool bf16 = false;
  int gemms = 0;
  // stored values a generated kernel computed with a tolerance (transcendental
  // results, reductions and what follows from them): a later kernel that
  // loads one carries the tolerance too
  std::set<int> tolerance_nodes;
  // Side-stream kernels (the leading SORTs) run concurrently with the main
  // kernels before side_join, the first main kernel that uses what they wrote;
  // the main stream waits for them there (-1: no side kernels).
  int side_join = -1;
  int parameter_slots = 0, input_slots = 0;
  std::vector<std::vector<int64_t>> parameter_shapes;
  std::vector<int> input_buffer;   // per input slot: buffer id (dense or indices)
  std::vector<int> input_node;     // per input slot: node index
  std::map<int, int> sort_of;      // selection node -> SORT kernel index
  // engine-backward plans: (scalar root, parameter node) -> gradient node
  std::map<std::pair<int, int>, int> gradient_of;
  std::string source;              // all generated kernels (one NVRTC program)
};

// Lowers a plan descriptor; throws std::runtime_error on malformed input.
std::unique_ptr<Program> lower(const tb_plan_desc* desc);
// payload/bf16.rs:39-55: the nearest bf16 as an f32 (ties to even)
float round_bf16(float v);

}  // namespace tb
