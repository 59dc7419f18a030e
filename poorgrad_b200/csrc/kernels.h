// kernels.h -- host launchers of the hand-written (non-emitted) kernels.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace tb {

// Stable sort of selection indices by target row, then per-row segments
// [rstart[r], rend[r]) of source positions in ascending source order.
void launch_selection_sort(const int* indices, int* keys, int* vals, int* tmp_keys,
                           int* tmp_vals, int* counts, int* rstart, int* rend, int64_t count,
                           int64_t rows, int passes, int64_t tiles, cudaStream_t stream);

// out[j] = part[0][j] + part[1][j] + ... (ascending block order).
void launch_final_sum(const float* part, float* out, int64_t blocks, int64_t width,
                      cudaStream_t stream);

// Up to kFinalSetMax narrow column finals sharing a partial-row count, one
// launch: entry e owns blocks [start[e], start[e + 1]), 8 columns each.
constexpr int kFinalSetMax = 8;
struct FinalSet {
  const float* part[kFinalSetMax];
  float* out[kFinalSetMax];
  int64_t width[kFinalSetMax];
  int start[kFinalSetMax + 1];
  int count;
};
void launch_final_sum_multi(const FinalSet& set, int64_t blocks, cudaStream_t stream);

// out[r, c] = 0 + perm[rstart[r], c] + ... + perm[rend[r]-1, c] (ascending rows);
// `count` (the number of source rows) selects the variant for long segments.
void launch_segment_sum(const float* perm, const int* rstart, const int* rend, float* out,
                        int64_t rows, int64_t width, int64_t count, cudaStream_t stream);

// A prepared GEMM operand: tf32 pairs (hi = rna_tf32(x), lo = x - hi) laid out
// [batch][rows][ld] floats.  K-major: a row per output row (M for A, N for B),
// the reduction index contiguous (ld = kp, zero-padded).  MN-major: a row per
// reduction index (rows = K, no padding needed), the output index contiguous
// (ld >= M or N, a multiple of 32).  A is M x K, B is given as N x K.
// A raw operand has no lo: `hi` holds the f32 values themselves, in the same
// layout (K-major rows then hold all kp reduction indices, ld >= kp), and the
// GEMM splits them into the pair on the way in.  The tcgen05 path takes a raw
// A only (it declines a raw B); the SIMT path takes either.
struct Operand {
  const float* hi = nullptr;
  const float* lo = nullptr;  // nullptr: raw f32 operand
  int mn = 0;        // 0: K-major, 1: MN-major
  int64_t ld = 0;    // floats between consecutive rows
  int64_t rows = 0;  // rows per batch entry
};
inline Operand k_major(const float* hi, const float* lo, int64_t rows, int64_t kp) {
  Operand o;
  o.hi = hi;
  o.lo = lo;
  o.ld = kp;
  o.rows = rows;
  return o;
}

// Scratch of the tcgen05 path's stream-K schedule, owned by the caller (one per
// stream of work: a plan instance): a workspace of kStreamKMaxCtas tiles of
// 128 x 256 floats and kStreamKMaxCtas * 8 flags, zero before the first launch
// (every launch leaves them zero).  Without it, tiles are walked whole.
constexpr int kStreamKMaxCtas = 160;
struct StreamK {
  float* workspace = nullptr;
  int* flags = nullptr;
};
constexpr size_t kStreamKWorkspaceBytes = (size_t)kStreamKMaxCtas * 128 * 256 * 4;
constexpr size_t kStreamKFlagBytes = (size_t)kStreamKMaxCtas * 8 * 4;

// C[b] = (Ahi+Alo)[b] . (Bhi+Blo)[b]^T over prepared operands; the tcgen05 path
// (split-K into `partial` when splits > 1; stream-K with `sk`), else a SIMT path.
void launch_gemm(const Operand& a, const Operand& b, float* c, float* partial, int splits,
                 int64_t batch, int64_t m, int64_t n, int64_t kp, cudaStream_t stream,
                 const StreamK* sk = nullptr);
// The SIMT path alone (tests compare the two).
void launch_gemm_simt(const Operand& a, const Operand& b, float* c, int64_t batch, int64_t m,
                      int64_t n, int64_t kp, cudaStream_t stream);
// The tcgen05 path; returns false when the shape or alignment is not served.
bool launch_gemm_tcgen05_split(const Operand& a, const Operand& b, float* c, float* partial,
                               int splits, int64_t batch, int64_t m, int64_t n, int64_t kp,
                               cudaStream_t stream, const StreamK* sk = nullptr);
// Turns the stream-K schedule on or off (tests compare the two).
void set_gemm_stream_k(int on);
// 2-D tensor map over row-major f32 [rows][width] (width a multiple of 4), no
// swizzle, boxes of box_cols x box_rows, zero fill outside; false if refused.
bool encode_rows_f32(CUtensorMap* map, const float* base, int64_t width, int64_t rows,
                     int box_cols, int box_rows);
// Error code recorded by a segment-sum kernel whose bounded wait expired (0 = none).
int segment_error();
// Tile width (32, 64, 128 or 256) the tcgen05 path uses for a shape; a test may force one.
int gemm_tile_n(int64_t batch, int64_t m, int64_t n, int64_t kp);
void set_gemm_tile_n(int tile);
// Split-K factor the tcgen05 path uses for a shape (1 = no split).
int gemm_splits(int64_t batch, int64_t m, int64_t n, int64_t kp);
// Error code recorded by a tcgen05 GEMM whose bounded wait expired (0 = none).
int gemm_error();
// Sets the thread-local message returned by tb_last_error().
void set_last_error(const char* message);
// Whether an earlier runtime failure poisoned the library.
bool poisoned();
// Records a runtime failure of a per-task face: the library answers
// TB_POISONED from then on (backend/cuda/kernels/mod.rs:94-105).
void poison_library(const char* why);
// Selects the GEMM engine: 0 = automatic, 1 = SIMT only, 2 = tcgen05 only.
void set_gemm_engine(int engine);
int gemm_engine();

struct OptEntry {
  float* p;
  const float* g;
  float* m;
  float* v;
  int64_t count;
  int64_t start;
  int32_t decay;
  int32_t pad;
};

// out[i] = the pairwise tree of `tree_sum` over shards[0..n) of element i, where
// shard s is g[s * count + i]: adjacent pairs summed left + right, an odd last
// shard carried up, until one remains (n <= 64).
void launch_tree_sum(const float* g, int shards, int64_t count, float* out, cudaStream_t stream);

// Per-step optimizer scalars: s[0]=beta1^t, s[1]=beta2^t, s[2]=1-beta1^t, s[3]=1-beta2^t.
void launch_adam_scalars(float* s, float beta1, float beta2, bool bf16, cudaStream_t stream);
// One multi-tensor step over all entries (kind: 0 SGD, 1 Adam, 2 AdamW).
void launch_optimizer(const OptEntry* entries, int count, int64_t total, const float* scalars,
                      const float* lr, int kind, float beta1, float beta2, float share1,
                      float share2, float eps, float decay, float gscale, bool bf16,
                      cudaStream_t stream);

}  // namespace tb
