// kernels.cu -- hand-written kernels that are not emitted per plan:
// the stable selection sort and the segment sums behind deterministic
// scatter-add (a TMA-fed folding warp for long segments), the partial-sum
// finalizers of fused column/full reductions, the SIMT GEMM path, the
// pairwise tree sum of the deterministic gradient reduction and the
// multi-tensor optimizer steps.  Every kernel begins with pdl_entry().
#include <cstdio>
#include <cstdlib>

#include <algorithm>

#include "kernels.h"
#include "launch.h"
#include "optimizer_rule.h"

namespace tb {
namespace {

constexpr int TILE = 1024;  // selection entries per warp tile

__global__ void k_sort_init(const int* __restrict__ idx, int* __restrict__ keys,
                            int* __restrict__ vals, int64_t count) {
  pdl_entry();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x) {
    keys[i] = idx[i];
    vals[i] = (int)i;
  }
}

// One block of TILE threads per tile, one item per thread: digit histogram,
// aggregated per warp before the shared-memory atomics.
__global__ void __launch_bounds__(TILE) k_radix_count(const int* __restrict__ keys,
                                                      int* __restrict__ counts, int64_t count,
                                                      int shift, int64_t tiles) {
  pdl_entry();
  __shared__ int hist[256];
  const int64_t tile = blockIdx.x;
  if (threadIdx.x < 256) hist[threadIdx.x] = 0;
  __syncthreads();
  const int64_t i = tile * TILE + threadIdx.x;
  const int lane = threadIdx.x & 31;
  const int digit = i < count ? (keys[i] >> shift) & 255 : 256 + lane;
  const unsigned peers = __match_any_sync(0xffffffffu, digit);
  if (digit < 256 && lane == 31 - __clz(peers)) atomicAdd(&hist[digit], __popc(peers));
  __syncthreads();
  if (threadIdx.x < 256) {
    counts[tile * 256 + threadIdx.x] = hist[threadIdx.x];
    if (hist[threadIdx.x]) atomicAdd(&counts[tiles * 256 + threadIdx.x], hist[threadIdx.x]);
  }
}

// Offsets from the tile-major counts [tiles][256] and the digit totals
// counts[tiles][...] (accumulated by the count kernel): thread d walks the
// tiles with coalesced loads, starting from the exclusive scan of the totals.
__global__ void __launch_bounds__(256) k_scan_digits(int* __restrict__ counts, int64_t tiles) {
  pdl_entry();
  __shared__ int totals[256];
  const int d = threadIdx.x;
  totals[d] = counts[tiles * 256 + d];
  __syncthreads();
  if (d == 0) {
    int acc = 0;
    for (int x = 0; x < 256; ++x) {
      const int v = totals[x];
      totals[x] = acc;
      acc += v;
    }
  }
  __syncthreads();
  int run = totals[d];
  int64_t t = 0;
  for (; t + 8 <= tiles; t += 8) {
    int v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = counts[(t + j) * 256 + d];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      counts[(t + j) * 256 + d] = run;
      run += v[j];
    }
  }
  for (; t < tiles; ++t) {
    const int v = counts[t * 256 + d];
    counts[t * 256 + d] = run;
    run += v;
  }
}

// One block of TILE threads per tile: a stable scatter by digit.  Within a
// warp, equal digits are ranked by lane; across warps, by a per-digit prefix
// over the warps in order -- so items keep their source order.
__global__ void __launch_bounds__(TILE) k_radix_scatter(const int* __restrict__ keys,
                                                        const int* __restrict__ vals,
                                                        int* __restrict__ keys_out,
                                                        int* __restrict__ vals_out,
                                                        const int* __restrict__ offsets,
                                                        int64_t count, int shift, int64_t tiles) {
  pdl_entry();
  __shared__ int warp_count[TILE / 32][256];
  const int64_t tile = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int x = threadIdx.x; x < (TILE / 32) * 256; x += TILE) (&warp_count[0][0])[x] = 0;
  __syncthreads();
  const int64_t i = tile * TILE + threadIdx.x;
  const bool valid = i < count;
  int key = 0, val = 0, digit = 256 + lane;
  if (valid) {
    key = keys[i];
    val = vals[i];
    digit = (key >> shift) & 255;
  }
  const unsigned peers = __match_any_sync(0xffffffffu, digit);
  const int rank = __popc(peers & ((1u << lane) - 1u));
  if (valid && lane == 31 - __clz(peers)) warp_count[warp][digit] = __popc(peers);
  __syncthreads();
  if (threadIdx.x < 256) {
    int run = offsets[tile * 256 + threadIdx.x];
    for (int w = 0; w < TILE / 32; ++w) {
      const int c = warp_count[w][threadIdx.x];
      warp_count[w][threadIdx.x] = run;
      run += c;
    }
  }
  __syncthreads();
  if (valid) {
    const int pos = warp_count[warp][digit] + rank;
    keys_out[pos] = key;
    vals_out[pos] = val;
  }
}

__global__ void k_segments(const int* __restrict__ keys, int* __restrict__ rstart,
                           int* __restrict__ rend, int64_t count) {
  pdl_entry();
  for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < count;
       p += (int64_t)gridDim.x * blockDim.x) {
    const int k = keys[p];
    if (p == 0 || keys[p - 1] != k) rstart[k] = (int)p;
    if (p == count - 1 || keys[p + 1] != k) rend[k] = (int)(p + 1);
  }
}

// CB columns per block: thread t takes column t % CB and every G-th partial row
// starting at t / CB (G = 256 / CB groups); the G group sums are then combined
// in group order (a fixed, deterministic association).  CB = 32 gives each
// warp whole 128-byte rows; CB = 8 (narrow outputs) spreads the partial rows
// over 32 groups and 4x the blocks, 32-byte sectors per group.
template <int CB>
__device__ __forceinline__ void final_sum_body(const float* __restrict__ part,
                                               float* __restrict__ out, int64_t blocks,
                                               int64_t width, int64_t block) {
  constexpr int G = 256 / CB;
  __shared__ float acc_s[G][CB];
  const int col = threadIdx.x % CB, grp = threadIdx.x / CB;
  const int64_t j = block * CB + col;
  float acc = 0.0f;
  bool any = false;
  if (j < width) {
    int64_t b = grp;
    for (; b + 7 * G < blocks; b += 8 * G) {  // eight rows per step: loads first, adds in order
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = part[(b + G * u) * width + j];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        acc = any ? __fadd_rn(acc, v[u]) : v[u];
        any = true;
      }
    }
    for (; b < blocks; b += G) {
      const float v = part[b * width + j];
      acc = any ? __fadd_rn(acc, v) : v;
      any = true;
    }
  }
  acc_s[grp][col] = acc;
  __syncthreads();
  if (grp == 0 && j < width) {
    float t = acc_s[0][col];
    for (int w = 1; w < G && w < blocks; ++w) t = __fadd_rn(t, acc_s[w][col]);
    out[j] = t;
  }
}

// CB columns per block: thread t takes column t % CB and every G-th partial row
// starting at t / CB (G = 256 / CB groups); the G group sums are then combined
// in group order (a fixed, deterministic association).  CB = 32 gives each
// warp whole 128-byte rows; CB = 8 (narrow outputs) spreads the partial rows
// over 32 groups and 4x the blocks, 32-byte sectors per group.
template <int CB>
__global__ void __launch_bounds__(256) k_final_sum(const float* __restrict__ part,
                                                   float* __restrict__ out, int64_t blocks,
                                                   int64_t width) {
  pdl_entry();
  final_sum_body<CB>(part, out, blocks, width, blockIdx.x);
}

// Several narrow finals of one row kernel in one launch: block ranges
// [start[e], start[e + 1]) serve entry e.
__global__ void __launch_bounds__(256) k_final_sum_multi(const FinalSet set, int64_t blocks) {
  pdl_entry();
  int e = 0;
  while (e + 1 < set.count && (int)blockIdx.x >= set.start[e + 1]) ++e;
  final_sum_body<8>(set.part[e], set.out[e], blocks, set.width[e], blockIdx.x - set.start[e]);
}

// One thread per output; the segment's rows are contiguous, loaded 64 at a
// time (many bytes in flight for long segments) and added in ascending order
// from zero.
__global__ void k_segment_sum(const float* __restrict__ perm, const int* __restrict__ rstart,
                              const int* __restrict__ rend, float* __restrict__ out,
                              int64_t rows, int64_t width) {
  pdl_entry();
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < rows * width;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = t / width, c = t % width;
    const int64_t q1 = rend[row];
    int64_t q = rstart[row];
    float acc = 0.0f;
    for (; q + 64 <= q1; q += 64) {
      float v[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) v[j] = perm[(q + j) * width + c];
#pragma unroll
      for (int j = 0; j < 64; ++j) acc = __fadd_rn(acc, v[j]);
    }
    for (; q + 8 <= q1; q += 8) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = perm[(q + j) * width + c];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc = __fadd_rn(acc, v[j]);
    }
    for (; q < q1; ++q) acc = __fadd_rn(acc, perm[q * width + c]);
    out[t] = acc;
  }
}

// Long segments (few target rows, many sources each -- an embedding table of a
// small vocabulary): the per-output chains above would leave most SMs idle.
// One block per (row, 32-column slice).  Warps 1..7 keep a ring of kSegSlots
// chunks of the segment (168 source rows each) in flight with cp.async, so
// the L2 latency is hidden behind kSegSlots - 1 chunks; warp 0 adds each
// landed chunk in ascending order from zero, one lane per column -- the same
// serial fold as k_segment_sum, so the result is bit-identical.
constexpr int kSegRowsPerWarp = 24;
constexpr int kSegStage = 7 * kSegRowsPerWarp;
constexpr int kSegSlots = 6;
constexpr size_t kSegSmem = sizeof(float) * kSegSlots * kSegStage * 32;

__device__ __forceinline__ void cp_async4(float* dst, const float* src, bool valid) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(d), "l"(src),
               "r"(valid ? 4 : 0));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__global__ void __launch_bounds__(256) k_segment_sum_staged(const float* __restrict__ perm,
                                                            const int* __restrict__ rstart,
                                                            const int* __restrict__ rend,
                                                            float* __restrict__ out,
                                                            int64_t width) {
  pdl_entry();
  extern __shared__ float ring[];  // [kSegSlots][kSegStage][32]; lane = column
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row = blockIdx.x;
  const int64_t c = (int64_t)blockIdx.y * 32 + lane;
  const bool live = c < width;
  const int64_t q0 = rstart[row], q1 = rend[row];
  const int64_t chunks = (q1 - q0 + kSegStage - 1) / kSegStage;
  // warp w (1..7) copies its 24 rows of chunk i into slot i % kSegSlots
  auto issue = [&](int64_t i) {
    if (i < chunks) {
      const int64_t base = q0 + i * kSegStage + (warp - 1) * kSegRowsPerWarp;
      float* slot = ring + (i % kSegSlots) * (kSegStage * 32) + (warp - 1) * kSegRowsPerWarp * 32;
#pragma unroll
      for (int j = 0; j < kSegRowsPerWarp; ++j) {
        const bool ok = live && base + j < q1;
        cp_async4(slot + j * 32 + lane, ok ? perm + (base + j) * width + c : perm, ok);
      }
    }
    cp_async_commit();  // an empty group past the end keeps the wait count uniform
  };
  if (warp > 0)
    for (int64_t i = 0; i < kSegSlots - 1; ++i) issue(i);
  float acc = 0.0f;
  for (int64_t i = 0; i < chunks; ++i) {
    if (warp > 0) cp_async_wait<kSegSlots - 2>();  // this warp's copies of chunk i landed
    __syncthreads();  // all of chunk i visible; warp 0 is done with chunk i - 1
    if (warp > 0) {
      issue(i + kSegSlots - 1);  // reuses the slot of chunk i - 1
    } else {
      const int64_t left = q1 - q0 - i * kSegStage;
      const float* slot = ring + (i % kSegSlots) * (kSegStage * 32);
      if (left >= kSegStage) {
#pragma unroll 24
        for (int j = 0; j < kSegStage; ++j) acc = __fadd_rn(acc, slot[j * 32 + lane]);
      } else {
        for (int j = 0; j < left; ++j) acc = __fadd_rn(acc, slot[j * 32 + lane]);
      }
    }
  }
  cp_async_wait<0>();
  if (warp == 0 && live) out[row * width + c] = acc;
}

// Long segments through TMA: one warp per (row, 32-column slice).  Lane 0 keeps
// kSegTmaSlots chunks of the segment in flight (one 32-column x kSegTmaRows
// box each, completing on a per-slot mbarrier); the warp adds each landed
// chunk in ascending row order from zero -- the same serial fold, so the
// result is bit-identical to k_segment_sum.  Rows past the segment (the next
// segment's, or zero fill past the end) are loaded but not added.
constexpr int kSegTmaRows = 256;
constexpr int kSegTmaSlots = 6;
constexpr size_t kSegTmaSmem = (size_t)kSegTmaSlots * kSegTmaRows * 32 * 4 + 128 + 64;
constexpr unsigned long long kSegWaitNs = 2000000000ull;  // 2 s per wait
__device__ int g_segment_error = 0;

__device__ __forceinline__ bool seg_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool seg_wait(uint32_t bar, uint32_t parity) {
  if (seg_try_wait(bar, parity)) return true;
  unsigned long long t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  while (!seg_try_wait(bar, parity)) {
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > kSegWaitNs) return false;
  }
  return true;
}

__global__ void __launch_bounds__(32) k_segment_sum_tma(const __grid_constant__ CUtensorMap map,
                                                        const int* __restrict__ rstart,
                                                        const int* __restrict__ rend,
                                                        float* __restrict__ out,
                                                        int64_t width) {
  pdl_entry();
  extern __shared__ uint8_t seg_raw[];
  float* ring = (float*)(((uintptr_t)seg_raw + 127) & ~(uintptr_t)127);
  uint64_t* full = (uint64_t*)(ring + (size_t)kSegTmaSlots * kSegTmaRows * 32);
  const int lane = threadIdx.x;
  const int64_t row = blockIdx.x;
  const int col0 = (int)blockIdx.y * 32;
  const int64_t c = col0 + lane;
  const int64_t q0 = rstart[row], q1 = rend[row];
  const int64_t chunks = (q1 - q0 + kSegTmaRows - 1) / kSegTmaRows;
  auto bar = [&](int s) { return (uint32_t)__cvta_generic_to_shared(&full[s]); };
  if (lane == 0) {
    for (int s = 0; s < kSegTmaSlots; ++s)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar(s)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  int64_t issued = 0;
  auto issue = [&](int64_t i) {  // lane 0: chunk i into slot i % kSegTmaSlots
    if (i >= chunks) return;
    const int s = (int)(i % kSegTmaSlots);
    const uint32_t dst =
        (uint32_t)__cvta_generic_to_shared(ring + (size_t)s * kSegTmaRows * 32);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar(s)),
                 "r"(kSegTmaRows * 32 * 4)
                 : "memory");
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"((uint64_t)&map), "r"(col0), "r"((int)(q0 + i * kSegTmaRows)), "r"(bar(s))
        : "memory");
    issued = i + 1;
  };
  if (lane == 0)
    for (int64_t i = 0; i < kSegTmaSlots; ++i) issue(i);
  float acc = 0.0f;
  int64_t done = 0;
  for (int64_t i = 0; i < chunks; ++i) {
    const int s = (int)(i % kSegTmaSlots);
    if (!seg_wait(bar(s), (uint32_t)((i / kSegTmaSlots) & 1))) {
      if (lane == 0) atomicExch(&g_segment_error, 1);
      break;
    }
    const float* slot = ring + (size_t)s * kSegTmaRows * 32;
    const int64_t left = q1 - q0 - i * kSegTmaRows;
    if (left >= kSegTmaRows) {
      // software-pipelined: each register is refilled with the row 64 ahead
      // as soon as its value is added, so loads stay ahead of the add chain
      float v[64];
#pragma unroll
      for (int u = 0; u < 64; ++u) v[u] = slot[u * 32 + lane];
#pragma unroll
      for (int jb = 0; jb < kSegTmaRows; jb += 64) {
#pragma unroll
        for (int u = 0; u < 64; ++u) {
          const float x = v[u];
          if (jb + 64 < kSegTmaRows) v[u] = slot[(jb + 64 + u) * 32 + lane];
          acc = __fadd_rn(acc, x);
        }
      }
    } else {
      for (int j = 0; j < left; ++j) acc = __fadd_rn(acc, slot[j * 32 + lane]);
    }
    done = i + 1;
    // the slot is read: order those reads before the copy that refills it
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) issue(i + kSegTmaSlots);
  }
  // after an expired wait, let this warp's copies in flight land (bounded)
  // before the shared memory is released
  issued = __shfl_sync(0xffffffffu, issued, 0);
  for (int64_t i = done; i < issued; ++i)
    if (!seg_wait(bar((int)(i % kSegTmaSlots)), (uint32_t)((i / kSegTmaSlots) & 1))) break;
  if (done == chunks && c < width) out[row * width + c] = acc;
}

// Four consecutive reduction indices k..k+3 of operand row r, as hi + lo
// (exactly the original f32 values), or the values themselves for a raw
// operand (no lo); zero outside the operand.
__device__ __forceinline__ float4 simt_quad(const float* __restrict__ h,
                                            const float* __restrict__ l, int mn, int64_t ld,
                                            int64_t rows, int64_t r, int64_t r_end, int64_t k) {
  float4 q = make_float4(0, 0, 0, 0);
  if (r >= r_end) return q;
  if (!mn) {
    const float4 a = *(const float4*)(h + r * ld + k);
    if (!l) return a;
    const float4 b = *(const float4*)(l + r * ld + k);
    return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
  }
  float v[4];
#pragma unroll
  for (int u = 0; u < 4; ++u)
    v[u] = k + u < rows ? h[(k + u) * ld + r] + (l ? l[(k + u) * ld + r] : 0.0f) : 0.0f;
  return make_float4(v[0], v[1], v[2], v[3]);
}

// SIMT GEMM over prepared operands of either layout: 64x64 tiles, 4x4 per
// thread.  The operands are reassembled as hi + lo (the original f32 values).
__global__ void __launch_bounds__(256) k_gemm_simt(const float* __restrict__ ahi,
                                                   const float* __restrict__ alo, int a_mn,
                                                   int64_t a_ld, int64_t a_rows,
                                                   const float* __restrict__ bhi,
                                                   const float* __restrict__ blo, int b_mn,
                                                   int64_t b_ld, int64_t b_rows,
                                                   float* __restrict__ c, int64_t m, int64_t n,
                                                   int64_t kp) {
  pdl_entry();
  __shared__ float As[16][68];
  __shared__ float Bs[16][68];
  const int64_t b = blockIdx.z;
  const int64_t m0 = (int64_t)blockIdx.y * 64, n0 = (int64_t)blockIdx.x * 64;
  const float* Ah = ahi + b * a_rows * a_ld;
  const float* Al = alo ? alo + b * a_rows * a_ld : nullptr;
  const float* Bh = bhi + b * b_rows * b_ld;
  const float* Bl = blo ? blo + b * b_rows * b_ld : nullptr;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {};
  const int lr = threadIdx.x >> 2;       // 0..63 row within tile
  const int lk = (threadIdx.x & 3) * 4;  // 0,4,8,12
  for (int64_t k0 = 0; k0 < kp; k0 += 16) {
    {
      const float4 v = simt_quad(Ah, Al, a_mn, a_ld, a_rows, m0 + lr, m, k0 + lk);
      As[lk + 0][lr] = v.x;
      As[lk + 1][lr] = v.y;
      As[lk + 2][lr] = v.z;
      As[lk + 3][lr] = v.w;
    }
    {
      const float4 v = simt_quad(Bh, Bl, b_mn, b_ld, b_rows, n0 + lr, n, k0 + lk);
      Bs[lk + 0][lr] = v.x;
      Bs[lk + 1][lr] = v.y;
      Bs[lk + 2][lr] = v.z;
      Bs[lk + 3][lr] = v.w;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
  float* C = c + b * m * n;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = m0 + ty * 4 + i;
    if (r >= m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t col = n0 + tx * 4 + j;
      if (col < n) C[r * n + col] = acc[i][j];
    }
  }
}

template <bool BF16>
__global__ void k_adam_scalars(float* s, float beta1, float beta2) {
  pdl_entry();
  if (threadIdx.x == 0 && blockIdx.x == 0) advance_powers<BF16>(s, beta1, beta2);
}

// Multi-tensor optimizer step: each element follows optimizer_update
// (optimizer_rule.h) in the element type of the parameters.
template <bool BF16>
__global__ void k_optimizer(const OptEntry* __restrict__ entries, int count, int64_t total,
                            const float* __restrict__ s, const float* __restrict__ lr_ptr,
                            int kind, float beta1, float beta2, float share1, float share2,
                            float eps, float decay, float gscale) {
  pdl_entry();
  OptimizerScalars sc;
  sc.kind = kind;
  sc.lr = *lr_ptr;
  sc.beta1 = beta1;
  sc.beta2 = beta2;
  sc.share1 = share1;
  sc.share2 = share2;
  sc.eps = eps;
  sc.decay = decay;
  sc.gscale = gscale;
  sc.c1 = kind ? s[2] : 0.0f;
  sc.c2 = kind ? s[3] : 0.0f;
  // Four consecutive elements per thread: one search of the entry table per
  // four elements (a step to the next entry where a tensor ends among them),
  // and four independent updates in flight.
  constexpr int PER = 4;
  for (int64_t base = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * PER; base < total;
       base += (int64_t)gridDim.x * blockDim.x * PER) {
    int lo = 0, hi = count - 1;
    while (lo < hi) {
      int mid = (lo + hi + 1) >> 1;
      if (entries[mid].start <= base) lo = mid; else hi = mid - 1;
    }
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int64_t i = base + u;
      if (i >= total) break;
      while (lo + 1 < count && entries[lo + 1].start <= i) ++lo;
      const OptEntry& e = entries[lo];
      const int64_t j = i - e.start;
      float p = e.p[j];
      if (kind == 0) {
        float unused = 0.0f;
        optimizer_update<BF16>(p, unused, unused, e.g[j], false, sc);
      } else {
        float m = e.m[j], v = e.v[j];
        optimizer_update<BF16>(p, m, v, e.g[j], e.decay != 0, sc);
        e.m[j] = m;
        e.v[j] = v;
      }
      e.p[j] = p;
    }
  }
}

int engine_from_env() {
  const char* e = getenv("TB_GEMM_ENGINE");
  return e ? atoi(e) : 0;
}
int g_engine = engine_from_env();

}  // namespace

void set_gemm_engine(int engine) { g_engine = engine; }
int gemm_engine() { return g_engine; }

void launch_selection_sort(const int* indices, int* keys, int* vals, int* tmp_keys,
                           int* tmp_vals, int* counts, int* rstart, int* rend, int64_t count,
                           int64_t rows, int passes, int64_t tiles, cudaStream_t stream) {
  int grid = (int)std::min<int64_t>((count + 255) / 256, 148 * 8);
  // start in the buffer pair that makes the last pass land in (keys, vals)
  const bool odd = passes % 2 == 1;
  int* src_k = odd ? tmp_keys : keys;
  int* src_v = odd ? tmp_vals : vals;
  int* dst_k = odd ? keys : tmp_keys;
  int* dst_v = odd ? vals : tmp_vals;
  launch_pdl(k_sort_init, grid, 256, 0, stream, indices, src_k, src_v, count);
  for (int p = 0; p < passes; ++p) {
    const int shift = 8 * p;
    cudaMemsetAsync(counts + tiles * 256, 0, 256 * 4, stream);  // digit totals
    launch_pdl(k_radix_count, (unsigned)tiles, TILE, 0, stream, src_k, counts, count, shift, tiles);
    launch_pdl(k_scan_digits, 1, 256, 0, stream, counts, tiles);
    launch_pdl(k_radix_scatter, (unsigned)tiles, TILE, 0, stream, src_k, src_v, dst_k, dst_v,
               counts, count, shift, tiles);
    std::swap(src_k, dst_k);
    std::swap(src_v, dst_v);
  }
  cudaMemsetAsync(rstart, 0, rows * 4, stream);
  cudaMemsetAsync(rend, 0, rows * 4, stream);  // rows without sources: empty segments
  launch_pdl(k_segments, grid, 256, 0, stream, keys, rstart, rend, count);
}

void launch_segment_sum(const float* perm, const int* rstart, const int* rend, float* out,
                        int64_t rows, int64_t width, int64_t count, cudaStream_t stream) {
  const int64_t slices = (width + 31) / 32;
  CUtensorMap map;
  if (count >= 64 * rows && rows <= 65535 && slices <= 65535 && count < (1LL << 31) &&
      encode_rows_f32(&map, perm, width, count, 32, kSegTmaRows)) {
    static bool sized[256] = {};  // opt in to > 48 KB of dynamic shared memory, per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 256 && !sized[dev]) {
      cudaFuncSetAttribute(k_segment_sum_tma, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kSegTmaSmem);
      sized[dev] = true;
    }
    launch_pdl(k_segment_sum_tma, dim3((unsigned)rows, (unsigned)slices), 32, kSegTmaSmem, stream,
               map, rstart, rend, out, width);
    return;
  }
  if (count >= 64 * rows && rows <= 65535 && slices <= 65535) {  // long segments on average
    static bool sized[256] = {};  // opt in to > 48 KB of dynamic shared memory, per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 256 && !sized[dev]) {
      cudaFuncSetAttribute(k_segment_sum_staged, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kSegSmem);
      sized[dev] = true;
    }
    launch_pdl(k_segment_sum_staged, dim3((unsigned)rows, (unsigned)slices), 256, kSegSmem, stream,
               perm, rstart, rend, out, width);
    return;
  }
  int grid = (int)std::max<int64_t>(1, std::min<int64_t>((rows * width + 255) / 256, 148 * 8));
  launch_pdl(k_segment_sum, grid, 256, 0, stream, perm, rstart, rend, out, rows, width);
}

__global__ void k_tree_sum(const float* __restrict__ g, int shards, int64_t count,
                           float* __restrict__ out) {
  pdl_entry();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x) {
    float v[64];
    for (int s = 0; s < shards; ++s) v[s] = g[(int64_t)s * count + i];
    int n = shards;
    while (n > 1) {
      const int half = n / 2;
      for (int j = 0; j < half; ++j) v[j] = __fadd_rn(v[2 * j], v[2 * j + 1]);
      if (n & 1) v[half] = v[n - 1];
      n = half + (n & 1);
    }
    out[i] = v[0];
  }
}

void launch_tree_sum(const float* g, int shards, int64_t count, float* out, cudaStream_t stream) {
  int grid = (int)std::max<int64_t>(1, std::min<int64_t>((count + 255) / 256, 148 * 8));
  launch_pdl(k_tree_sum, grid, 256, 0, stream, g, shards, count, out);
}

int segment_error() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_segment_error, sizeof(int));
  return v;
}

void launch_final_sum_multi(const FinalSet& set, int64_t blocks, cudaStream_t stream) {
  launch_pdl(k_final_sum_multi, (unsigned)set.start[set.count], 256, 0, stream, set, blocks);
}

void launch_final_sum(const float* part, float* out, int64_t blocks, int64_t width,
                      cudaStream_t stream) {
  if ((width + 31) / 32 >= 148)
    launch_pdl(k_final_sum<32>, (unsigned)((width + 31) / 32), 256, 0, stream, part, out, blocks,
               width);
  else
    launch_pdl(k_final_sum<8>, (unsigned)((width + 7) / 8), 256, 0, stream, part, out, blocks,
               width);
}

void launch_gemm_simt(const Operand& a, const Operand& b, float* c, int64_t batch, int64_t m,
                      int64_t n, int64_t kp, cudaStream_t stream) {
  dim3 grid((unsigned)((n + 63) / 64), (unsigned)((m + 63) / 64), (unsigned)batch);
  launch_pdl(k_gemm_simt, grid, 256, 0, stream, a.hi, a.lo, a.mn, a.ld, a.rows, b.hi, b.lo, b.mn,
             b.ld, b.rows, c, m, n, kp);
}

void launch_gemm(const Operand& a, const Operand& b, float* c, float* partial, int splits,
                 int64_t batch, int64_t m, int64_t n, int64_t kp, cudaStream_t stream,
                 const StreamK* sk) {
  if (g_engine != 1 &&
      launch_gemm_tcgen05_split(a, b, c, partial, splits, batch, m, n, kp, stream, sk))
    return;
  launch_gemm_simt(a, b, c, batch, m, n, kp, stream);
}

void launch_adam_scalars(float* s, float beta1, float beta2, bool bf16, cudaStream_t stream) {
  if (bf16) launch_pdl(k_adam_scalars<true>, 1, 32, 0, stream, s, beta1, beta2);
  else launch_pdl(k_adam_scalars<false>, 1, 32, 0, stream, s, beta1, beta2);
}

void launch_optimizer(const OptEntry* entries, int count, int64_t total, const float* scalars,
                      const float* lr, int kind, float beta1, float beta2, float share1,
                      float share2, float eps, float decay, float gscale, bool bf16,
                      cudaStream_t stream) {
  int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 1023) / 1024, 148 * 8));
  if (bf16)
    launch_pdl(k_optimizer<true>, grid, 256, 0, stream, entries, count, total, scalars, lr, kind,
               beta1, beta2, share1, share2, eps, decay, gscale);
  else
    launch_pdl(k_optimizer<false>, grid, 256, 0, stream, entries, count, total, scalars, lr,
               kind, beta1, beta2, share1, share2, eps, decay, gscale);
}

}  // namespace tb
