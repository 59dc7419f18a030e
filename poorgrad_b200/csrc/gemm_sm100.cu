// gemm_sm100.cu -- 3xTF32 GEMM on the 5th-generation tensor cores (tcgen05).
//
// C[b] = A[b] . B[b]^T over operands prepared as tf32 pairs (hi = rna_tf32(x),
// lo = x - hi): C = Ahi.Bhi + Ahi.Blo + Alo.Bhi, the f32 accumulator held in
// tensor memory (TMEM).  Each operand is K-major (reduction index contiguous)
// or MN-major (output index contiguous; the same prepared buffer then serves a
// product and its transpose).  One CTA computes a 128 x BN tile:
//   warp 0      TMA producer: four tiles per k-block (A hi/lo, B hi/lo) into a
//               STAGES-deep ring guarded by mbarriers.  A K-major tile is one
//               box of BK-float rows; an MN-major tile is one box of 32-wide
//               MN blocks (BK rows of 128 bytes each, 32-byte swizzle atoms);
//   warp 1      MMA issuer: one elected thread issues tcgen05.mma kind::tf32
//               (M=128, N=BN, K=8), three products per k-step (two on the
//               32- and 64-wide tiles, which read B's hi and lo tiles as one
//               2N-wide operand), and commits each stage back to the producer;
//   warps 2..   epilogue (one warpgroup per 128 columns of the tile): every
//               CHUNK k-blocks the tensor-memory partial is read (tcgen05.ld,
//               each warp its TMEM lane quarter) and added in IEEE f32 to
//               register accumulators; the finished tile goes out through
//               per-warp 32 x 32 staging slabs in the 128-byte swizzle, one TMA
//               store each (or one 128-byte row segment per store instruction
//               where the output rows are not 16-byte multiples); warp 2 owns
//               the TMEM allocation.
// The tensor cores accumulate with truncating adders, so an accumulation chain
// of k terms drifts like k ulps; draining the accumulator every CHUNK k-blocks
// (two TMEM buffers, the MMA warp filling one while the epilogue drains the
// other) bounds the chain and keeps the result as accurate as a serial f32 sum.
// The kernel is persistent (one CTA per SM walking the tiles).
// A may also arrive raw: its f32 values in the same layout, where the product
// is bound by memory rather than by the tensor cores.  A stage then holds the
// f32 A tile and B's pair, so more k-blocks fit in flight; the epilogue warps,
// each lane one row of the tile, split the row into hi = rna_tf32(x) and
// lo = x - hi -- the pair a prepared operand holds -- and store both into one
// of four tensor-memory A buffers, from which the MMA reads A.  Half of A's
// bytes cross HBM, and the product is bit for bit the one over the pair.
// Split-K writes ordered partials that a second kernel sums in split order.
// No TMA multicast is used anywhere (operands may live on any GPU's arena).
// Every mbarrier wait is bounded by the global timer: on expiry the kernel
// records an error code, stops issuing work and releases its TMEM.
// Launched with programmatic stream serialization: the kernel waits for its
// predecessors (griddepcontrol.wait) before touching global memory.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <cstdio>
#include <algorithm>
#include <cmath>
#include <mutex>

#include <cstdlib>

#include "kernels.h"
#include "launch.h"

namespace tb {
namespace {

constexpr int BM = 128;

// The two tile shapes.  128 x 128 with 32-float k-blocks (128-byte swizzle,
// 3 stages, one epilogue warpgroup) and 128 x 256 with 16-float k-blocks
// (64-byte swizzle, 4 stages, two epilogue warpgroups); both keep 128 k per
// tensor-memory accumulation chain and about 192 KB of staging.
template <int BN_>
struct Cfg;
template <>
struct Cfg<128> {
  static constexpr int BN = 128, BK = 32, STAGES = 3, CHUNK = 4, GROUPS = 1;
  static constexpr uint64_t SWIZZLE = 2, SBO = 1024;  // 128-byte swizzle
  static constexpr CUtensorMapSwizzle TMA_SWIZZLE = CU_TENSOR_MAP_SWIZZLE_128B;
};
template <>
struct Cfg<256> {
  static constexpr int BN = 256, BK = 16, STAGES = 4, CHUNK = 8, GROUPS = 2;
  static constexpr uint64_t SWIZZLE = 4, SBO = 512;  // 64-byte swizzle
  static constexpr CUtensorMapSwizzle TMA_SWIZZLE = CU_TENSOR_MAP_SWIZZLE_64B;
};
// 128 x 64 for outputs 33 to 64 wide (attention's per-head products): a
// 128-wide tile would double their tensor work; four 48 KB stages.
template <>
struct Cfg<64> {
  static constexpr int BN = 64, BK = 32, STAGES = 4, CHUNK = 4, GROUPS = 1;
  static constexpr uint64_t SWIZZLE = 2, SBO = 1024;  // 128-byte swizzle
  static constexpr CUtensorMapSwizzle TMA_SWIZZLE = CU_TENSOR_MAP_SWIZZLE_128B;
};
// 128 x 32 for outputs at most 32 wide (a 27-symbol head): a 128-wide tile
// would be three quarters padding; five 40 KB stages keep more k-blocks in
// flight for these memory-bound products.
template <>
struct Cfg<32> {
  static constexpr int BN = 32, BK = 32, STAGES = 5, CHUNK = 4, GROUPS = 1;
  static constexpr uint64_t SWIZZLE = 2, SBO = 1024;  // 128-byte swizzle
  static constexpr CUtensorMapSwizzle TMA_SWIZZLE = CU_TENSOR_MAP_SWIZZLE_128B;
};
template <class C>
struct Derived {
  static constexpr int TILE_A = BM * C::BK * 4;
  static constexpr int TILE_B = C::BN * C::BK * 4;
  static constexpr int STAGE_BYTES = 2 * TILE_A + 2 * TILE_B;
  static constexpr int THREADS = 64 + 128 * C::GROUPS;
  // raw A: a stage is the f32 A tile and B's pair; the bytes of the paired
  // layout's stages hold RAW_STAGES of them.  A's pairs live in A_BUFS
  // tensor-memory buffers of 64 columns (hi, then lo) after the accumulators.
  static constexpr int RAW_STAGE_BYTES = TILE_A + 2 * TILE_B;
  static constexpr int RAW_STAGES_FIT = C::STAGES * STAGE_BYTES / RAW_STAGE_BYTES;
  static constexpr int RAW_STAGES = RAW_STAGES_FIT > 8 ? 8 : RAW_STAGES_FIT;
  static constexpr int A_BUFS = 4;
  static constexpr int MAX_STAGES = RAW_STAGES > C::STAGES ? RAW_STAGES : C::STAGES;
  // per epilogue warp: a 32 x 32 float tile in the 128-byte swizzle (16-byte
  // chunk c of row r at chunk c ^ (r % 8)), 1024-byte aligned, so that a TMA
  // store can take it whole and the lanes' row writes and column reads are
  // free of bank conflicts
  static constexpr int EPI_STAGE_BYTES = 32 * 32 * 4;
  static constexpr int SMEM_BYTES =
      C::STAGES * STAGE_BYTES + 1024 + 1024 + 4 * C::GROUPS * EPI_STAGE_BYTES;
  static constexpr int EPI_COLS = C::BN / C::GROUPS;  // 128 columns per epilogue warpgroup
};
constexpr unsigned long long WAIT_NS = 4000000000ull;  // 4 s per wait

__device__ int g_gemm_error = 0;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false (and the error flag set) when the deadline passes.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int code) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long start = now_ns();
  while (!mbar_try(bar, parity)) {
    if (now_ns() - start > WAIT_NS) {
      atomicExch(&g_gemm_error, code);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            int w, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}
// K-major operand tile, swizzled rows of BK floats, 8-row atoms SBO bytes apart.
template <class C>
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;              // leading byte offset (unused for swizzled K-major): 16 B
  d |= (uint64_t)(C::SBO >> 4) << 32;  // stride byte offset between 8-row atoms
  d |= (uint64_t)1 << 46;              // descriptor version for tcgen05
  d |= C::SWIZZLE << 61;               // swizzle mode
  return d;
}
// MN-major operand tile: 32-float (128-byte) MN blocks of BK rows each, `lbo`
// bytes apart.  For 32-bit types the tensor cores read MN-major data only in
// the 128-byte swizzle with 32-byte atoms (32-byte chunks of a 128-byte row
// permuted by the row index mod 4; descriptor layout type 1, the TMA map's
// CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B): 4-row groups of 512 bytes, so one MMA
// k-step (8 rows) advances 1024 bytes.
__device__ __forceinline__ uint64_t smem_desc_mn(uint32_t addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;  // leading byte offset: next MN block
  d |= (uint64_t)(512 >> 4) << 32;             // stride byte offset: next 4-row group
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)1 << 61;  // 128-byte swizzle, 32-byte atoms
  return d;
}
// kind::tf32 instruction descriptor: f32 accumulator, tf32 A and B; bits 15/16
// mark A/B as MN-major.
__host__ __device__ constexpr uint32_t instr_desc(int m, int n, int a_mn, int b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void umma_tf32(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t addr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(addr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// TMA store of a 32 x 32 staging tile to (x, y, plane) of the output map.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int x, int y,
                                             int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
          (uint64_t)map),
      "r"(x), "r"(y), "r"(z), "r"(smem_u32(src))
      : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Offset (in floats) of element (r, c) of a swizzled 32 x 32 staging tile.
__device__ __forceinline__ int stage_at(int r, int c) {
  return r * 32 + ((((c >> 2) ^ (r & 7))) << 2) + (c & 3);
}

// Work item w of tiles_n x tiles_m x (batch * splits).  The faster-varying
// tile index is the one whose operand is smaller, so consecutive work items
// (running concurrently on neighbouring SMs) share the larger operand's tile
// and the smaller operand is what gets re-read from L2.
struct Work {
  int n0, m0, split, batch;
};
template <class C>
__device__ __forceinline__ Work decode(int w, int tiles_n, int tiles_m, int splits, int m_fast) {
  Work r;
  if (m_fast) {
    r.m0 = (w % tiles_m) * BM;
    w /= tiles_m;
    r.n0 = (w % tiles_n) * C::BN;
    w /= tiles_n;
  } else {
    r.n0 = (w % tiles_n) * C::BN;
    w /= tiles_n;
    r.m0 = (w % tiles_m) * BM;
    w /= tiles_m;
  }
  r.split = w % splits;
  r.batch = w / splits;
  return r;
}

// The work of one launch.  Items [0, dp_items) are whole work items (a tile,
// or one split-K slice of a tile) walked data-parallel: CTA b takes items
// b, b + grid, ...  The remaining tiles are walked stream-K: their k-blocks
// form one range of sk_units, cut into `grid` contiguous pieces, one per CTA,
// so every CTA ends the launch at the same point.  A tile cut between CTAs
// is summed by the CTA holding its first k-blocks (the owner; that piece is
// the owner's last), which adds the later pieces in k order from the other
// CTAs' workspace slots (each of them their CTA's first stream-K piece).
struct Sched {
  int tiles_n, tiles_m, splits, split_blocks, k_blocks, m_fast;
  int dp_items;         // whole items walked data-parallel
  long long sk_units;   // k-blocks of the stream-K tiles (0: none)
};
// One piece of work: a tile's k-blocks [kb0, kb0 + nkb).  kind: 0 = the whole
// item, 1 = a later piece of a cut tile (to the workspace), 2 = the first
// piece of a cut tile (its owner).
struct Seg {
  Work t;
  int kb0, nkb, kind;
  long long tile_u0;    // stream-K unit where the owned tile starts
};
struct SegIter {
  int w;
  long long u, u_end;
};
__device__ __forceinline__ long long sk_start(const Sched& s, int cta, int grid) {
  return s.sk_units * cta / grid;
}
__device__ __forceinline__ SegIter seg_begin(const Sched& s) {
  SegIter it;
  it.w = blockIdx.x;
  it.u = sk_start(s, blockIdx.x, gridDim.x);
  it.u_end = sk_start(s, blockIdx.x + 1, gridDim.x);
  return it;
}
template <class C, bool SK>
__device__ __forceinline__ bool seg_next(const Sched& s, SegIter& it, Seg& g) {
  if (it.w < s.dp_items) {
    g.t = decode<C>(it.w, s.tiles_n, s.tiles_m, s.splits, s.m_fast);
    g.kb0 = g.t.split * s.split_blocks;
    g.nkb = min(s.k_blocks, g.kb0 + s.split_blocks) - g.kb0;
    g.kind = 0;
    g.tile_u0 = 0;
    it.w += gridDim.x;
    return true;
  }
  if (SK && it.u < it.u_end) {
    const long long tile = it.u / s.k_blocks;
    const int lo = (int)(it.u - tile * s.k_blocks);
    const int hi = (int)min((long long)s.k_blocks, lo + (it.u_end - it.u));
    g.t = decode<C>(s.dp_items + (int)tile, s.tiles_n, s.tiles_m, 1, s.m_fast);
    g.kb0 = lo;
    g.nkb = hi - lo;
    g.kind = (lo == 0 && hi == s.k_blocks) ? 0 : (lo > 0 ? 1 : 2);
    g.tile_u0 = tile * s.k_blocks;
    it.u += hi - lo;
    return true;
  }
  return false;
}
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// A in tensor memory (tf32, K along the columns), B from shared memory.
__device__ __forceinline__ void umma_tf32_ta(uint32_t tmem, uint32_t a_tmem, uint64_t b,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void tmem_st16(uint32_t addr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(addr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
// Persistent: each CTA walks its pieces of work (Sched); the stage ring and
// the two accumulator buffers carry their phases across pieces, so the
// epilogue of one overlaps the main loop of the next.
template <class C, bool SK, bool RAW>
__global__ void __launch_bounds__(Derived<C>::THREADS, 1)
    k_gemm_tcgen05(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
                   const __grid_constant__ CUtensorMap tb_hi, const __grid_constant__ CUtensorMap tb_lo,
                   const __grid_constant__ CUtensorMap tc, int tma_store,
                   float* __restrict__ out, int m, int n, const Sched sched,
                   long long split_stride, int a_mn, int b_mn,
                   float* __restrict__ sk_ws, int* __restrict__ sk_flags) {
  pdl_entry();
  using D = Derived<C>;
  static_assert(4 * C::GROUPS <= 8, "the stream-K flags hold eight epilogue warps per CTA");
  static_assert(!RAW || C::GROUPS == 1, "raw A needs the one-warpgroup epilogue");
  constexpr int BN = C::BN, BK = C::BK, CHUNK = C::CHUNK;
  constexpr int TILE_A = D::TILE_A, TILE_B = D::TILE_B;
  // stages: [A hi | A lo | B hi | B lo], or with raw A [A f32 | B hi | B lo]
  constexpr int STAGES = RAW ? D::RAW_STAGES : C::STAGES;
  constexpr int STAGE_BYTES = RAW ? D::RAW_STAGE_BYTES : D::STAGE_BYTES;
  constexpr int B_OFF = RAW ? TILE_A : 2 * TILE_A;
  constexpr int A_BUFS = D::A_BUFS;
  // Narrow tiles read B's hi and lo tiles, adjacent in the stage, as one
  // 2N-wide operand: A_hi.[B_hi | B_lo] into columns [0, 2N) and A_lo.B_hi
  // added into [N, 2N) -- two tensor-core instructions per k-step instead of
  // three.  A narrow product costs about as much per instruction as a wide
  // one, so this is a third fewer cycles; the epilogue adds the halves.
  constexpr bool JOINT_B = BN <= 64;
  constexpr uint32_t ACC_W = JOINT_B ? 2 * BN : BN;  // columns of one accumulator buffer
  constexpr uint32_t A_COL0 = 2 * ACC_W;  // tensor-memory column of A buffer 0 (RAW)
  constexpr uint32_t TMEM_COLS = RAW ? 512 : 2 * ACC_W;
  static_assert(!RAW || A_COL0 + 64 * A_BUFS <= TMEM_COLS, "A buffers fit in tensor memory");
  constexpr int EPI_COLS = D::EPI_COLS;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  // barriers and flags after the paired layout's stages (the raw layout's fit inside)
  uint64_t* full = (uint64_t*)(smem + C::STAGES * D::STAGE_BYTES);
  uint64_t* empty = full + D::MAX_STAGES;
  uint64_t* a_full = empty + D::MAX_STAGES;  // [A_BUFS]: A's pair stored in tensor memory (RAW)
  uint64_t* a_empty = a_full + A_BUFS;       // [A_BUFS]: its products done (RAW)
  uint64_t* acc_full = a_empty + A_BUFS;     // [2]: chunk partial ready in TMEM buffer b
  uint64_t* acc_empty = acc_full + 2;        // [2]: TMEM buffer b drained by the epilogue
  uint32_t* tmem_slot = (uint32_t*)(acc_empty + 2);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  float* epi_stage = (float*)(smem + C::STAGES * D::STAGE_BYTES + 1024);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int q = 0; q < A_BUFS; ++q) {
      mbar_init(&a_full[q], 128);
      mbar_init(&a_empty[q], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128 * C::GROUPS);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t g = 0;  // k-blocks issued by this CTA so far
      SegIter it = seg_begin(sched);
      Seg sg;
      while (!*abort_flag && seg_next<C, SK>(sched, it, sg)) {
        const Work t = sg.t;
        const int kb0 = sg.kb0;
        const int nkb = sg.nkb;
        for (int i = 0; i < nkb; ++i, ++g) {
          const int s = g % STAGES;
          const uint32_t round = g / STAGES;
          if (!mbar_wait(&empty[s], (round & 1) ^ 1, 1)) {
            *abort_flag = 1;
            break;
          }
          if (*abort_flag) break;
          uint8_t* base = smem + s * STAGE_BYTES;
          mbar_expect_tx(&full[s], STAGE_BYTES);
          const int kx = (kb0 + i) * BK;
          // raw A: the f32 tile alone (its map is over the values)
          if (!a_mn) {
            tma_load_3d(base, &ta_hi, kx, t.m0, t.batch, &full[s]);
            if (!RAW) tma_load_3d(base + TILE_A, &ta_lo, kx, t.m0, t.batch, &full[s]);
          } else {  // one box: BM/32 MN blocks of BK rows
            tma_load_4d(base, &ta_hi, 0, kx, t.m0 / 32, t.batch, &full[s]);
            if (!RAW) tma_load_4d(base + TILE_A, &ta_lo, 0, kx, t.m0 / 32, t.batch, &full[s]);
          }
          uint8_t* bb = base + B_OFF;
          if (!b_mn) {
            tma_load_3d(bb, &tb_hi, kx, t.n0, t.batch, &full[s]);
            tma_load_3d(bb + TILE_B, &tb_lo, kx, t.n0, t.batch, &full[s]);
          } else {
            tma_load_4d(bb, &tb_hi, 0, kx, t.n0 / 32, t.batch, &full[s]);
            tma_load_4d(bb + TILE_B, &tb_lo, 0, kx, t.n0 / 32, t.batch, &full[s]);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // A in tensor memory is K-major whatever its layout in HBM
      const uint32_t idesc = instr_desc(BM, BN, RAW ? 0 : a_mn, b_mn);
      const uint32_t idesc2 = instr_desc(BM, 2 * BN, RAW ? 0 : a_mn, b_mn);  // JOINT_B
      // operand descriptor of k-step kk: K-major steps 32 bytes along the
      // swizzled row, MN-major steps one 1024-byte atom (8 rows of 128 bytes)
      auto desc_of = [&](uint32_t tile, int mn, int kk) -> uint64_t {
        return mn ? smem_desc_mn(tile + kk * 1024, BK * 128) : smem_desc<C>(tile + kk * 32);
      };
      uint32_t g = 0, gc = 0;  // k-blocks and chunks consumed by this CTA so far
      SegIter it = seg_begin(sched);
      Seg sg;
      while (!*abort_flag && seg_next<C, SK>(sched, it, sg)) {
        const int nkb = sg.nkb;
        const int chunks = (nkb + CHUNK - 1) / CHUNK;
        for (int c = 0; c < chunks && !*abort_flag; ++c, ++gc) {
          const int b = gc & 1;
          if (!mbar_wait(&acc_empty[b], ((gc >> 1) & 1) ^ 1, 4)) {
            *abort_flag = 1;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t acc = tmem + b * ACC_W;
          const int i_end = min(nkb, (c + 1) * CHUNK);
          for (int i = c * CHUNK; i < i_end; ++i, ++g) {
            const int s = g % STAGES;
            const uint32_t round = g / STAGES;
            if (!mbar_wait(&full[s], round & 1, 2)) {
              *abort_flag = 1;
              break;
            }
            // raw A: its pair in tensor-memory buffer g % A_BUFS
            const int qa = (int)(g % A_BUFS);
            if (RAW && !mbar_wait(&a_full[qa], (g / A_BUFS) & 1, 7)) {
              *abort_flag = 1;
              break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
            const uint32_t a_hi = base, a_lo = base + TILE_A;
            const uint32_t b_hi = base + B_OFF, b_lo = b_hi + TILE_B;
            const uint32_t ta = tmem + A_COL0 + 64 * qa;  // hi columns, then lo
#pragma unroll
            for (int kk = 0; kk < BK / 8; ++kk) {
              const uint32_t first = (i > c * CHUNK || kk > 0) ? 1u : 0u;
              const uint64_t dbh = desc_of(b_hi, b_mn, kk), dbl = desc_of(b_lo, b_mn, kk);
              if constexpr (JOINT_B && RAW) {
                umma_tf32_ta(acc, ta + kk * 8, dbh, idesc2, first);
                umma_tf32_ta(acc + BN, ta + 32 + kk * 8, dbh, idesc, 1u);
              } else if constexpr (JOINT_B) {
                const uint64_t dah = desc_of(a_hi, a_mn, kk), dal = desc_of(a_lo, a_mn, kk);
                umma_tf32(acc, dah, dbh, idesc2, first);
                umma_tf32(acc + BN, dal, dbh, idesc, 1u);
              } else if constexpr (RAW) {
                umma_tf32_ta(acc, ta + 32 + kk * 8, dbh, idesc, first);
                umma_tf32_ta(acc, ta + kk * 8, dbl, idesc, 1u);
                umma_tf32_ta(acc, ta + kk * 8, dbh, idesc, 1u);
              } else {
                const uint64_t dah = desc_of(a_hi, a_mn, kk), dal = desc_of(a_lo, a_mn, kk);
                umma_tf32(acc, dal, dbh, idesc, first);
                umma_tf32(acc, dah, dbl, idesc, 1u);
                umma_tf32(acc, dah, dbh, idesc, 1u);
              }
            }
            umma_commit(&empty[s]);
            if (RAW) umma_commit(&a_empty[qa]);
          }
          umma_commit(&acc_full[b]);
        }
      }
    }
  } else {
    // epilogue: warps 2..9; lane quarter warp % 4, column half (warp - 2) / 4
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const int c0 = half * EPI_COLS;
    uint32_t gc = 0;
    bool ok = true;
    const int ew = warp - 2;  // epilogue warp index
    // Raw A: these warps also split A, each lane its row of the tile, into
    // tensor memory.  The conversions run ahead of the drains: before chunk
    // c is drained, every k-block through A_BUFS - 1 past its end is split,
    // so the MMA warp has work while the chunk drains, the next piece's
    // first k-blocks included.  (Splitting k-block g waits for the products
    // of g - A_BUFS, which lie in chunk c or before: no wait goes around.)
    SegIter cit = seg_begin(sched);
    Seg csg;
    bool chave = RAW && seg_next<C, SK>(sched, cit, csg);
    int ci = 0;        // k-blocks of csg split
    uint32_t cg = 0;   // k-blocks split by this CTA
    uint32_t g0 = 0;   // this CTA's k-blocks before the current piece
    auto convert_until = [&](uint32_t target) {
      if constexpr (RAW) {
        static_assert(BK == 32, "a k-block is 32 tensor-memory columns");
        const int r = q * 32 + lane;  // this lane's row of the A tile
        // The stores of one k-block complete while the next is loaded and
        // split: its buffer is released (a_full) only after that, so a store's
        // latency is paid once per call, not once per k-block.
        int pending = -1;  // A buffer whose stores are in flight
        auto release = [&]() {
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&a_full[pending]))
                       : "memory");
          pending = -1;
        };
        while (ok && chave && cg < target) {
          if (ci >= csg.nkb) {
            ci = 0;
            chave = seg_next<C, SK>(sched, cit, csg);
            continue;
          }
          const int s = (int)(cg % STAGES), qa = (int)(cg % A_BUFS);
          if (!mbar_wait(&full[s], (cg / STAGES) & 1, 6) ||
              !mbar_wait(&a_empty[qa], ((cg / A_BUFS) & 1) ^ 1, 8)) {
            ok = false;
            *abort_flag = 1;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const float* at = (const float*)(smem + s * STAGE_BYTES);
          float x[32];
          if (!a_mn) {
            // K-major tile: 128-byte rows, 16-byte chunk j at j ^ (r % 8)
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 v = *(const float4*)(at + stage_at(r, 4 * j));
              x[4 * j] = v.x;
              x[4 * j + 1] = v.y;
              x[4 * j + 2] = v.z;
              x[4 * j + 3] = v.w;
            }
          } else {
            // MN-major tile, unswizzled: [row block][k][32 rows]
#pragma unroll
            for (int j = 0; j < 32; ++j) x[j] = at[((r >> 5) * BK + j) * 32 + (r & 31)];
          }
          uint32_t hi[32], lo[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            // rna_tf32 (the prepared operands' rounding) in integer
            // arithmetic: half a tf32 unit added to the magnitude and the 13
            // low bits cleared -- nearest, ties away from zero, a carry into
            // the exponent rounding up; infinities and NaNs kept
            const uint32_t u = __float_as_uint(x[j]);
            const uint32_t h =
                (u & 0x7f800000u) == 0x7f800000u ? u : ((u + 0x1000u) & 0xffffe000u);
            hi[j] = h;
            lo[j] = __float_as_uint(__fsub_rn(x[j], __uint_as_float(h)));
          }
          if (pending >= 0) release();
          const uint32_t col = tmem + lane_base + A_COL0 + 64 * qa;
          tmem_st16(col, hi);
          tmem_st16(col + 16, hi + 16);
          tmem_st16(col + 32, lo);
          tmem_st16(col + 48, lo + 16);
          pending = qa;
          ++ci;
          ++cg;
        }
        if (pending >= 0) release();
      }
    };
    SegIter it = seg_begin(sched);
    Seg sg;
    while (ok && seg_next<C, SK>(sched, it, sg)) {
      const Work t = sg.t;
      const int nkb = sg.nkb;
      const int chunks = (nkb + CHUNK - 1) / CHUNK;
      float total[EPI_COLS];
#pragma unroll
      for (int j = 0; j < EPI_COLS; ++j) total[j] = 0.0f;
      for (int c = 0; c < chunks; ++c, ++gc) {
        const int b = gc & 1;
        convert_until(g0 + (uint32_t)min(nkb, (c + 1) * CHUNK) + (A_BUFS - 1));
        if (!ok) break;
        if (!mbar_wait(&acc_full[b], (gc >> 1) & 1, 3)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
        for (int gq = 0; gq < EPI_COLS / 16; ++gq) {
          uint32_t r[16];
          tmem_ld16(tmem + lane_base + b * ACC_W + c0 + gq * 16, r);
          if constexpr (JOINT_B) {
            // the chunk's partial: Ahi.Bhi + (Ahi.Blo + Alo.Bhi)
            uint32_t x[16];
            tmem_ld16(tmem + lane_base + b * ACC_W + BN + c0 + gq * 16, x);
#pragma unroll
            for (int j = 0; j < 16; ++j)
              r[j] = __float_as_uint(__fadd_rn(__uint_as_float(r[j]), __uint_as_float(x[j])));
          }
#pragma unroll
          for (int j = 0; j < 16; ++j)
            total[gq * 16 + j] = c == 0 ? __uint_as_float(r[j])
                                        : __fadd_rn(total[gq * 16 + j], __uint_as_float(r[j]));
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&acc_empty[b]))
                     : "memory");
      }
      g0 += nkb;
      if (!ok || *abort_flag) break;
      if (SK && sg.kind == 1) {
        // a later piece of a cut tile: to this CTA's workspace slot, laid out
        // [epilogue warp][column][lane] so that each store writes 128
        // consecutive bytes; then this warp's flag, released at gpu scope.
        // Each epilogue warp hands over its own rows and columns, so no
        // barrier wider than a warp is needed.
        float* slot = sk_ws + (long long)blockIdx.x * (BM * BN) + (long long)ew * EPI_COLS * 32;
#pragma unroll
        for (int j = 0; j < EPI_COLS; ++j) __stcg(slot + j * 32 + lane, total[j]);
        __threadfence();
        __syncwarp();
        if (lane == 0) st_release(&sk_flags[blockIdx.x * 8 + ew], 1);
        continue;
      }
      if (SK && sg.kind == 2) {
        // the owner: add the later pieces in k order, each from the CTA whose
        // stream-K range starts inside this tile (the same epilogue warp there)
        const long long tile_u1 = sg.tile_u0 + sched.k_blocks;
        for (int c = blockIdx.x + 1;
             c < (int)gridDim.x && sk_start(sched, c, gridDim.x) < tile_u1 && ok; ++c) {
          if (sk_start(sched, c + 1, gridDim.x) == sk_start(sched, c, gridDim.x)) continue;
          int* flag = &sk_flags[c * 8 + ew];
          const unsigned long long start = now_ns();
          while (ld_acquire(flag) == 0) {
            if (now_ns() - start > WAIT_NS) {
              atomicExch(&g_gemm_error, 5);
              ok = false;
              break;
            }
          }
          if (!__all_sync(0xffffffffu, ok)) {
            ok = false;
            break;
          }
          const float* slot = sk_ws + (long long)c * (BM * BN) + (long long)ew * EPI_COLS * 32;
#pragma unroll
          for (int j = 0; j < EPI_COLS; ++j)
            total[j] = __fadd_rn(total[j], __ldcg(slot + j * 32 + lane));
          __syncwarp();
          // consumed: the flag starts the next launch at zero
          if (lane == 0) st_release(flag, 0);
        }
        if (!ok) break;
      }
      // stores: 32-column slabs through this warp's staging tile.  Each lane
      // writes its row (+ 0 on the way: a product never leaves as -0, so a
      // `0 + c` gradient seed over it is the product's own buffer); then one
      // TMA store moves the slab, or, where the output's rows are not
      // 16-byte multiples, each store instruction writes one row's 32
      // consecutive floats.
      float* dst = out + (long long)t.split * split_stride + (long long)t.batch * m * n;
      float* st = epi_stage + ew * 32 * 32;
      const int row0 = t.m0 + q * 32;
      const int plane = t.split * (int)(split_stride / ((long long)m * n)) + t.batch;
#pragma unroll
      for (int g = 0; g < EPI_COLS / 32; ++g) {
#pragma unroll
        for (int cc = 0; cc < 8; ++cc)
          *(float4*)(st + stage_at(lane, cc * 4)) =
              make_float4(__fadd_rn(total[g * 32 + cc * 4], 0.0f),
                          __fadd_rn(total[g * 32 + cc * 4 + 1], 0.0f),
                          __fadd_rn(total[g * 32 + cc * 4 + 2], 0.0f),
                          __fadd_rn(total[g * 32 + cc * 4 + 3], 0.0f));
        const int col0 = t.n0 + c0 + g * 32;
        if (tma_store) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0 && row0 < m && col0 < n) {
            tma_store_3d(&tc, st, col0, row0, plane);
            // the slab is read before the next one overwrites it
            asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
          }
          __syncwarp();
          continue;
        }
        __syncwarp();
        const int col = col0 + lane;
        if (col < n) {
          float* p = dst + (long long)row0 * n + col;
          const int rows = min(32, m - row0);
#pragma unroll 8
          for (int r = 0; r < rows; ++r) p[(long long)r * n] = st[stage_at(r, lane)];
        }
        __syncwarp();
      }
    }
  }
  if (warp >= 2 && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 2) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(TMEM_COLS));
  }
}

__global__ void k_split_sum(const float* __restrict__ partial, float* __restrict__ out,
                            long long count, int splits) {
  pdl_entry();
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < count;
       i += (long long)gridDim.x * blockDim.x) {
    float acc = partial[i];
    for (int s = 1; s < splits; ++s) acc = __fadd_rn(acc, partial[(long long)s * count + i]);
    out[i] = __fadd_rn(acc, 0.0f);  // never -0, as the unsplit epilogue
  }
}

typedef CUresult (*EncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiled)p;
  });
  return fn;
}

// Tensor map over one prepared buffer [batch][rows][ld] floats; the box is
// box_x floats along a row by box_rows rows.
bool make_map(CUtensorMap* map, const float* base, int64_t ld, int64_t rows, int64_t batch,
              int box_x, int box_rows, CUtensorMapSwizzle swizzle) {
  EncodeTiled enc = encoder();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)ld, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 4), (cuuint64_t)(rows * ld * 4)};
  cuuint32_t box[3] = {(cuuint32_t)box_x, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)base, dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int g_tile_override = -1;  // TB_GEMM_TILE_N, or a test's forced choice
int g_tma_store = -1;      // TB_GEMM_TMA_STORE=0 keeps the warps' row-segment stores
bool tma_store_enabled() {
  if (g_tma_store < 0) {
    const char* e = getenv("TB_GEMM_TMA_STORE");
    g_tma_store = e ? atoi(e) : 1;
  }
  return g_tma_store != 0;
}
int g_narrow_tile = -1;    // TB_GEMM_NARROW_TILE=0 keeps outputs <= 64 wide on 128-wide tiles
// Stream-K is off unless TB_GEMM_STREAM_K=1 (or a test turns it on): measured on
// B200 it made the C4 step's 16384x512x512 products slower (57 against 46 us,
// two partial-tile epilogues per CTA where whole tiles overlap theirs with the
// next tile's main loop) and saved about 5% of cycles on 4096^3, which the
// power cap of a dense GEMM takes back in clock.
int g_stream_k = -1;
bool stream_k_enabled() {
  if (g_stream_k < 0) {
    const char* e = getenv("TB_GEMM_STREAM_K");
    g_stream_k = e ? atoi(e) : 0;
  }
  return g_stream_k != 0;
}

}  // namespace

bool encode_rows_f32(CUtensorMap* map, const float* base, int64_t width, int64_t rows,
                     int box_cols, int box_rows) {
  EncodeTiled enc = encoder();
  if (!enc || width % 4 != 0 || ((uintptr_t)base & 15)) return false;
  cuuint64_t dims[2] = {(cuuint64_t)width, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(width * 4)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace {


}  // namespace

static int splits_for(int bn, int64_t batch, int64_t m, int64_t n, int64_t kp) {
  const int bk = bn == 256 ? Cfg<256>::BK : Cfg<128>::BK;  // the 32- and 64-wide tiles share the 128-wide tile's BK
  const int64_t tiles = batch * ((m + BM - 1) / BM) * ((n + bn - 1) / bn);
  const int64_t kb = kp / bk;
  if (tiles >= 120 || kb < 16) return 1;
  // as many splits as fill one wave of SMs without starting a second one
  int64_t s = 148 / tiles;
  s = std::min<int64_t>(s, kb / 8);
  s = std::max<int64_t>(s, 1);
  // every split must own at least one k-block
  const int64_t per = (kb + s - 1) / s;
  return (int)((kb + per - 1) / per);
}

// Tile width for a shape (from a sweep of the configs' GEMMs on B200, split-K
// filling at most one wave, coalesced epilogue stores): the 256-wide tile moves
// 25% less operand data per flop and wins everywhere except narrow outputs,
// where half of its columns would be empty.
int gemm_tile_n(int64_t batch, int64_t m, int64_t n, int64_t kp) {
  (void)batch;
  (void)m;
  (void)kp;
  if (g_tile_override < 0) {
    const char* e = getenv("TB_GEMM_TILE_N");
    g_tile_override = e ? atoi(e) : 0;
  }
  if (g_tile_override == 32 || g_tile_override == 64 || g_tile_override == 128 ||
      g_tile_override == 256)
    return g_tile_override;
  if (g_narrow_tile < 0) {
    const char* e = getenv("TB_GEMM_NARROW_TILE");
    g_narrow_tile = e ? atoi(e) : 1;
  }
  if (n <= 32 && g_narrow_tile) return 32;
  if (n <= 64) return g_narrow_tile ? 64 : 128;
  return 256;
}

void set_gemm_tile_n(int tile) { g_tile_override = tile; }
void set_gemm_stream_k(int on) { g_stream_k = on ? 1 : 0; }

int gemm_splits(int64_t batch, int64_t m, int64_t n, int64_t kp) {
  return splits_for(gemm_tile_n(batch, m, n, kp), batch, m, n, kp);
}

namespace {
// Tensor map over an MN-major buffer [batch][rows][ld] seen as 32-float MN
// blocks: dimensions (32 floats, rows, ld / 32 blocks 128 bytes apart, batch),
// so one box of (32, bk, tile / 32) lands block after block -- the operand
// tile the MMA reads.  Every address stays inside its row of ld floats.  A
// raw A tile, which the epilogue warps read rather than the MMA, is unswizzled.
bool make_map_mn(CUtensorMap* map, const float* base, int64_t ld, int64_t rows, int64_t batch,
                 int tile, int bk,
                 CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B) {
  EncodeTiled enc = encoder();
  if (!enc) return false;
  cuuint64_t dims[4] = {32, (cuuint64_t)rows, (cuuint64_t)(ld / 32), (cuuint64_t)batch};
  cuuint64_t strides[3] = {(cuuint64_t)(ld * 4), 128, (cuuint64_t)(rows * ld * 4)};
  cuuint32_t box[4] = {32, (cuuint32_t)bk, (cuuint32_t)(tile / 32), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (void*)base, dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tensor maps of one operand's hi and lo buffers: K-major boxes are BK floats
// by the tile's rows (the config's swizzle), MN-major boxes the tile's MN
// blocks of 32 floats by BK rows (128-byte swizzle of 32-byte atoms).
// A raw operand (no lo buffer) has one map, over its f32 values; `lo` then
// repeats it and is never loaded.
template <class C>
bool operand_maps(CUtensorMap* hi, CUtensorMap* lo, const Operand& o, int tile, int64_t batch) {
  if (o.mn) {
    if (!o.lo) {
      if (!make_map_mn(hi, o.hi, o.ld, o.rows, batch, tile, C::BK, CU_TENSOR_MAP_SWIZZLE_NONE))
        return false;
      return (*lo = *hi, true);
    }
    if (!make_map_mn(hi, o.hi, o.ld, o.rows, batch, tile, C::BK)) return false;
    return make_map_mn(lo, o.lo, o.ld, o.rows, batch, tile, C::BK);
  }
  if (!make_map(hi, o.hi, o.ld, o.rows, batch, C::BK, tile, C::TMA_SWIZZLE)) return false;
  if (!o.lo) return (*lo = *hi, true);
  return make_map(lo, o.lo, o.ld, o.rows, batch, C::BK, tile, C::TMA_SWIZZLE);
}

template <class C, bool RAW>
bool configure(int dev) {
  using D = Derived<C>;
  static bool configured[256] = {};  // the attributes are set per device
  if (configured[dev]) return true;
  if (cudaFuncSetAttribute(k_gemm_tcgen05<C, false, RAW>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           D::SMEM_BYTES) != cudaSuccess ||
      cudaFuncSetAttribute(k_gemm_tcgen05<C, true, RAW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           D::SMEM_BYTES) != cudaSuccess)
    return false;
  configured[dev] = true;
  return true;
}

template <class C>
bool launch_cfg(const Operand& a, const Operand& b, float* c, float* partial, int splits,
                int64_t batch, int64_t m, int64_t n, int64_t kp, cudaStream_t stream,
                const StreamK* sk) {
  using D = Derived<C>;
  if (kp % C::BK != 0) return false;
  CUtensorMap ma, mal, mb, mbl;
  if (!operand_maps<C>(&ma, &mal, a, BM, batch) || !operand_maps<C>(&mb, &mbl, b, C::BN, batch))
    return false;
  // raw A is split into tensor memory; a raw B is not served here
  if (!b.lo) return false;
  const int raw = a.lo ? 0 : 1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 256) return false;
  if constexpr (C::GROUPS == 1) {
    if (!(raw ? configure<C, true>(dev) : configure<C, false>(dev))) return false;
  } else {
    if (raw || !configure<C, false>(dev)) return false;
  }
  const int kb = (int)(kp / C::BK);
  if (splits < 1 || !partial) splits = 1;
  const int per = (kb + splits - 1) / splits;
  float* target = splits > 1 ? partial : c;
  const int tiles_n = (int)((n + C::BN - 1) / C::BN), tiles_m = (int)((m + BM - 1) / BM);
  const long long items = (long long)tiles_n * tiles_m * batch * splits;
  if (items >= (1LL << 31)) return false;
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const int grid = (int)std::min<long long>(items, sms);
  Sched sched;
  sched.tiles_n = tiles_n;
  sched.tiles_m = tiles_m;
  sched.splits = splits;
  sched.split_blocks = per;
  sched.k_blocks = kb;
  sched.m_fast = m > 0 && n > m ? 1 : 0;
  sched.dp_items = (int)items;
  sched.sk_units = 0;
  // Stream-K for the tiles past the last whole wave but one, when the last
  // wave would leave SMs idle: whole tiles cost ceil(items / grid) tile
  // times per CTA, stream-K items / grid plus the hand-over of cut tiles.
  if (sk && sk->workspace && sk->flags && stream_k_enabled() && splits == 1 && batch == 1 &&
      items > grid && grid <= kStreamKMaxCtas) {
    const double waves = (double)items / grid;
    const long long whole = items / grid;
    if (std::ceil(waves) - waves > 0.15) {
      const long long dp_waves = whole;
      sched.dp_items = (int)(dp_waves * grid);
      sched.sk_units = (items - sched.dp_items) * (long long)kb;
    }
  }
  // the output as planes [batch * splits][m][n] for TMA stores of 32 x 32
  // slabs (rows must be 16-byte multiples; otherwise the warps store)
  CUtensorMap mc;
  memset(&mc, 0, sizeof mc);
  int tma_store = 0;
  if (n % 4 == 0 && ((uintptr_t)target & 15) == 0 && tma_store_enabled()) {
    EncodeTiled enc = encoder();
    cuuint64_t dims[3] = {(cuuint64_t)n, (cuuint64_t)m, (cuuint64_t)(batch * splits)};
    cuuint64_t strides[2] = {(cuuint64_t)(n * 4), (cuuint64_t)(m * n * 4)};
    cuuint32_t box[3] = {32, 32, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    tma_store = enc && enc(&mc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)target, dims, strides,
                           box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  }
  const long long plane = batch * m * n;
  float* ws = sched.sk_units > 0 ? sk->workspace : nullptr;
  int* flags = sched.sk_units > 0 ? sk->flags : nullptr;
  if constexpr (C::GROUPS == 1) {
    if (sched.sk_units > 0 && raw)
      launch_pdl(k_gemm_tcgen05<C, true, true>, grid, D::THREADS, D::SMEM_BYTES, stream, ma,
                 mal, mb, mbl, mc, tma_store, target, (int)m, (int)n, sched, plane, (int)a.mn,
                 (int)b.mn, ws, flags);
    else if (raw)
      launch_pdl(k_gemm_tcgen05<C, false, true>, grid, D::THREADS, D::SMEM_BYTES, stream,
                 ma, mal, mb, mbl, mc, tma_store, target, (int)m, (int)n, sched, plane,
                 (int)a.mn, (int)b.mn, ws, flags);
  }
  if (raw) {
    // launched above (the one-warpgroup tiles only)
  } else if (sched.sk_units > 0)
    launch_pdl(k_gemm_tcgen05<C, true, false>, grid, D::THREADS, D::SMEM_BYTES, stream, ma,
               mal, mb, mbl, mc, tma_store, target, (int)m, (int)n, sched, plane, (int)a.mn,
               (int)b.mn, ws, flags);
  else
    launch_pdl(k_gemm_tcgen05<C, false, false>, grid, D::THREADS, D::SMEM_BYTES, stream,
               ma, mal, mb, mbl, mc, tma_store, target, (int)m, (int)n, sched, plane, (int)a.mn,
               (int)b.mn, ws, flags);
  if (splits > 1) {
    const long long count = batch * m * n;
    int blocks = (int)std::min<long long>((count + 255) / 256, 148 * 8);
    launch_pdl(k_split_sum, blocks, 256, 0, stream, partial, c, count, splits);
  }
  return cudaPeekAtLastError() == cudaSuccess;
}
}  // namespace

bool launch_gemm_tcgen05_split(const Operand& a, const Operand& b, float* c, float* partial,
                               int splits, int64_t batch, int64_t m, int64_t n, int64_t kp,
                               cudaStream_t stream, const StreamK* sk) {
  if (m >= (1LL << 31) || n >= (1LL << 31) || batch > 65535) return false;
  if (((uintptr_t)a.hi | (uintptr_t)a.lo | (uintptr_t)b.hi | (uintptr_t)b.lo) & 15) return false;
  // row strides: 16-byte multiples for the tensor maps; an MN-major row holds
  // whole 32-float blocks
  for (const Operand* o : {&a, &b})
    if (o->ld % 4 != 0 || o->rows < 1 || (o->mn && o->ld % 32 != 0)) return false;
  int tile = gemm_tile_n(batch, m, n, kp);
  // the 256-wide tile's two epilogue warpgroups leave no registers for the
  // converters: raw operands take the 128-wide tile
  if (tile == 256 && !a.lo) tile = 128;
  if (tile == 256)
    return launch_cfg<Cfg<256>>(a, b, c, partial, splits, batch, m, n, kp, stream, sk);
  if (tile == 32)
    return launch_cfg<Cfg<32>>(a, b, c, partial, splits, batch, m, n, kp, stream, sk);
  if (tile == 64)
    return launch_cfg<Cfg<64>>(a, b, c, partial, splits, batch, m, n, kp, stream, sk);
  return launch_cfg<Cfg<128>>(a, b, c, partial, splits, batch, m, n, kp, stream, sk);
}

int gemm_error() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_gemm_error, sizeof(int));
  return v;
}

}  // namespace tb
