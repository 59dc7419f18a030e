// kernel_emulator.h -- TEST INFRASTRUCTURE: the CUDA built-ins that the
// lowering's generated kernels use, restated for the host so that a lowered
// program can run on the CPU in the tests (tests/kernel_emulator.py).  The
// product never uses this; it checks what the emitter writes, not how fast.
//
// Execution model: one OS thread per CUDA thread of a block; the blocks of a
// launch run one after another, so `__shared__` storage is static and shared
// by the block's threads; `__syncthreads` is a barrier of the block's
// threads; `__shfl_xor_sync` exchanges through per-warp slots between two
// barriers of the warp's 32 threads.  Arithmetic intrinsics are the IEEE
// operations they name (the source is compiled without contraction).
#pragma once
#include <barrier>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <functional>
#include <memory>
#include <thread>
#include <vector>

#define __global__
#define __device__
#define __forceinline__ inline
#define __shared__ static
#define __launch_bounds__(...)

struct emu_dim3 {
  unsigned x = 0, y = 0, z = 0;
};
inline thread_local emu_dim3 threadIdx, blockIdx;
inline emu_dim3 blockDim, gridDim;

struct float4 {
  float x, y, z, w;
};
inline float4 make_float4(float x, float y, float z, float w) { return float4{x, y, z, w}; }

inline float __fadd_rn(float a, float b) { return a + b; }
inline float __fsub_rn(float a, float b) { return a - b; }
inline float __fmul_rn(float a, float b) { return a * b; }
inline float __fdiv_rn(float a, float b) { return a / b; }
inline float __fsqrt_rn(float a) { return std::sqrt(a); }
inline float __fmaf_rn(float a, float b, float c) { return std::fma(a, b, c); }
using std::isfinite;
inline float __int_as_float(int v) {
  float f;
  std::memcpy(&f, &v, 4);
  return f;
}
inline float __uint_as_float(unsigned v) {
  float f;
  std::memcpy(&f, &v, 4);
  return f;
}
inline unsigned __float_as_uint(float f) {
  unsigned v;
  std::memcpy(&v, &f, 4);
  return v;
}
using std::isnan;

// tf32 rounding to nearest, ties away from zero (the `cvt.rna.tf32.f32`
// the prelude asks for): keep 10 mantissa bits.
inline unsigned emu_tf32_bits(float x) {
  unsigned b = __float_as_uint(x);
  if ((b & 0x7f800000u) == 0x7f800000u) return b;  // inf / nan unchanged
  return (b + 0x1000u) & 0xffffe000u;
}

namespace emu {
struct Block {
  unsigned threads = 0;
  std::unique_ptr<std::barrier<>> all;
  std::vector<std::unique_ptr<std::barrier<>>> warps;
  std::vector<float> slots;
};
inline Block* current = nullptr;
}  // namespace emu

inline void __syncthreads() { emu::current->all->arrive_and_wait(); }

inline float __shfl_xor_sync(unsigned, float v, int lane_mask) {
  emu::Block& b = *emu::current;
  const unsigned t = threadIdx.x, warp = t / 32, lane = t % 32;
  b.slots[t] = v;
  b.warps[warp]->arrive_and_wait();
  const float r = b.slots[warp * 32 + (lane ^ (unsigned)lane_mask)];
  b.warps[warp]->arrive_and_wait();
  return r;
}

// Runs `body` as a launch of `grid` blocks of `block` threads.
inline void emu_launch(long grid, unsigned block, const std::function<void()>& body) {
  emu::Block b;
  b.threads = block;
  b.all = std::make_unique<std::barrier<>>(block);
  for (unsigned w = 0; w < (block + 31) / 32; ++w)
    b.warps.push_back(std::make_unique<std::barrier<>>(std::min(32u, block - 32 * w)));
  b.slots.assign(block, 0.0f);
  emu::current = &b;
  blockDim.x = block;
  blockDim.y = blockDim.z = 1;
  gridDim.x = (unsigned)grid;
  gridDim.y = gridDim.z = 1;
  std::vector<std::thread> threads;
  for (unsigned t = 0; t < block; ++t)
    threads.emplace_back([&, t]() {
      threadIdx.x = t;
      for (long g = 0; g < grid; ++g) {
        blockIdx.x = (unsigned)g;
        body();
        b.all->arrive_and_wait();  // the next block's threads start together
      }
    });
  for (auto& th : threads) th.join();
  emu::current = nullptr;
}
