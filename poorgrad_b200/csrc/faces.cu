// faces.cu -- the per-task offers of the backend seam (`Elementary::gemm` and
// `Elementary::map`, payload/elementary.rs:74-95) for callers that are not
// running a whole compiled plan.  Same contract as the reference cuda backend
// (backend/cuda/kernels/gemm.rs:54-163, mod.rs:69-89): host slices in, an owned
// row-major result out, "declined" for tasks below the size threshold.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/topos_b200.h"
#include "kernels.h"

namespace {

// Tasks with 2mnk below this many flops stay on the caller's path
// (the reference's cuda backend threshold, backend/cuda/kernels/mod.rs:34).
constexpr int64_t kMinFlops = int64_t(1) << 24;

__device__ __forceinline__ float tf32_rna(float x) {
  unsigned r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Strided [rows, depth] operand -> K-major hi/lo [rows, kp].
__global__ void k_prep_strided(const float* __restrict__ x, int64_t s_row, int64_t s_depth,
                               int64_t rows, int64_t depth, int64_t kp, float* __restrict__ hi,
                               float* __restrict__ lo) {
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < rows * kp;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = t / kp, k = t % kp;
    const float v = k < depth ? x[r * s_row + k * s_depth] : 0.0f;
    const float h = tf32_rna(v);
    hi[t] = h;
    lo[t] = __fsub_rn(v, h);
  }
}

__global__ void k_map(int op, const float* __restrict__ in, float* __restrict__ out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = in[i];
    float r = v;
    switch (op) {
      case TB_OP_EXP: r = expf(v); break;
      case TB_OP_LN: r = logf(v); break;
      case TB_OP_SQRT: r = __fsqrt_rn(v); break;
      case TB_OP_TANH: r = tanhf(v); break;
    }
    out[i] = r;
  }
}

// One thread per feature: the statistics fold down the batch in row order,
// seeded with the first row, exactly as the recorded formula's sum_along(0).
__global__ void k_batch_norm(const float* __restrict__ x, const float* __restrict__ scale,
                             const float* __restrict__ shift, float epsilon, int64_t batch,
                             int64_t features, float* __restrict__ out, float* __restrict__ mean,
                             float* __restrict__ variance) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= features) return;
  const float count = (float)batch;
  float s = x[j];
  for (int64_t b = 1; b < batch; ++b) s = __fadd_rn(s, x[b * features + j]);
  const float m = __fdiv_rn(s, count);
  float c = __fsub_rn(x[j], m);
  float q = __fmul_rn(c, c);
  for (int64_t b = 1; b < batch; ++b) {
    c = __fsub_rn(x[b * features + j], m);
    q = __fadd_rn(q, __fmul_rn(c, c));
  }
  const float v = __fdiv_rn(q, count);
  const float dev = __fsqrt_rn(__fadd_rn(v, epsilon));
  const float g = scale[j], h = shift[j];
  for (int64_t b = 0; b < batch; ++b) {
    const float n = __fdiv_rn(__fsub_rn(x[b * features + j], m), dev);
    out[b * features + j] = __fadd_rn(__fmul_rn(n, g), h);
  }
  mean[j] = m;
  variance[j] = v;
}

int64_t span_of(int64_t rows, int64_t cols, const int64_t s[2]) {
  return (rows - 1) * s[0] + (cols - 1) * s[1] + 1;
}

}  // namespace

extern "C" int tb_gemm_f32(const float* a, int64_t a_len, const int64_t a_strides[2],
                           const float* b, int64_t b_len, const int64_t b_strides[2], int64_t m,
                           int64_t k, int64_t n, float* out) {
  char msg[8];
  int s = tb_status(msg, sizeof msg);
  if (s != TB_OK) return s;
  if (m <= 1 || n <= 1 || 2 * m * n * k < kMinFlops) return TB_DECLINED;
  if (a_strides[0] < 0 || a_strides[1] < 0 || b_strides[0] < 0 || b_strides[1] < 0)
    return TB_DECLINED;
  if (span_of(m, k, a_strides) > a_len || span_of(k, n, b_strides) > b_len) return TB_INVALID;
  const int64_t kp = (k + 31) / 32 * 32;
  float *da = nullptr, *db = nullptr, *dc = nullptr, *ws = nullptr;
  const int64_t al = span_of(m, k, a_strides), bl = span_of(k, n, b_strides);
  cudaStream_t st = nullptr;
  int rc = TB_OK;
  do {
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) { rc = TB_RUNTIME; break; }
    if (cudaMalloc(&da, al * 4) || cudaMalloc(&db, bl * 4) || cudaMalloc(&dc, m * n * 4) ||
        cudaMalloc(&ws, (2 * m * kp + 2 * n * kp) * 4)) { rc = TB_RUNTIME; break; }
    cudaMemcpyAsync(da, a, al * 4, cudaMemcpyHostToDevice, st);
    cudaMemcpyAsync(db, b, bl * 4, cudaMemcpyHostToDevice, st);
    float* ahi = ws;
    float* alo = ahi + m * kp;
    float* bhi = alo + m * kp;
    float* blo = bhi + n * kp;
    int grid = 148 * 4;
    k_prep_strided<<<grid, 256, 0, st>>>(da, a_strides[0], a_strides[1], m, k, kp, ahi, alo);
    // B^T as [n, k]: row j of B^T walks column j of B
    k_prep_strided<<<grid, 256, 0, st>>>(db, b_strides[1], b_strides[0], n, k, kp, bhi, blo);
    tb::launch_gemm(tb::k_major(ahi, alo, m, kp), tb::k_major(bhi, blo, n, kp), dc, nullptr, 1,
                    1, m, n, kp, st);
    cudaMemcpyAsync(out, dc, m * n * 4, cudaMemcpyDeviceToHost, st);
    if (cudaStreamSynchronize(st) != cudaSuccess) rc = TB_RUNTIME;
  } while (false);
  if (da) cudaFree(da);
  if (db) cudaFree(db);
  if (dc) cudaFree(dc);
  if (ws) cudaFree(ws);
  if (st) cudaStreamDestroy(st);
  return rc;
}

extern "C" int tb_map_f32(int32_t op, const float* in, int64_t count, float* out) {
  char msg[8];
  int s = tb_status(msg, sizeof msg);
  if (s != TB_OK) return s;
  if (op != TB_OP_EXP && op != TB_OP_LN && op != TB_OP_SQRT && op != TB_OP_TANH)
    return TB_DECLINED;
  if (count < (1 << 17)) return TB_DECLINED;
  float *d = nullptr;
  if (cudaMalloc(&d, count * 8) != cudaSuccess) return TB_RUNTIME;
  cudaMemcpy(d, in, count * 4, cudaMemcpyHostToDevice);
  k_map<<<148 * 8, 256>>>(op, d, d + count, count);
  cudaMemcpy(out, d + count, count * 4, cudaMemcpyDeviceToHost);
  cudaError_t e = cudaGetLastError();
  cudaFree(d);
  return e == cudaSuccess ? TB_OK : TB_RUNTIME;
}

extern "C" int tb_batch_norm_f32(const float* input, const float* scale, const float* shift,
                                 float epsilon, int64_t batch, int64_t features, float* output,
                                 float* mean, float* variance) {
  char msg[8];
  int s = tb_status(msg, sizeof msg);
  if (s != TB_OK) return s;
  if (batch < 1 || features < 1) return TB_INVALID;
  if (batch * features < (1 << 17)) return TB_DECLINED;
  const int64_t n = batch * features;
  float* d = nullptr;
  if (cudaMalloc(&d, (2 * n + 4 * features) * 4) != cudaSuccess) return TB_RUNTIME;
  float *dx = d, *dout = d + n, *dscale = d + 2 * n, *dshift = dscale + features,
        *dmean = dshift + features, *dvar = dmean + features;
  cudaMemcpy(dx, input, n * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(dscale, scale, features * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(dshift, shift, features * 4, cudaMemcpyHostToDevice);
  k_batch_norm<<<(unsigned)((features + 127) / 128), 128>>>(dx, dscale, dshift, epsilon, batch,
                                                            features, dout, dmean, dvar);
  cudaMemcpy(output, dout, n * 4, cudaMemcpyDeviceToHost);
  cudaMemcpy(mean, dmean, features * 4, cudaMemcpyDeviceToHost);
  cudaMemcpy(variance, dvar, features * 4, cudaMemcpyDeviceToHost);
  cudaError_t e = cudaGetLastError();
  cudaFree(d);
  return e == cudaSuccess ? TB_OK : TB_RUNTIME;
}

// ---- internal hooks for tests (not part of the public ABI)
extern "C" void tbx_set_gemm_engine(int engine) { tb::set_gemm_engine(engine); }
// Operand layouts: a_mn / b_mn select MN-major ([batch][k rows][ld], ld a
// multiple of 32); K-major operands are [batch][m or n][kp].
extern "C" int tbx_gemm_prepared_layout(const float* a_hi, const float* a_lo, int a_mn,
                                        int64_t a_ld, const float* b_hi, const float* b_lo,
                                        int b_mn, int64_t b_ld, float* c, float* partial,
                                        int splits, int64_t batch, int64_t m, int64_t n,
                                        int64_t k, int64_t kp, int engine) {
  tb::Operand a = tb::k_major(a_hi, a_lo, m, kp), b = tb::k_major(b_hi, b_lo, n, kp);
  if (a_mn) {
    a.mn = 1;
    a.ld = a_ld;
    a.rows = k;
  }
  if (b_mn) {
    b.mn = 1;
    b.ld = b_ld;
    b.rows = k;
  }
  cudaStream_t st = 0;
  if (engine == 1)
    tb::launch_gemm_simt(a, b, c, batch, m, n, kp, st);
  else if (!tb::launch_gemm_tcgen05_split(a, b, c, partial, splits, batch, m, n, kp, st))
    return TB_DECLINED;
  return cudaDeviceSynchronize() == cudaSuccess ? TB_OK : TB_RUNTIME;
}
extern "C" int tbx_gemm_prepared(const float* a_hi, const float* a_lo, const float* b_hi,
                                 const float* b_lo, float* c, float* partial, int splits,
                                 int64_t batch, int64_t m, int64_t n, int64_t kp, int engine) {
  return tbx_gemm_prepared_layout(a_hi, a_lo, 0, kp, b_hi, b_lo, 0, kp, c, partial, splits, batch,
                                  m, n, kp, kp, engine);
}
extern "C" int tbx_gemm_error(void) { return tb::gemm_error(); }
extern "C" int tbx_segment_error(void) { return tb::segment_error(); }
extern "C" int tbx_tree_sum(const float* g, int shards, int64_t count, float* out) {
  if (shards < 1 || shards > 64) return TB_INVALID;
  tb::launch_tree_sum(g, shards, count, out, 0);
  return cudaDeviceSynchronize() == cudaSuccess ? TB_OK : TB_RUNTIME;
}
extern "C" void tbx_set_gemm_tile_n(int tile) { tb::set_gemm_tile_n(tile); }
extern "C" int tbx_gemm_splits(int64_t batch, int64_t m, int64_t n, int64_t kp) {
  return tb::gemm_splits(batch, m, n, kp);
}

// ---- allocation-free GEMM
//
// Some callers cannot let this library call cudaMalloc: a host framework that
// owns every device allocation through its own pool (and accounts for it), or
// code that must never allocate after start-up.  tb_gemm_f32_noalloc serves
// them: the caller passes device inputs and output, and the only scratch --
// the tf32 hi/lo split of both operands -- lives in the fixed array below.
// The array is a file-scope device variable: every GPU that loads the library
// holds its 16 MiB until the process exits.  All calls on a device share it,
// so calls that overlap on the GPU (different streams, or different host
// threads) race on it; callers serialize them.  Each call rewrites every
// scratch element it reads (padding included), so nothing needs clearing.
namespace {
constexpr int64_t kNoAllocScratchFloats = int64_t(4) << 20;  // 16 MiB of f32
__device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

std::mutex g_noalloc_mutex;
float* g_noalloc_ptr[256] = {};  // per device: the array's device address

// Host code cannot use the array's name as a device address: resolve it once
// per device, with that device current.
float* noalloc_scratch(int device) {
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (device < 0 || device >= 256) return nullptr;
  if (!g_noalloc_ptr[device]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) return nullptr;
    g_noalloc_ptr[device] = (float*)p;
  }
  return g_noalloc_ptr[device];
}
}  // namespace

extern "C" int tb_gemm_f32_noalloc(const float* a, const int64_t a_strides[2], const float* b,
                                   const int64_t b_strides[2], int64_t m, int64_t k, int64_t n,
                                   float* out, void* stream) {
  // readiness without the library's lazy set-up (which initializes the context
  // through a cudaFree(nullptr) call this entry point must not make)
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    tb::set_last_error("tb_gemm_f32_noalloc: no CUDA device");
    return TB_PLATFORM_UNSUPPORTED;
  }
  if (tb::poisoned()) {
    tb::set_last_error("tb_gemm_f32_noalloc: the backend is poisoned");
    return TB_POISONED;
  }
  if (m < 1 || n < 1 || k < 1 || a_strides[0] < 0 || a_strides[1] < 0 || b_strides[0] < 0 ||
      b_strides[1] < 0) {
    tb::set_last_error("tb_gemm_f32_noalloc: invalid shape or strides");
    return TB_INVALID;
  }
  const int64_t kp = (k + 31) / 32 * 32;
  const int64_t need = 2 * (m + n) * kp;
  if (need > kNoAllocScratchFloats) {
    char text[200];
    snprintf(text, sizeof text,
             "tb_gemm_f32_noalloc: needs %lld floats of scratch (2*(m+n)*roundup(k,32)); the "
             "fixed scratch holds %lld (16 MiB)",
             (long long)need, (long long)kNoAllocScratchFloats);
    tb::set_last_error(text);
    return TB_INVALID;
  }
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return TB_RUNTIME;
  float* ws = noalloc_scratch(device);
  if (!ws) {
    tb::set_last_error("tb_gemm_f32_noalloc: cudaGetSymbolAddress failed");
    return TB_RUNTIME;
  }
  cudaStream_t st = (cudaStream_t)stream;
  float* ahi = ws;
  float* alo = ahi + m * kp;
  float* bhi = alo + m * kp;
  float* blo = bhi + n * kp;
  const int grid = 148 * 4;
  k_prep_strided<<<grid, 256, 0, st>>>(a, a_strides[0], a_strides[1], m, k, kp, ahi, alo);
  k_prep_strided<<<grid, 256, 0, st>>>(b, b_strides[1], b_strides[0], n, k, kp, bhi, blo);
  tb::launch_gemm(tb::k_major(ahi, alo, m, kp), tb::k_major(bhi, blo, n, kp), out, nullptr, 1, 1,
                  m, n, kp, st);
  return cudaPeekAtLastError() == cudaSuccess ? TB_OK : TB_RUNTIME;
}
