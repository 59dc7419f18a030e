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

// Device workspace of the host-buffer faces, one per device, grown on demand
// and kept for the process: a face call allocates only when a task is larger
// than every earlier one on that device.  The mutex serializes face calls on a
// device (the reference shares one cuBLAS handle behind a mutex the same way,
// backend/cuda/kernels/context.rs:203-212).
struct FaceDevice {
  std::mutex mutex;
  cudaStream_t stream = nullptr;
  void* buffer = nullptr;
  size_t bytes = 0;
};
FaceDevice g_face[64];

// Poisons the library for a CUDA failure inside a face: one runtime failure
// disables the backend for good (backend/cuda/kernels/mod.rs:94-105).
int face_failed(const char* face, cudaError_t e) {
  char text[256];
  snprintf(text, sizeof text, "%s: %s", face, cudaGetErrorString(e));
  tb::poison_library(text);
  return TB_RUNTIME;
}

// Claims the calling device's face workspace of at least `bytes` (lock held).
cudaError_t face_workspace(FaceDevice*& fd, std::unique_lock<std::mutex>& lock, size_t bytes,
                           void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  fd = &g_face[dev];
  lock = std::unique_lock<std::mutex>(fd->mutex);
  if (!fd->stream && (e = cudaStreamCreateWithFlags(&fd->stream, cudaStreamNonBlocking)))
    return e;
  if (fd->bytes < bytes) {
    if (fd->buffer) cudaFree(fd->buffer);
    fd->buffer = nullptr;
    fd->bytes = 0;
    if ((e = cudaMalloc(&fd->buffer, bytes)) != cudaSuccess) return e;
    fd->bytes = bytes;
  }
  *out = fd->buffer;
  return cudaSuccess;
}

// Checks the work a face enqueued: launch errors, the stream, and the tcgen05
// GEMM's wait-expiry flag.
cudaError_t face_finish(cudaStream_t st) {
  cudaError_t e = cudaStreamSynchronize(st);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e == cudaSuccess && tb::gemm_error() != 0) e = cudaErrorLaunchTimeout;
  return e;
}

size_t round256(size_t bytes) { return (bytes + 255) / 256 * 256; }

}  // namespace

extern "C" int tb_gemm_f32(const float* a, int64_t a_len, const int64_t a_strides[2],
                           const float* b, int64_t b_len, const int64_t b_strides[2], int64_t m,
                           int64_t k, int64_t n, float* out) {
  char msg[8];
  int s = tb_status(msg, sizeof msg);
  if (s != TB_OK) return s;
  if (m <= 1 || n <= 1 || k < 1 || 2 * m * n * k < kMinFlops) return TB_DECLINED;
  if (a_strides[0] < 0 || a_strides[1] < 0 || b_strides[0] < 0 || b_strides[1] < 0)
    return TB_DECLINED;
  if (span_of(m, k, a_strides) > a_len || span_of(k, n, b_strides) > b_len) return TB_INVALID;
  const int64_t kp = (k + 31) / 32 * 32;
  const int64_t al = span_of(m, k, a_strides), bl = span_of(k, n, b_strides);
  const size_t ab = round256(al * 4), bb = round256(bl * 4), cb = round256(m * n * 4);
  const size_t wb = (size_t)(2 * m * kp + 2 * n * kp) * 4;
  FaceDevice* fd = nullptr;
  std::unique_lock<std::mutex> lock;
  void* base = nullptr;
  cudaGetLastError();  // an earlier call's launch error is not this call's
  cudaError_t e = face_workspace(fd, lock, ab + bb + cb + wb, &base);
  if (e != cudaSuccess) return face_failed("tb_gemm_f32", e);
  cudaStream_t st = fd->stream;
  float* da = (float*)base;
  float* db = (float*)((char*)base + ab);
  float* dc = (float*)((char*)base + ab + bb);
  float* ahi = (float*)((char*)base + ab + bb + cb);
  float* alo = ahi + m * kp;
  float* bhi = alo + m * kp;
  float* blo = bhi + n * kp;
  if ((e = cudaMemcpyAsync(da, a, al * 4, cudaMemcpyHostToDevice, st)) ||
      (e = cudaMemcpyAsync(db, b, bl * 4, cudaMemcpyHostToDevice, st)))
    return face_failed("tb_gemm_f32", e);
  const int grid = 148 * 4;
  k_prep_strided<<<grid, 256, 0, st>>>(da, a_strides[0], a_strides[1], m, k, kp, ahi, alo);
  // B^T as [n, k]: row j of B^T walks column j of B
  k_prep_strided<<<grid, 256, 0, st>>>(db, b_strides[1], b_strides[0], n, k, kp, bhi, blo);
  tb::launch_gemm(tb::k_major(ahi, alo, m, kp), tb::k_major(bhi, blo, n, kp), dc, nullptr, 1, 1,
                  m, n, kp, st);
  if ((e = cudaGetLastError()) != cudaSuccess ||
      (e = cudaMemcpyAsync(out, dc, m * n * 4, cudaMemcpyDeviceToHost, st)) != cudaSuccess ||
      (e = face_finish(st)) != cudaSuccess)
    return face_failed("tb_gemm_f32", e);
  return TB_OK;
}

extern "C" int tb_map_f32(int32_t op, const float* in, int64_t count, float* out) {
  char msg[8];
  int s = tb_status(msg, sizeof msg);
  if (s != TB_OK) return s;
  if (op != TB_OP_EXP && op != TB_OP_LN && op != TB_OP_SQRT && op != TB_OP_TANH)
    return TB_DECLINED;
  if (count < (1 << 17)) return TB_DECLINED;
  FaceDevice* fd = nullptr;
  std::unique_lock<std::mutex> lock;
  void* base = nullptr;
  cudaGetLastError();
  cudaError_t e = face_workspace(fd, lock, (size_t)count * 8, &base);
  if (e != cudaSuccess) return face_failed("tb_map_f32", e);
  float* d = (float*)base;
  cudaStream_t st = fd->stream;
  if ((e = cudaMemcpyAsync(d, in, count * 4, cudaMemcpyHostToDevice, st)) != cudaSuccess)
    return face_failed("tb_map_f32", e);
  k_map<<<148 * 8, 256, 0, st>>>(op, d, d + count, count);
  if ((e = cudaGetLastError()) != cudaSuccess ||
      (e = cudaMemcpyAsync(out, d + count, count * 4, cudaMemcpyDeviceToHost, st)) ||
      (e = face_finish(st)) != cudaSuccess)
    return face_failed("tb_map_f32", e);
  return TB_OK;
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
  FaceDevice* fd = nullptr;
  std::unique_lock<std::mutex> lock;
  void* base = nullptr;
  cudaGetLastError();
  cudaError_t e = face_workspace(fd, lock, (size_t)(2 * n + 4 * features) * 4, &base);
  if (e != cudaSuccess) return face_failed("tb_batch_norm_f32", e);
  float* d = (float*)base;
  float *dx = d, *dout = d + n, *dscale = d + 2 * n, *dshift = dscale + features,
        *dmean = dshift + features, *dvar = dmean + features;
  cudaStream_t st = fd->stream;
  if ((e = cudaMemcpyAsync(dx, input, n * 4, cudaMemcpyHostToDevice, st)) ||
      (e = cudaMemcpyAsync(dscale, scale, features * 4, cudaMemcpyHostToDevice, st)) ||
      (e = cudaMemcpyAsync(dshift, shift, features * 4, cudaMemcpyHostToDevice, st)))
    return face_failed("tb_batch_norm_f32", e);
  k_batch_norm<<<(unsigned)((features + 127) / 128), 128, 0, st>>>(
      dx, dscale, dshift, epsilon, batch, features, dout, dmean, dvar);
  if ((e = cudaGetLastError()) ||
      (e = cudaMemcpyAsync(output, dout, n * 4, cudaMemcpyDeviceToHost, st)) ||
      (e = cudaMemcpyAsync(mean, dmean, features * 4, cudaMemcpyDeviceToHost, st)) ||
      (e = cudaMemcpyAsync(variance, dvar, features * 4, cudaMemcpyDeviceToHost, st)) ||
      (e = face_finish(st)))
    return face_failed("tb_batch_norm_f32", e);
  return TB_OK;
}

// ---- internal hooks for tests (not part of the public ABI)
extern "C" void tbx_set_gemm_engine(int engine) { tb::set_gemm_engine(engine); }
// Operand layouts: a_mn / b_mn select MN-major ([batch][k rows][ld], ld a
// multiple of 32); K-major operands are [batch][m or n][kp].  engine: 1 = the
// SIMT kernel, otherwise the tcgen05 path.
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
  // the tests' stream-K scratch, allocated once per process (test hook only)
  static tb::StreamK sk;
  if (!sk.workspace) {
    if (cudaMalloc((void**)&sk.workspace, tb::kStreamKWorkspaceBytes) != cudaSuccess ||
        cudaMalloc((void**)&sk.flags, tb::kStreamKFlagBytes) != cudaSuccess ||
        cudaMemset(sk.flags, 0, tb::kStreamKFlagBytes) != cudaSuccess)
      return TB_RUNTIME;
  }
  if (engine == 1)
    tb::launch_gemm_simt(a, b, c, batch, m, n, kp, st);
  else if (!tb::launch_gemm_tcgen05_split(a, b, c, partial, splits, batch, m, n, kp, st, &sk))
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
extern "C" void tbx_set_gemm_stream_k(int on) { tb::set_gemm_stream_k(on); }
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
// The array is a file-scope device variable of 16 MiB.  It is committed on a
// device when the library's device code loads there (with CUDA's lazy module
// loading, at the first call that needs it, e.g. this entry point's first
// call) and is held until the process exits.  All calls on a device share it,
// so calls that overlap on the GPU (different streams, or different host
// threads) race on it; callers serialize them.  Each call rewrites every
// scratch element it reads (padding included), so nothing needs clearing.
namespace {
constexpr int64_t kNoAllocScratchFloats = int64_t(4) << 20;  // 16 MiB of f32
__device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

// Host code cannot use the array's name as a device address: it is resolved
// on every call, with the calling device current, so a cached address can
// never outlive its context (a device reset, another context).
float* noalloc_scratch() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) return nullptr;
  return (float*)p;
}
}  // namespace

extern "C" int tb_gemm_f32_noalloc(const float* a, const int64_t a_strides[2], const float* b,
                                   const int64_t b_strides[2], int64_t m, int64_t k, int64_t n,
                                   float* out, void* stream) {
  // the request first: a malformed or oversized one is refused before any CUDA call
  if (!a || !b || !out || m < 1 || n < 1 || k < 1 || a_strides[0] < 0 || a_strides[1] < 0 ||
      b_strides[0] < 0 || b_strides[1] < 0) {
    tb::set_last_error("tb_gemm_f32_noalloc: invalid pointers, shape or strides");
    return TB_INVALID;
  }
  // each extent alone must fit before any product is formed, so that the size
  // arithmetic below cannot overflow
  if (m > kNoAllocScratchFloats || n > kNoAllocScratchFloats || k > kNoAllocScratchFloats ||
      2 * (m + n) * ((k + 31) / 32 * 32) > kNoAllocScratchFloats) {
    char text[240];
    snprintf(text, sizeof text,
             "tb_gemm_f32_noalloc: m=%lld k=%lld n=%lld needs 2*(m+n)*roundup(k,32) floats of "
             "scratch; the fixed scratch holds %lld (16 MiB)",
             (long long)m, (long long)k, (long long)n, (long long)kNoAllocScratchFloats);
    tb::set_last_error(text);
    return TB_INVALID;
  }
  // then readiness, without the library's lazy set-up (which initializes the context
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
  const int64_t kp = (k + 31) / 32 * 32;
  float* ws = noalloc_scratch();
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
  cudaGetLastError();  // a launch error left by earlier, unrelated work is not this call's
  k_prep_strided<<<grid, 256, 0, st>>>(a, a_strides[0], a_strides[1], m, k, kp, ahi, alo);
  k_prep_strided<<<grid, 256, 0, st>>>(b, b_strides[1], b_strides[0], n, k, kp, bhi, blo);
  tb::launch_gemm(tb::k_major(ahi, alo, m, kp), tb::k_major(bhi, blo, n, kp), out, nullptr, 1, 1,
                  m, n, kp, st);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return face_failed("tb_gemm_f32_noalloc", e);
  return TB_OK;
}
