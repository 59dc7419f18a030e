// optimizer_rule.h -- the per-element optimizer updates of the device step,
// in the operation order of neural/optimizer.rs:40-51 (SGD) and
// neural/adam.rs:40-104, 137-170 (Adam, AdamW).
//
// `BF16` is the element type of the parameters: a bf16 network rounds every
// operation's f32 result once to bf16 (payload/bf16.rs:131-170); in f32 the
// rounding is the identity and the sequence is the plain IEEE one.  The header
// compiles for the device (the optimizer kernel; TB_HD is `__device__`) and,
// with TB_HD defined empty and the CUDA intrinsics restated, for the host
// checks of the tests.
#pragma once
#include <cstdint>

#ifndef TB_HD
#define TB_HD __device__
#endif

namespace tb {

// payload/bf16.rs:39-55: the nearest bf16 (ties to even, carried into the
// exponent) as an f32; a NaN keeps its top half with a mantissa bit forced on.
TB_HD inline float bf16_nearest(float x) {
  const unsigned b = __float_as_uint(x);
  return __uint_as_float(isnan(x) ? ((b >> 16) | 0x40u) << 16
                                  : ((b + 0x7fffu + ((b >> 16) & 1u)) >> 16) << 16);
}

template <bool BF16>
TB_HD inline float element(float x) {
  return BF16 ? bf16_nearest(x) : x;
}

// Per-step scalars: `c1`, `c2` are 1 - beta1^t and 1 - beta2^t; `share1`,
// `share2` are 1 - beta1 and 1 - beta2 (adam.rs:46-47), each already an element
// of the parameters' type.
struct OptimizerScalars {
  int kind;  // 0 SGD, 1 Adam, 2 AdamW
  float lr, beta1, beta2, share1, share2, eps, decay, gscale, c1, c2;
};

// One parameter element: `p` and the moments `m`, `v` updated in place from
// gradient `g`; `decays` is AdamW's structural policy for this parameter.
template <bool BF16>
TB_HD inline void optimizer_update(float& p, float& m, float& v, float g, bool decays,
                                   const OptimizerScalars& s) {
  if (s.gscale != 1.0f) g = element<BF16>(__fmul_rn(g, s.gscale));
  const float p0 = p;
  if (s.kind == 0) {
    p = element<BF16>(__fsub_rn(p0, element<BF16>(__fmul_rn(g, s.lr))));
    return;
  }
  const float first = element<BF16>(__fadd_rn(element<BF16>(__fmul_rn(m, s.beta1)),
                                              element<BF16>(__fmul_rn(g, s.share1))));
  const float squared = element<BF16>(__fmul_rn(g, g));
  const float second = element<BF16>(__fadd_rn(element<BF16>(__fmul_rn(v, s.beta2)),
                                               element<BF16>(__fmul_rn(squared, s.share2))));
  m = first;
  v = second;
  const float cf = element<BF16>(__fdiv_rn(first, s.c1));
  const float cs = element<BF16>(__fdiv_rn(second, s.c2));
  const float root = element<BF16>(__fsqrt_rn(cs));
  const float d = element<BF16>(__fdiv_rn(cf, element<BF16>(__fadd_rn(root, s.eps))));
  const float stepped = element<BF16>(__fsub_rn(p0, element<BF16>(__fmul_rn(d, s.lr))));
  if (s.kind == 2 && decays) {
    const float decayed = element<BF16>(__fmul_rn(element<BF16>(__fmul_rn(p0, s.decay)), s.lr));
    p = element<BF16>(__fsub_rn(stepped, decayed));
  } else {
    p = stepped;
  }
}

// Advances the beta powers (adam.rs:72-75): s[0..1] = beta^t, s[2..3] = 1 - beta^t.
template <bool BF16>
TB_HD inline void advance_powers(float* s, float beta1, float beta2) {
  s[0] = element<BF16>(__fmul_rn(s[0], beta1));
  s[1] = element<BF16>(__fmul_rn(s[1], beta2));
  s[2] = element<BF16>(__fsub_rn(1.0f, s[0]));
  s[3] = element<BF16>(__fsub_rn(1.0f, s[1]));
}

}  // namespace tb
