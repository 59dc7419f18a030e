"""The device optimizer's per-element rule (`csrc/optimizer_rule.h`, the body
of the optimizer kernel) compiled for the host against the kernel emulator's
intrinsics and stepped for several generations: bitwise equal to the host
restatement of the reference's SGD, Adam and AdamW (`oracle/optim.py`), in f32
and in bf16.  The scalars are prepared as the runtime prepares them (bf16
hyperparameters, shares `1 - beta` rounded once)."""
import ctypes as C
import hashlib
import os
import subprocess
import tempfile

import numpy as np
import pytest

import oracle
from oracle import optim

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "poorgrad_b200", "csrc")

HARNESS = r'''
#include "kernel_emulator.h"
#define TB_HD
#include "optimizer_rule.h"
extern "C" void rule_step(int kind, int bf16, long n, float* p, float* m, float* v,
                          const float* g, int decays, float* s, float lr, float beta1,
                          float beta2, float share1, float share2, float eps, float decay) {
  if (kind) {
    if (bf16) tb::advance_powers<true>(s, beta1, beta2);
    else tb::advance_powers<false>(s, beta1, beta2);
  }
  tb::OptimizerScalars sc{kind, lr, beta1, beta2, share1, share2, eps, decay, 1.0f,
                          kind ? s[2] : 0.0f, kind ? s[3] : 0.0f};
  for (long i = 0; i < n; ++i) {
    if (bf16) tb::optimizer_update<true>(p[i], m[i], v[i], g[i], decays != 0, sc);
    else tb::optimizer_update<false>(p[i], m[i], v[i], g[i], decays != 0, sc);
  }
}
'''


@pytest.fixture(scope="module")
def rule():
    with open(os.path.join(CSRC, "optimizer_rule.h")) as f:
        key = hashlib.sha1((HARNESS + f.read()).encode()).hexdigest()[:16]
    work = os.path.join(tempfile.gettempdir(), "tb_kernel_emulator")
    os.makedirs(work, exist_ok=True)
    lib = os.path.join(work, "rule_" + key + ".so")
    if not os.path.exists(lib):
        src = os.path.join(work, "rule_" + key + ".cpp")
        with open(src, "w") as f:
            f.write(HARNESS)
        subprocess.check_call(["g++", "-std=c++20", "-O1", "-ffp-contract=off", "-fno-fast-math",
                               "-fPIC", "-shared", "-pthread", "-w", "-I", HERE, "-I", CSRC,
                               "-o", lib + ".tmp", src])
        os.replace(lib + ".tmp", lib)
    return C.CDLL(lib)


def fptr(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


@pytest.mark.parametrize("element", [np.float32, optim.BF16])
@pytest.mark.parametrize("kind", ["sgd", "adam", "adamw"])
def test_the_device_rule_is_the_reference_rule_bitwise(built, rule, element, kind):
    bf16 = element == optim.BF16
    r = (lambda x: float(oracle.round_bf16(np.array([x], np.float32))[0])) if bf16 else \
        (lambda x: float(np.float32(x)))
    hyper = dict(beta1=0.9, beta2=0.95, eps=1e-8, decay=0.1)
    lr = 3e-3
    host = optim.make(kind, hyper, element)
    rng = np.random.default_rng(7)
    shapes = [(6, 9), (9,)]  # a weight AdamW decays and a bias it spares
    params = [rng.standard_normal(s).astype(np.float32) for s in shapes]
    if bf16:
        params = [oracle.round_bf16(p.reshape(-1)).reshape(p.shape) for p in params]
    dev = [p.copy().reshape(-1) for p in params]
    moments = [(np.zeros(p.size, np.float32), np.zeros(p.size, np.float32)) for p in params]
    code = {"sgd": 0, "adam": 1, "adamw": 2}[kind]
    b1, b2 = r(hyper["beta1"]), r(hyper["beta2"])
    scalars = (C.c_float * 4)(1.0, 1.0, 0.0, 0.0)
    for _ in range(5):
        grads = [rng.standard_normal(s).astype(np.float32) for s in shapes]
        if bf16:
            grads = [oracle.round_bf16(g.reshape(-1)).reshape(g.shape) for g in grads]
        params = host.step(params, grads, lr)
        powers = list(scalars)
        for i, (p, g) in enumerate(zip(dev, grads)):
            if i:  # the powers advance once per step, not once per parameter
                scalars[:] = powers
            m, v = moments[i]
            gg = np.ascontiguousarray(g.reshape(-1), np.float32)
            rule.rule_step(code, int(bf16), C.c_long(p.size), fptr(p), fptr(m), fptr(v),
                           fptr(gg), int(g.ndim >= 2), scalars, C.c_float(r(lr)),
                           C.c_float(b1), C.c_float(b2), C.c_float(r(1.0 - b1)),
                           C.c_float(r(1.0 - b2)), C.c_float(r(hyper["eps"])),
                           C.c_float(r(hyper["decay"])))
        for a, b in zip(dev, params):
            assert a.tobytes() == b.reshape(-1).tobytes()
