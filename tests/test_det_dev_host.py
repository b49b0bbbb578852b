"""Host-compiled device det arithmetic against the oracle (CPU).

The kernels' arithmetic header (det_dev.cuh) is compiled for the host with
g++ beside the oracle's restatement of det_num ops.rs, and each function is
compared on edge values plus millions of seeded random inputs.  This pins the
device formulations (floor-shift requantize, double-estimate inv_sqrt and
softmax division, 64-bit rounding divisions) without a GPU; the GPU parity
tests then confirm that nvcc compiles the same header to the same results.
"""
import ctypes
import os
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "det_dev_host.cpp")
OUT = os.path.join(HERE, "_build", "libdet_dev_host.so")
DEPS = [SRC, os.path.join(HERE, "..", "raster-inference_b200", "csrc", "det_dev.cuh"),
        os.path.join(HERE, "..", "oracle", "det_num.hpp")]


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(OUT) or any(os.path.getmtime(d) > os.path.getmtime(OUT) for d in DEPS):
        os.makedirs(os.path.dirname(OUT), exist_ok=True)
        subprocess.run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-o", OUT, SRC], check=True)
    L = ctypes.CDLL(OUT)
    L.rdet_host_check.restype = ctypes.c_int64
    L.rdet_host_check.argtypes = [ctypes.c_char_p, ctypes.c_uint64, ctypes.c_int64]
    return L


CASES = [
    ("inv_sqrt_acc", 2_000_000),
    ("rms_norm_scale", 200_000),
    ("requantize", 2_000_000),
    ("requantize_edges", 1),
    ("rshift_rte", 2_000_000),
    ("div_act", 1_000_000),
    ("div_acc_by_u32", 1_000_000),
    ("div_edges", 1_000_000),
    ("acc_mul", 1_000_000),
    ("exp_term", 1_000_000),
    ("exp_term_all", 1_000_000),
    ("softmax_weight", 1_000_000),
    ("tanh_act", 1_000_000),
    ("softcap_act", 500_000),
    ("gelu_act", 1_000_000),
    ("sin_cos_acc", 500_000),
    ("pos_angle", 1_000_000),
]


@pytest.mark.parametrize("fn,n", CASES, ids=[c[0] for c in CASES])
def test_device_arith_matches_oracle(lib, fn, n):
    for seed in (1, 0xDE7):
        bad = lib.rdet_host_check(fn.encode(), seed, n)
        assert bad == 0, f"{fn}: {bad} mismatches (seed {seed})"


def test_unknown_function_rejected(lib):
    assert lib.rdet_host_check(b"no_such_fn", 1, 10) == -1
