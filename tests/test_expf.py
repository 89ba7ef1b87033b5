"""The float exp of the kernels against the reference's, on every float.

The reference computes its float exps with std::exp on a float - glibc's expf - in route_topk's softmax
(engine/src/model.cpp:4030), the Sampler's weights (engine/src/sampler.cpp:27), silu, sigmoid and softplus
(engine/src/kernels.hpp:141-168) and the Gated DeltaNet's decay (engine/src/model.cpp:3609). Router weights and sampled
acceptance are bit-exact only if the kernels' exp gives glibc's bits. glibc's expf is not correctly rounded, so a
double exp rounded to float is not a stand-in (the sweep below counts where the two differ); the kernels restate
glibc's algorithm (geode_b200/csrc/common.cuh, expf_ref), and so does the oracle (go_expf_restated). Here: the
restatement against this host's glibc on all 2^32 floats (the device's table against glibc: tests/test_expf_gpu.py).
"""
import os

import numpy as np

import oracle_py as op


def _threads():
    return max(1, min(32, os.cpu_count() or 1))


def test_restated_expf_equals_glibc_on_every_float():
    O = op.oracle_lib()
    first = np.zeros(16, np.uint32)
    bad = O.go_expf_mismatch(0, 1 << 32, 1, _threads(), first.ctypes.data, 16)
    assert bad == 0, [hex(int(b)) for b in first[: min(bad, 16)]]


def test_double_rounded_exp_is_no_stand_in():
    """Why the restatement: (float)exp((double)x) differs from glibc's expf on some floats (170 648 of 2^32 with
    this image's glibc). Swept over one binade of small arguments, where the differences cluster."""
    O = op.oracle_lib()
    first = np.zeros(4, np.uint32)
    lo, hi = 0x38800000, 0x39800000   # [2^-14, 2^-12)
    bad = O.go_expf_mismatch(lo, hi, 0, _threads(), first.ctypes.data, 4)
    assert bad > 0
    assert O.go_expf_mismatch(lo, hi, 1, _threads(), first.ctypes.data, 4) == 0
