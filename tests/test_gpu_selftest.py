"""The failure path of the library's bounded device waits, exercised without a fault.

Every pipeline wait in the GEMM and GEMV kernels is bounded: when a barrier
phase does not complete within its limit the waiting thread records a site
code in the device error word, raises the CTA's abort flag and returns, so a
lost arrival shows up as an error status instead of a hung GPU.  The library's
self-test kernel waits on an mbarrier that nothing ever arrives at through
that same bounded wait (1 ms limit here), with no copy in flight and no
tensor memory held; this test checks that the kernel returns, that
q6_get_device_error reports the self-test site, that q6_clear_device_error
resets the word, and that the context stays usable afterwards.
"""

from __future__ import annotations

import time

import numpy as np
import pytest
import torch

import oracle
from qwen_image_shardedit_mlx_b200 import _lib, ops
from tests.helpers import assert_close, f32, from_bits, random_bf16, random_weights, weights_to_torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_reports_its_site_and_clears():
    ops.clear_device_error()
    try:
        t0 = time.perf_counter()
        code = ops.selftest_bounded_wait(1_000_000)  # 1 ms limit; reading the word synchronises
        elapsed = time.perf_counter() - t0
        assert code == _lib.Q6_SITE_SELFTEST
        assert elapsed < 5.0  # the kernel returned on its own
        # the word keeps the first site until cleared
        assert ops.device_error() == _lib.Q6_SITE_SELFTEST
    finally:
        ops.clear_device_error()
    assert ops.device_error() == 0
    # the context is still usable: a q6 linear right after gives correct results
    rng = np.random.default_rng(12)
    w = random_weights(rng, 256, 512, 64)
    x = random_bf16(rng, (64, 512))
    got = ops.q6_linear(from_bits(x), *weights_to_torch(w), group_size=64)
    torch.cuda.synchronize()
    assert_close(f32(got), oracle.linear(oracle.bf16_bits_to_f32(x), w, weight_dtype="bf16"))
    assert ops.device_error() == 0


def test_longer_limit_takes_longer():
    """The limit is the one given: 50 ms of waiting shows up on the host clock."""

    ops.clear_device_error()
    try:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        code = ops.selftest_bounded_wait(50_000_000)
        elapsed = time.perf_counter() - t0
        assert code == _lib.Q6_SITE_SELFTEST
        assert 0.045 <= elapsed < 5.0
    finally:
        ops.clear_device_error()
