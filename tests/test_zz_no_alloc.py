"""q6_mlp_bf16_noalloc against q6_mlp_bf16, through the C ABI.

The no-allocation entry point serves callers that hold only input and output
device pointers and cannot call cudaMalloc (plugin hosts, FFI bindings,
serving loops that must not synchronise on allocation): it keeps the MLP's
hidden activations in a library-owned static device array instead of a
caller workspace.  These tests check that it computes what the workspace
entry point computes, on two calls in a row (the array keeps the previous
call's contents), and that it rejects problems larger than its array.

This file is named so that pytest collects it last.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from qwen_image_shardedit_mlx_b200 import _lib, ops
from tests.helpers import assert_close, f32, from_bits, random_bf16, random_weights, weights_to_torch

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 32 << 20


def _noalloc(x, w1, w2, y, m, d, h, gs=64, residual=None, gate=None):
    stream = torch.cuda.current_stream().cuda_stream
    return _lib.lib().q6_mlp_bf16_noalloc(
        x.data_ptr(), w1[0].data_ptr(), w1[1].data_ptr(), w1[2].data_ptr(), w1[3].data_ptr(),
        w2[0].data_ptr(), w2[1].data_ptr(), w2[2].data_ptr(), w2[3].data_ptr(),
        None if residual is None else residual.data_ptr(), None if gate is None else gate.data_ptr(),
        y.data_ptr(), m, d, h, gs, stream,
    )


@pytest.mark.parametrize("m,d,h", [(300, 512, 2048), (1024, 3072, 12288)])
def test_noalloc_matches_workspace_entry_point_twice(m, d, h):
    rng = np.random.default_rng(m + d + h)
    fc1 = weights_to_torch(random_weights(rng, h, d, 64))
    fc2 = weights_to_torch(random_weights(rng, d, h, 64))
    for call in range(2):
        x = from_bits(random_bf16(rng, (m, d)))
        ref = ops.q6_mlp(x, fc1, fc2, group_size=64)
        y = torch.full((m, d), float("nan"), dtype=torch.bfloat16, device="cuda")
        st = _noalloc(x, fc1, fc2, y, m, d, h)
        assert st == _lib.Q6_OK, _lib.status_string(st)
        torch.cuda.synchronize()
        assert bool(torch.isfinite(y).all()), f"call {call}: output not fully written"
        assert_close(f32(y), f32(ref), what=f"call {call}")
    assert ops.device_error() == 0


def test_noalloc_residual_gate_epilogue():
    rng = np.random.default_rng(5)
    m, d, h = 200, 256, 1024
    fc1 = weights_to_torch(random_weights(rng, h, d, 64))
    fc2 = weights_to_torch(random_weights(rng, d, h, 64))
    x = from_bits(random_bf16(rng, (m, d)))
    residual = from_bits(random_bf16(rng, (m, d)))
    gate = from_bits(random_bf16(rng, (d,), 0.5))
    ref = ops.q6_mlp(x, fc1, fc2, group_size=64, residual=residual, gate=gate)
    y = torch.empty((m, d), dtype=torch.bfloat16, device="cuda")
    assert _noalloc(x, fc1, fc2, y, m, d, h, residual=residual, gate=gate) == _lib.Q6_OK
    torch.cuda.synchronize()
    assert_close(f32(y), f32(ref))


def test_noalloc_at_the_array_limit():
    """The largest problem the array holds (M * H * 2 bytes = 32 MiB, 1365
    tokens at H = 12288), where no split-K space is left over."""

    h, d = 12288, 3072
    m = SCRATCH_BYTES // (2 * h)
    rng = np.random.default_rng(1365)
    fc1 = weights_to_torch(random_weights(rng, h, d, 64))
    fc2 = weights_to_torch(random_weights(rng, d, h, 64))
    x = from_bits(random_bf16(rng, (m, d)))
    ref = ops.q6_mlp(x, fc1, fc2, group_size=64)
    y = torch.full((m, d), float("nan"), dtype=torch.bfloat16, device="cuda")
    st = _noalloc(x, fc1, fc2, y, m, d, h)
    assert st == _lib.Q6_OK, _lib.status_string(st)
    torch.cuda.synchronize()
    assert bool(torch.isfinite(y).all())
    assert_close(f32(y), f32(ref), what="array limit")


def test_noalloc_small_m_uses_leftover_space_for_split_k():
    """64 tokens of the image-FF shapes: the array's space past the hidden
    activations holds the split-K partials of both linears (checked with the
    library's own size query), and the result matches the workspace entry
    point with the same split-K space."""

    h, d, m = 12288, 3072, 64
    lib = _lib.lib()
    split = max(lib.q6_linear_tc_workspace_bytes(m, h, d), lib.q6_linear_tc_workspace_bytes(m, d, h))
    assert split > 0
    assert (m * h * 2 + 255) // 256 * 256 + split <= SCRATCH_BYTES
    rng = np.random.default_rng(64)
    fc1 = weights_to_torch(random_weights(rng, h, d, 64))
    fc2 = weights_to_torch(random_weights(rng, d, h, 64))
    for call in range(2):
        x = from_bits(random_bf16(rng, (m, d)))
        ref = ops.q6_mlp(x, fc1, fc2, group_size=64)  # its own workspace carries split-K space too
        y = torch.full((m, d), float("nan"), dtype=torch.bfloat16, device="cuda")
        assert _noalloc(x, fc1, fc2, y, m, d, h) == _lib.Q6_OK
        torch.cuda.synchronize()
        assert bool(torch.isfinite(y).all())
        assert torch.equal(y, ref), f"call {call}: split-K in the array differs from split-K in a workspace"


def test_noalloc_rejects_problems_larger_than_its_array():
    h = 12288
    m_max = SCRATCH_BYTES // (2 * h)  # 1365 tokens
    dummy = torch.empty(16, dtype=torch.uint8, device="cuda")
    p = dummy.data_ptr()
    w = (dummy, dummy, dummy, dummy)
    st = _lib.lib().q6_mlp_bf16_noalloc(p, p, p, p, p, p, p, p, p, None, None, p, m_max + 1, 3072, h, 64, None)
    assert st == _lib.Q6_ERR_WORKSPACE
    del w
