"""QwenFeedForward.forward_host_stream: host batches in, host results out, with
the copies overlapping the kernels.  The results must be exactly the per-call
``ff(x)`` results (same kernels, same inputs), batch by batch."""

from __future__ import annotations

import pytest
import torch

from qwen_image_shardedit_mlx_b200 import QwenFeedForward, ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tokens,batches", [(300, 5), (3456, 3), (17, 1)])
def test_host_stream_matches_per_call(tokens, batches):
    g = torch.Generator(device="cuda").manual_seed(tokens)
    ff = QwenFeedForward.random(3072, 12288, generator=g)
    cg = torch.Generator().manual_seed(tokens)
    xs = [torch.randn((tokens, 3072), generator=cg).to(torch.bfloat16).pin_memory() for _ in range(batches)]
    ys = [torch.full((tokens, 3072), float("nan"), dtype=torch.bfloat16).pin_memory() for _ in range(batches)]
    ff.forward_host_stream(xs, ys)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    for x, y in zip(xs, ys):
        ref = ff(x.cuda()).cpu()
        assert torch.equal(y, ref)
