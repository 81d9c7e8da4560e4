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


@pytest.mark.parametrize("tokens,chunks", [(3456, None), (1030, None), (2048, 4), (300, None)])
def test_host_tensor_call_matches_device_chunks(tokens, chunks):
    """ff(x) on a host tensor: chunked, copies overlapped, result on the host;
    each chunk's rows equal the device call on that chunk."""

    g = torch.Generator(device="cuda").manual_seed(tokens + 1)
    ff = QwenFeedForward.random(3072, 12288, generator=g)
    x = torch.randn((tokens, 3072), generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).pin_memory()
    y = ff(x) if chunks is None else ff.forward_host(x, chunks=chunks)
    assert y.device.type == "cpu" and y.shape == x.shape
    n = chunks or max(1, min(4, tokens // 512))
    while tokens % n:
        n -= 1
    step = tokens // n
    for i in range(n):
        ref = ff(x[i * step:(i + 1) * step].cuda()).cpu()
        assert torch.equal(y[i * step:(i + 1) * step], ref)
    assert ops.device_error() == 0


def test_host_stream_with_lora_matches_device_call():
    g = torch.Generator(device="cuda").manual_seed(8)
    ff = QwenFeedForward.random(512, 2048, generator=g)
    a = (torch.randn((512, 32), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    b = (torch.randn((32, 2048), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    ff.mlp_in.set_lora(a, b, 0.5)
    x = torch.randn((256, 512), generator=torch.Generator().manual_seed(4)).to(torch.bfloat16).pin_memory()
    y = torch.empty_like(x).pin_memory()
    ff.forward_host_stream([x], [y])
    torch.cuda.synchronize()
    assert torch.equal(y, ff(x.cuda()).cpu())
