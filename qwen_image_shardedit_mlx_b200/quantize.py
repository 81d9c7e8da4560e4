"""MLX-layout affine 6-bit quantisation of dense weights (weight preparation).

Produces the tensor triplet the q6 path consumes: packed codes uint32
[N, K*6/32] (code k of a row in bits [6k, 6k+6) of its little-endian word
stream, the layout shardedit_mlx/q6_metal_mlp.py:28-40 reads), and bf16
scales / biases [N, K/group_size].  Per group: scale = max((max - min) / 63,
1e-7), bias = min, both rounded to bf16, q = clip(round((w - bias) / scale),
0, 63) - the published MLX affine scheme (`nn.QuantizedLinear.from_linear`,
used by the reference's tests, e.g. tests/test_q6_metal_mlp.py:17-32).

This is a load-time transform, not the hot path; it runs with torch ops on
whatever device the weight is on.
"""

from __future__ import annotations

import torch

GROUP_SIZES = (32, 64, 128)


def pack_codes(codes: torch.Tensor) -> torch.Tensor:
    """codes [..., K] (ints < 64, K % 16 == 0) -> uint32 [..., K*6/32]."""

    k = codes.shape[-1]
    if k % 16:
        raise ValueError(f"K={k} must be a multiple of 16")
    c = codes.to(torch.int64).reshape(*codes.shape[:-1], k // 16, 16) & 63
    w0 = c[..., 0] | c[..., 1] << 6 | c[..., 2] << 12 | c[..., 3] << 18 | c[..., 4] << 24 | (c[..., 5] & 3) << 30
    w1 = (c[..., 5] >> 2) | c[..., 6] << 4 | c[..., 7] << 10 | c[..., 8] << 16 | c[..., 9] << 22 | (c[..., 10] & 15) << 28
    w2 = (c[..., 10] >> 4) | c[..., 11] << 2 | c[..., 12] << 8 | c[..., 13] << 14 | c[..., 14] << 20 | c[..., 15] << 26
    words = torch.stack([w0, w1, w2], dim=-1).reshape(*codes.shape[:-1], k * 6 // 32)
    words = torch.where(words >= 2**31, words - 2**32, words).to(torch.int32)
    return words.view(torch.uint32)


def unpack_codes(packed: torch.Tensor, k: int) -> torch.Tensor:
    """uint32 [..., K*6/32] -> int64 codes [..., K]."""

    w = packed.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    t = w.reshape(*packed.shape[:-1], k // 16, 3)
    w0, w1, w2 = t[..., 0], t[..., 1], t[..., 2]
    cols = [
        w0, w0 >> 6, w0 >> 12, w0 >> 18, w0 >> 24, (w0 >> 30) | (w1 << 2),
        w1 >> 4, w1 >> 10, w1 >> 16, w1 >> 22, (w1 >> 28) | (w2 << 4),
        w2 >> 2, w2 >> 8, w2 >> 14, w2 >> 20, w2 >> 26,
    ]
    return (torch.stack(cols, dim=-1) & 63).reshape(*packed.shape[:-1], k)


@torch.no_grad()
def quantize_affine_q6(w: torch.Tensor, group_size: int = 64) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Dense weight [N, K] -> (packed uint32 [N, K*6/32], scales bf16, biases bf16)."""

    if group_size not in GROUP_SIZES:
        raise ValueError(f"group_size must be one of {GROUP_SIZES}")
    if w.dim() != 2:
        raise ValueError("weight must be 2-D [out_features, in_features]")
    n, k = w.shape
    if k % group_size:
        raise ValueError(f"in_features {k} is not a multiple of group_size {group_size}")
    g = w.to(torch.float32).reshape(n, k // group_size, group_size)
    w_max = g.amax(dim=-1)
    w_min = g.amin(dim=-1)
    scale = torch.clamp((w_max - w_min) / 63.0, min=1e-7)
    scale_bf = scale.to(torch.bfloat16)
    bias_bf = w_min.to(torch.bfloat16)
    s = scale_bf.to(torch.float32).unsqueeze(-1)
    b = bias_bf.to(torch.float32).unsqueeze(-1)
    q = torch.clamp(torch.round((g - b) / s), 0, 63).to(torch.int64).reshape(n, k)
    return pack_codes(q), scale_bf, bias_bf


def random_q6(n: int, k: int, *, group_size: int = 64, std: float = 0.02, generator: torch.Generator | None = None,
              device: torch.device | str = "cpu") -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Quantised N(0, std^2) weights: the synthetic stand-in for checkpoint tensors."""

    w = torch.randn((n, k), generator=generator, device=device, dtype=torch.float32) * std
    return quantize_affine_q6(w, group_size)
