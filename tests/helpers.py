"""Shared helpers for the GPU parity tests (tolerances, torch <-> oracle conversion)."""

from __future__ import annotations

import numpy as np
import torch

import oracle

# Matmul outputs vs the oracle: max|err| <= 2e-2 * max|ref|
# and mean|err| <= 1e-3 * rms(ref).
MAX_ABS_REL = 2e-2
MEAN_ABS_REL = 1e-3


def to_bits(t: torch.Tensor) -> np.ndarray:
    """bf16 torch tensor -> uint16 bit patterns (numpy)."""

    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def from_bits(a: np.ndarray, device: str = "cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).view(torch.bfloat16).to(device)


def u32_to_torch(a: np.ndarray, device: str = "cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint32).view(np.int32)).to(device).view(torch.uint32)


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def weights_to_torch(w: oracle.Q6Weights, device: str = "cuda"):
    bias = None if w.bias is None else from_bits(w.bias, device)
    return u32_to_torch(w.weight, device), from_bits(w.scales, device), from_bits(w.biases, device), bias


def random_weights(rng: np.random.Generator, n: int, k: int, gs: int = 64, *, bias: bool = True,
                   std: float = 0.02) -> oracle.Q6Weights:
    w = rng.normal(0.0, std, size=(n, k)).astype(np.float32)
    packed, scales, biases = oracle.affine_quantize(w, group_size=gs)
    b = oracle.f32_to_bf16_bits(rng.normal(0.0, 0.01, size=(n,)).astype(np.float32)) if bias else None
    return oracle.Q6Weights(packed, scales, biases, b, gs)


def random_bf16(rng: np.random.Generator, shape, scale: float = 1.0) -> np.ndarray:
    return oracle.f32_to_bf16_bits((rng.standard_normal(shape) * scale).astype(np.float32))


def assert_close(got: np.ndarray, ref: np.ndarray, *, max_abs_rel: float = MAX_ABS_REL,
                 mean_abs_rel: float = MEAN_ABS_REL, what: str = "", bf16_output: bool = True) -> dict:
    """Tolerance check of a kernel output against the oracle.

    With ``bf16_output`` the oracle's fp32 result is first rounded to bf16, as
    the reference kernel rounds its own result (``T(acc)``,
    shardedit_mlx/q6_metal_mlp.py:82); comparing a bf16 output with an
    unrounded value would charge the output format's own rounding
    (~1.1e-3 * rms on average) to the kernel.
    """

    if bf16_output:
        ref = oracle.round_bf16(np.asarray(ref, dtype=np.float32))
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    err = np.abs(got - ref)
    scale = float(np.abs(ref).max()) or 1.0
    rms = float(np.sqrt(np.mean(ref * ref))) or 1.0
    stats = {"max_abs": float(err.max()), "max_abs_rel": float(err.max()) / scale,
             "mean_abs_rel_rms": float(err.mean()) / rms}
    assert stats["max_abs_rel"] <= max_abs_rel, f"{what}: {stats}"
    assert stats["mean_abs_rel_rms"] <= mean_abs_rel, f"{what}: {stats}"
    return stats
