"""Dense image MLP from q6 layers, with the reference's LoRA rules.

Mirrors shardedit_mlx/dense_img_ff_window.py: ``materialize_dense_linear``
dequantises a q6 layer once (here on the GPU dequant kernel) and folds
several adapters into the dense weight (:93-153); a single adapter stays
additive (:95-118); ``DenseFeedForward`` runs dense Linear math with the
optional additive adapters (:32-67); ``materialize_dense_img_ff`` builds one
from an ``img_ff``-shaped module and reports the dense bytes (:156-196).

This is the dense comparator of the q6 path (library GEMMs on dequantised
weights), kept for A/B checks and for callers that trade HBM for speed.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from qwen_image_shardedit_mlx_b200.lora import LoRAAdapter, iter_adapters, lora_delta_weight
from qwen_image_shardedit_mlx_b200.q6_metal_mlp import DenseLinearWeights, dequantize_linear, quantized_linear_spec


class DenseFeedForward:
    """img_ff replacement: dense Linear math matching QwenFeedForward."""

    def __init__(self, mlp_in: DenseLinearWeights, mlp_out: DenseLinearWeights, *,
                 mlp_in_lora: tuple[torch.Tensor, torch.Tensor, float] | None = None,
                 mlp_out_lora: tuple[torch.Tensor, torch.Tensor, float] | None = None) -> None:
        self.mlp_in = mlp_in
        self.mlp_out = mlp_out
        self.mlp_in_lora = mlp_in_lora
        self.mlp_out_lora = mlp_out_lora

    @staticmethod
    def _linear(hidden: torch.Tensor, weights: DenseLinearWeights,
                lora: tuple[torch.Tensor, torch.Tensor, float] | None) -> torch.Tensor:
        out = hidden @ weights.weight.T
        if weights.bias is not None:
            out = out + weights.bias
        if lora is not None:
            a, b, scale = lora
            out = out + scale * ((hidden @ a) @ b)
        return out

    def __call__(self, hidden: torch.Tensor) -> torch.Tensor:
        hidden = self._linear(hidden, self.mlp_in, self.mlp_in_lora)
        hidden = F.gelu(hidden, approximate="tanh")
        return self._linear(hidden, self.mlp_out, self.mlp_out_lora)


def _nbytes(t: torch.Tensor | None) -> int:
    return 0 if t is None else t.numel() * t.element_size()


def _dense_nbytes(w: DenseLinearWeights) -> int:
    return _nbytes(w.weight) + _nbytes(w.bias)


def materialize_dense_linear(layer: torch.nn.Module, *, dtype: torch.dtype = torch.bfloat16) -> DenseLinearWeights:
    """Dequantise a q6 layer; with two or more adapters fold sum s_i (A_i B_i)^T
    into the weight (the reference keeps a single adapter additive)."""

    dense = dequantize_linear(quantized_linear_spec(layer), dtype=dtype)
    adapters = list(iter_adapters(layer))
    if len(adapters) >= 2:
        delta = lora_delta_weight(adapters, dtype=torch.float32)
        if tuple(delta.shape) != tuple(dense.weight.shape):
            raise ValueError(f"LoRA delta shape {tuple(delta.shape)} != weight shape {tuple(dense.weight.shape)}")
        dense = DenseLinearWeights(weight=(dense.weight.to(torch.float32) + delta.to(dense.weight.device)).to(dtype),
                                   bias=dense.bias)
    return dense


def _additive(layer: torch.nn.Module, dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor, float] | None:
    adapters: list[LoRAAdapter] = list(iter_adapters(layer))
    if len(adapters) != 1:
        return None
    ad = adapters[0]
    return ad.lora_A.to(dtype), ad.lora_B.to(dtype), float(ad.scale)


def materialize_dense_img_ff(img_ff: torch.nn.Module, *,
                             dtype: torch.dtype = torch.bfloat16) -> tuple[DenseFeedForward, int]:
    """Dequantise one feed-forward's mlp_in / mlp_out into a DenseFeedForward;
    returns it with the dense weight bytes."""

    mlp_in = materialize_dense_linear(img_ff.mlp_in, dtype=dtype)
    mlp_out = materialize_dense_linear(img_ff.mlp_out, dtype=dtype)
    dense = DenseFeedForward(mlp_in, mlp_out, mlp_in_lora=_additive(img_ff.mlp_in, dtype),
                             mlp_out_lora=_additive(img_ff.mlp_out, dtype))
    return dense, _dense_nbytes(mlp_in) + _dense_nbytes(mlp_out)
