"""GPU parity of the layers that checkpoint loading and LoRA patching produce.

* several adapters on one q6 layer (stacked into one fused delta) against the
  oracle's sum of adapters;
* a safetensors checkpoint written from oracle weights, loaded into device
  memory, run through the loaded ``img_ff`` against the oracle MLP;
* checkpoint LoRA keys patched onto loaded layers;
* the dense materialisation (reference dense_img_ff_window.py) against the q6
  path, with one additive adapter and with a folded pair.
"""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_close, f32, from_bits, random_bf16, random_weights, to_bits, weights_to_torch
from qwen_image_shardedit_mlx_b200 import ops
from qwen_image_shardedit_mlx_b200.dense_img_ff_window import DenseFeedForward, materialize_dense_img_ff
from qwen_image_shardedit_mlx_b200.lora import apply_lora_weights
from qwen_image_shardedit_mlx_b200.q6_metal_mlp import QuantizedLinear, QwenFeedForward
from qwen_image_shardedit_mlx_b200.qwen_block_loader import (
    block_layers,
    load_block_window,
    load_transformer_layout,
    save_safetensors,
)

pytestmark = pytest.mark.gpu


def _layer(w: oracle.Q6Weights) -> QuantizedLinear:
    wt, st, bt, bias = weights_to_torch(w)
    return QuantizedLinear(wt, st, bt, bias, group_size=w.group_size)


MULTI_CASES = [
    # (m, n, k, [(r, scale), ...])
    (300, 640, 1024, [(16, 0.5), (48, 1.75), (64, -0.4)]),   # total 128 (one 64-wide box per stage)
    (96, 512, 768, [(96, 0.8), (64, 0.8)]),                  # common scale: B unscaled, total 160
    (200, 384, 512, [(128, 1.0), (128, 0.25)]),              # the fused maximum, 256
    (5, 256, 256, [(8, 2.0), (4, 0.5)]),                     # ragged small ranks, padded to 32
]


@pytest.mark.parametrize("m,n,k,adapters", MULTI_CASES)
def test_multi_adapter_layer_vs_oracle(m, n, k, adapters):
    rng = np.random.default_rng(m + n + k + len(adapters))
    w = random_weights(rng, n, k, 64)
    lin = _layer(w)
    x = random_bf16(rng, (m, k))
    ref_loras = []
    for r, s in adapters:
        a_bits, b_bits = random_bf16(rng, (k, r), 0.02), random_bf16(rng, (r, n), 0.02)
        lin.add_lora(from_bits(a_bits), from_bits(b_bits), s)
        ref_loras.append((oracle.bf16_bits_to_f32(a_bits), oracle.bf16_bits_to_f32(b_bits), s))
    got = lin(from_bits(x))
    torch.cuda.synchronize()
    assert ops.last_path() == "tensor"
    ref = oracle.linear(oracle.bf16_bits_to_f32(x), w, weight_dtype="bf16", lora=ref_loras)
    assert_close(f32(got), ref, what=f"multi-lora {m}x{n}x{k} {adapters}")
    plain = oracle.linear(oracle.bf16_bits_to_f32(x), w, weight_dtype="bf16")
    assert float(np.abs(ref - plain).max()) > 5e-3 * float(np.abs(ref).max())


D, H = 512, 1024


def _write_checkpoint(root, rng, blocks: int = 2) -> dict[str, oracle.Q6Weights]:
    tdir = root / "transformer"
    tdir.mkdir()
    weights: dict[str, oracle.Q6Weights] = {}
    weight_map = {}
    for i in range(blocks):
        tensors = {}
        for name, (n, k) in {"img_ff.mlp_in": (H, D), "img_ff.mlp_out": (D, H), "attn.to_q": (D, D)}.items():
            w = random_weights(rng, n, k, 64)
            full = f"transformer_blocks.{i}.{name}"
            weights[full] = w
            wt, st, bt, bias = weights_to_torch(w, "cpu")
            tensors.update({f"{full}.weight": wt, f"{full}.scales": st, f"{full}.biases": bt, f"{full}.bias": bias})
        tensors[f"transformer_blocks.{i}.norm1.weight"] = torch.ones(D, dtype=torch.bfloat16)
        shard = f"model-{i + 1:05d}-of-{blocks:05d}.safetensors"
        save_safetensors(tdir / shard, tensors)
        weight_map.update({name: shard for name in tensors})
    (tdir / "model.safetensors.index.json").write_text(json.dumps({"weight_map": weight_map}))
    return weights


def test_loaded_blocks_run_the_q6_mlp(tmp_path):
    rng = np.random.default_rng(11)
    weights = _write_checkpoint(tmp_path, rng)
    layout = load_transformer_layout(tmp_path, block_count=2)
    blocks = load_block_window(layout, (0, 1), device="cuda")
    x = random_bf16(rng, (300, D))
    for blk in blocks:
        ff = blk.module.img_ff
        assert isinstance(ff, QwenFeedForward) and ff.mlp_in.weight.is_cuda
        got = ff(from_bits(x))
        torch.cuda.synchronize()
        pre = f"transformer_blocks.{blk.block_index}."
        ref = oracle.fused_mlp(oracle.bf16_bits_to_f32(x), weights[pre + "img_ff.mlp_in"],
                               weights[pre + "img_ff.mlp_out"])
        assert_close(f32(got), ref, what=f"loaded block {blk.block_index} img_ff")
        q = blk.module.linears["attn.to_q"](from_bits(x))
        torch.cuda.synchronize()
        assert_close(f32(q), oracle.linear(oracle.bf16_bits_to_f32(x), weights[pre + "attn.to_q"]),
                     what="loaded to_q")


def test_checkpoint_lora_patched_onto_loaded_layers(tmp_path):
    rng = np.random.default_rng(12)
    weights = _write_checkpoint(tmp_path, rng, blocks=1)
    blocks = load_block_window(load_transformer_layout(tmp_path, block_count=1), (0,), device="cuda")
    layers = block_layers(blocks)
    r, alpha = 16, 8.0
    down = random_bf16(rng, (r, D), 0.02)   # PEFT layout [r, in]
    up = random_bf16(rng, (H, r), 0.02)     # [out, r]
    key = "transformer.transformer_blocks.0.img_mlp.net.0.proj"
    lora_sd = {f"{key}.lora_A.weight": from_bits(down, "cpu"), f"{key}.lora_B.weight": from_bits(up, "cpu"),
               f"{key}.alpha": torch.tensor(alpha)}
    applied, matched = apply_lora_weights(layers, lora_sd, scale=0.6)
    assert applied == 1 and len(matched) == 3
    x = random_bf16(rng, (128, D))
    got = blocks[0].module.img_ff(from_bits(x))
    torch.cuda.synchronize()
    s = 0.6 * alpha / r
    lora = (oracle.bf16_bits_to_f32(down).T.copy(), oracle.bf16_bits_to_f32(up).T.copy(), s)
    h = oracle.round_bf16(oracle.linear(oracle.bf16_bits_to_f32(x), weights["transformer_blocks.0.img_ff.mlp_in"],
                                        apply_gelu=True, lora=lora))
    ref = oracle.linear(h, weights["transformer_blocks.0.img_ff.mlp_out"])
    assert_close(f32(got), ref, what="checkpoint lora img_ff")


@pytest.mark.parametrize("adapters", [[(8, 0.5)], [(8, 0.5), (16, 2.0)]])
def test_dense_materialisation_matches_q6(adapters):
    """reference tests/test_dense_img_ff_window.py:47-92: dense vs q6 within 0.05."""

    rng = np.random.default_rng(13 + len(adapters))
    mlp_in, mlp_out = _layer(random_weights(rng, H, D)), _layer(random_weights(rng, D, H))
    for r, s in adapters:
        mlp_in.add_lora(from_bits(random_bf16(rng, (D, r), 0.01)), from_bits(random_bf16(rng, (r, H), 0.01)), s)
    ff = QwenFeedForward(mlp_in, mlp_out)
    dense, nbytes = materialize_dense_img_ff(ff)
    assert isinstance(dense, DenseFeedForward) and nbytes == 2 * (H * D * 2) + (H + D) * 2
    assert (dense.mlp_in_lora is not None) == (len(adapters) == 1)  # two or more fold into the weight
    x = from_bits(random_bf16(rng, (4, 8, D)))
    y_q6, y_dense = ff(x), dense(x)
    torch.cuda.synchronize()
    err = float((y_q6.float() - y_dense.float()).abs().max())
    assert err < 0.05, err
    assert to_bits(y_q6).shape == (4, 8, D)
