"""LoRA host logic on the CPU: the multi-adapter fold, rank padding, the dense
fold, checkpoint key plans and patching.

The key-plan cases restate the reference's own tests (tests/test_lora_plan.py:10-95).
"""

from __future__ import annotations

from dataclasses import FrozenInstanceError

import pytest
import torch

from qwen_image_shardedit_mlx_b200.lora import (
    MAX_FUSED_RANK,
    LoRAAdapter,
    apply_lora_weights,
    fold_lora_adapters,
    lora_delta_weight,
    pad_lora_rank,
    plan_qwen_lora_keys,
    select_lora_keys,
)
from qwen_image_shardedit_mlx_b200.q6_metal_mlp import QuantizedLinear
from qwen_image_shardedit_mlx_b200.quantize import quantize_affine_q6


def _adapter(k: int, n: int, r: int, scale: float, seed: int) -> LoRAAdapter:
    g = torch.Generator().manual_seed(seed)
    return LoRAAdapter((torch.randn(k, r, generator=g) * 0.05).to(torch.bfloat16),
                       (torch.randn(r, n, generator=g) * 0.05).to(torch.bfloat16), scale)


def _kernel_delta(x: torch.Tensor, fused) -> torch.Tensor:
    """What the fused kernel adds: (x @ A) @ bf16(scale * B), fp64 sums."""

    a, b, s = fused
    b_eff = (b.to(torch.float32) * torch.tensor(s, dtype=torch.float32)).to(torch.bfloat16)
    return (x.double() @ a.double()) @ b_eff.double()


def test_single_adapter_is_passed_through():
    ad = _adapter(64, 32, 16, 0.5, 0)
    a, b, s = fold_lora_adapters([ad])
    assert torch.equal(a, ad.lora_A) and torch.equal(b, ad.lora_B) and s == 0.5
    assert fold_lora_adapters([]) is None


def test_fold_with_distinct_scales_reproduces_each_adapter():
    ads = [_adapter(96, 80, 16, 0.5, 1), _adapter(96, 80, 48, 1.75, 2), _adapter(96, 80, 8, -0.3, 3)]
    a, b, s = fold_lora_adapters(ads)
    assert s == 1.0 and a.shape == (96, 72) and b.shape == (72, 80)
    row = 0
    for ad in ads:
        # rows of B' are exactly bf16(s_i * B_i): the kernel's own single-adapter operand
        want = (ad.lora_B.float() * torch.tensor(ad.scale)).to(torch.bfloat16)
        assert torch.equal(b[row:row + ad.rank], want)
        assert torch.equal(a[:, row:row + ad.rank], ad.lora_A)
        row += ad.rank
    x = torch.randn(5, 96, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
    want = sum(_kernel_delta(x, (ad.lora_A, ad.lora_B, ad.scale)) for ad in ads)
    assert torch.allclose(_kernel_delta(x, (a, b, s)), want, rtol=0, atol=1e-12)


def test_fold_with_one_common_scale_keeps_b_unscaled():
    ads = [_adapter(64, 64, 32, 0.8, 4), _adapter(64, 64, 32, 0.8, 5)]
    a, b, s = fold_lora_adapters(ads)
    assert s == 0.8 and torch.equal(b, torch.cat([ads[0].lora_B, ads[1].lora_B]))


def test_fold_rejects_mismatched_or_oversized_adapters():
    with pytest.raises(ValueError, match="LoRA A must be"):
        fold_lora_adapters([_adapter(64, 64, 8, 1.0, 0), _adapter(32, 64, 8, 1.0, 1)])
    with pytest.raises(ValueError, match="LoRA A must be"):
        fold_lora_adapters([_adapter(64, 64, 8, 1.0, 0)], out_features=32)
    with pytest.raises(ValueError, match="exceeds"):
        fold_lora_adapters([_adapter(64, 64, 128, 1.0, 0), _adapter(64, 64, MAX_FUSED_RANK - 127, 1.0, 1)])


@pytest.mark.parametrize("r", [1, 8, 31, 32, 33, 200])
def test_pad_lora_rank_is_exact(r):
    ad = _adapter(40, 24, r, 1.0, r)
    a, b = pad_lora_rank(ad.lora_A, ad.lora_B)
    assert a.shape[1] % 32 == 0 and a.shape[1] - r < 32 and b.shape[0] == a.shape[1]
    assert torch.equal(a[:, :r], ad.lora_A) and not a[:, r:].any() and not b[r:].any()
    x = torch.randn(3, 40, dtype=torch.float64)
    # the padded products are exact zeros (only the BLAS summation order may differ)
    assert torch.allclose((x @ a.double()) @ b.double(), (x @ ad.lora_A.double()) @ ad.lora_B.double(),
                          rtol=0, atol=1e-13)


def test_dense_fold_matches_the_sum_of_products():
    ads = [_adapter(48, 40, 8, 0.5, 6), _adapter(48, 40, 4, 2.0, 7)]
    d = lora_delta_weight(ads, dtype=torch.float32)
    want = sum(ad.scale * (ad.lora_A.double() @ ad.lora_B.double()) for ad in ads).T
    assert d.shape == (40, 48) and torch.allclose(d.double(), want, atol=1e-6)
    assert lora_delta_weight([]) is None


def _layer(n: int, k: int, seed: int) -> QuantizedLinear:
    w, s, b = quantize_affine_q6(torch.randn(n, k, generator=torch.Generator().manual_seed(seed)) * 0.02, 64)
    return QuantizedLinear(w, s, b, None)


def test_quantized_linear_keeps_adapters_and_their_fold():
    lin = _layer(64, 128, 0)
    a1, a2 = _adapter(128, 64, 16, 0.5, 1), _adapter(128, 64, 32, 2.0, 2)
    lin.set_lora(a1.lora_A, a1.lora_B, 0.5)
    assert len(lin.loras) == 1 and lin.lora[2] == 0.5
    lin.add_lora(a2.lora_A, a2.lora_B, 2.0)
    assert len(lin.loras) == 2 and lin.lora[0].shape == (128, 48) and lin.lora[2] == 1.0
    with pytest.raises(ValueError):
        lin.add_lora(torch.zeros(64, 8), torch.zeros(8, 64))
    assert len(lin.loras) == 2  # a rejected adapter leaves the layer as it was
    lin.set_lora(None)
    assert lin.lora is None and lin.loras == []


# --- key plans (reference tests/test_lora_plan.py) -------------------------------------------

def test_qwen_lora_plan_groups_supported_namespaces_by_block():
    plan = plan_qwen_lora_keys(
        (
            "transformer_blocks.0.attn.to_q.lora_up.weight",
            "transformer.transformer_blocks.1.attn.to_q.lora.down.weight",
            "diffusion_model.transformer_blocks.1.attn.to_q.lora_B.weight",
            "lora_unet_transformer_blocks_2_attn_to_q.alpha",
        ),
        block_count=3,
    )
    assert plan.key_count == 4
    assert plan.keys_by_block[0] == ("transformer_blocks.0.attn.to_q.lora_up.weight",)
    assert len(plan.keys_by_block[1]) == 2
    assert plan.keys_by_block[2] == ("lora_unet_transformer_blocks_2_attn_to_q.alpha",)


def test_select_lora_keys_preserves_block_then_key_order():
    plan = plan_qwen_lora_keys(
        (
            "transformer_blocks.1.attn.to_v.lora_up.weight",
            "transformer_blocks.0.attn.to_q.lora_up.weight",
            "transformer_blocks.1.attn.to_q.lora_up.weight",
        ),
        block_count=2,
    )
    assert select_lora_keys(plan, (0, 1)) == (
        "transformer_blocks.0.attn.to_q.lora_up.weight",
        "transformer_blocks.1.attn.to_q.lora_up.weight",
        "transformer_blocks.1.attn.to_v.lora_up.weight",
    )


def test_qwen_lora_plan_is_immutable():
    plan = plan_qwen_lora_keys(("transformer_blocks.0.attn.to_q.alpha",), block_count=1)
    with pytest.raises(FrozenInstanceError):
        plan.key_count = 0  # type: ignore[misc]


@pytest.mark.parametrize(("keys", "block_count", "message"), [
    ((), 1, "cannot be empty"),
    (("transformer_blocks.0.attn.to_q.alpha",), 0, "must be positive"),
    (("unrecognized.key",), 1, "without a Transformer block index"),
    (("transformer_blocks.2.attn.to_q.alpha",), 2, "outside the model"),
    (("transformer_blocks.0.attn.to_q.alpha", "transformer_blocks.0.attn.to_q.alpha"), 1, "must be unique"),
])
def test_qwen_lora_plan_rejects_invalid_keys(keys, block_count, message):
    with pytest.raises(ValueError, match=message):
        plan_qwen_lora_keys(keys, block_count=block_count)


def test_select_lora_keys_rejects_unknown_blocks():
    plan = plan_qwen_lora_keys(("transformer_blocks.0.attn.to_q.alpha",), block_count=1)
    with pytest.raises(ValueError, match="outside the LoRA plan"):
        select_lora_keys(plan, (1,))


# --- patching checkpoint adapters onto layers ---------------------------------------------------

def test_apply_lora_weights_resolves_key_styles_and_alpha():
    layers = {
        "transformer_blocks.0.img_ff.mlp_in": _layer(128, 64, 1),
        "transformer_blocks.0.attn.to_q": _layer(64, 64, 2),
        "transformer_blocks.1.attn.add_k_proj": _layer(64, 64, 3),
    }
    g = torch.Generator().manual_seed(0)

    def t(*shape):
        return torch.randn(*shape, generator=g).to(torch.bfloat16)

    weights = {
        # diffusers module name + PEFT suffixes: down [r, in], up [out, r]
        "transformer.transformer_blocks.0.img_mlp.net.0.proj.lora_A.weight": t(8, 64),
        "transformer.transformer_blocks.0.img_mlp.net.0.proj.lora_B.weight": t(128, 8),
        # kohya underscored form with alpha
        "lora_unet_transformer_blocks_0_attn_to_q.lora_down.weight": t(4, 64),
        "lora_unet_transformer_blocks_0_attn_to_q.lora_up.weight": t(64, 4),
        "lora_unet_transformer_blocks_0_attn_to_q.alpha": torch.tensor(2.0),
        "transformer_blocks.1.attn.add_k_proj.lora.down.weight": t(16, 64),
        "transformer_blocks.1.attn.add_k_proj.lora.up.weight": t(64, 16),
        "transformer_blocks.7.attn.to_q.lora_A.weight": t(4, 64),  # no such layer: ignored
    }
    applied, matched = apply_lora_weights(layers, weights, scale=0.5)
    assert applied == 3 and len(matched) == 7
    ff = layers["transformer_blocks.0.img_ff.mlp_in"]
    a, b, s = ff.lora
    assert torch.equal(a, weights["transformer.transformer_blocks.0.img_mlp.net.0.proj.lora_A.weight"].T)
    assert torch.equal(b, weights["transformer.transformer_blocks.0.img_mlp.net.0.proj.lora_B.weight"].T)
    assert s == 0.5
    assert layers["transformer_blocks.0.attn.to_q"].lora[2] == pytest.approx(0.5 * 2.0 / 4)
    # a second checkpoint stacks onto the same layer
    applied, _ = apply_lora_weights(layers, {
        "transformer_blocks.0.img_ff.mlp_in.lora_A.weight": t(8, 64),
        "transformer_blocks.0.img_ff.mlp_in.lora_B.weight": t(128, 8),
    }, scale=1.0)
    assert applied == 1 and len(ff.loras) == 2 and ff.lora[0].shape == (64, 16)


def test_apply_lora_weights_rejects_half_pairs_and_bad_shapes():
    layers = {"transformer_blocks.0.attn.to_q": _layer(64, 64, 2)}
    with pytest.raises(ValueError, match="both its down"):
        apply_lora_weights(layers, {"transformer_blocks.0.attn.to_q.lora_A.weight": torch.zeros(4, 64)})
    with pytest.raises(ValueError, match="do not pair"):
        apply_lora_weights(layers, {"transformer_blocks.0.attn.to_q.lora_A.weight": torch.zeros(4, 64),
                                    "transformer_blocks.0.attn.to_q.lora_B.weight": torch.zeros(64, 5)})
    with pytest.raises(ValueError, match="LoRA A must be"):
        apply_lora_weights(layers, {"transformer_blocks.0.attn.to_q.lora_A.weight": torch.zeros(4, 32),
                                    "transformer_blocks.0.attn.to_q.lora_B.weight": torch.zeros(64, 4)})
