"""MMDiT block host logic on the CPU: rotary tables, the block oracle's own
invariants, block construction and FLOP count."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import block as ob
from oracle.oracle import Q6Weights, affine_quantize
from qwen_image_shardedit_mlx_b200.block import (
    LINEAR_SHAPES,
    NORM_NAMES,
    QwenTransformerBlock,
    block_flops,
    qwen_rope_angles,
)
from qwen_image_shardedit_mlx_b200.q6_metal_mlp import QuantizedLinear
from qwen_image_shardedit_mlx_b200.qwen_block_loader import build_block
from qwen_image_shardedit_mlx_b200.quantize import quantize_affine_q6


@pytest.mark.parametrize("shapes,txt", [([(36, 48)], 256), ([(36, 48), (36, 48)], 256), ([(5, 7)], 3)])
def test_rope_tables_match_the_oracle(shapes, txt):
    img, tx = qwen_rope_angles(shapes, txt)
    oimg, otx = ob.qwen_rope_angles(shapes, txt)
    assert img.shape == (sum(h * w for h, w in shapes), 64) and tx.shape == (txt, 64)
    # the same formula in torch and numpy: equal up to the last bit of a float64 power
    np.testing.assert_allclose(img.numpy(), oimg, rtol=1e-14, atol=0)
    np.testing.assert_allclose(tx.numpy(), otx, rtol=1e-14, atol=0)


def test_rope_table_layout():
    img, tx = qwen_rope_angles([(4, 6), (4, 6)], 5)
    # frame axis: image 0 has angle 0 on its 8 frame frequencies, image 1 angle = frequency
    assert torch.all(img[:24, :8] == 0) and torch.allclose(img[24, :8], img[24, :8] / img[24, 0] * img[24, 0])
    # text positions continue after the largest centred image position (max(4 // 2, 6 // 2) = 3)
    assert torch.allclose(tx[:, 0], torch.arange(3, 8, dtype=torch.float64))


def test_oracle_rope_is_a_rotation():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((7, 256))
    ang = rng.uniform(-3, 3, (7, 64))
    y = ob.rope_pairs(x, np.cos(ang), np.sin(ang))
    pair_norm = lambda a: np.hypot(a.reshape(7, 2, 64, 2)[..., 0], a.reshape(7, 2, 64, 2)[..., 1])  # noqa: E731
    np.testing.assert_allclose(pair_norm(y), pair_norm(x), rtol=1e-12)
    np.testing.assert_allclose(ob.rope_pairs(y, np.cos(-ang), np.sin(-ang)), x, atol=1e-12)


def test_oracle_layernorm_and_rmsnorm():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((5, 512)) * 3 + 1
    n = ob.layernorm_modulate(x, np.zeros(512), np.zeros(512)).astype(np.float64)
    np.testing.assert_allclose(n.mean(axis=1), 0, atol=1e-5)
    np.testing.assert_allclose(n.std(axis=1), 1, atol=1e-4)
    r = ob.rmsnorm_heads(x, np.ones(128))
    np.testing.assert_allclose((r.reshape(5, 4, 128) ** 2).mean(axis=-1), 1, atol=1e-5)


def test_oracle_attention_is_a_weighted_mean():
    rng = np.random.default_rng(2)
    q = rng.standard_normal((9, 256))
    k = rng.standard_normal((9, 256))
    v = np.ones((9, 256))
    np.testing.assert_allclose(ob.attention(q, k, v, 2), 1, atol=1e-12)


def test_block_flops_matches_the_profile_total():
    # 3456 image + 256 text tokens, D = 3072: 840.7 GFLOP of linears, 169.3 of attention, 0.2 of modulation
    assert block_flops(3456, 256, 3072) == 24 * 3712 * 3072 ** 2 + 4 * 3712 ** 2 * 3072 + 24 * 3072 ** 2
    assert abs(block_flops(3456, 256, 3072) / 1e9 - 1010.28) < 0.01


def _linears(dim: int, device="cpu"):
    out = {}
    for name, (fo, fi) in LINEAR_SHAPES.items():
        w, s, b = quantize_affine_q6(torch.randn(fo * dim, fi * dim) * 0.02, 64)
        out[name] = QuantizedLinear(w, s, b, torch.zeros(fo * dim, dtype=torch.bfloat16))
    return out


def test_block_construction_checks():
    lin = _linears(256)
    norms = {n: torch.ones(128) for n in NORM_NAMES}
    blk = QwenTransformerBlock(lin, norms, heads=2)
    assert blk.dim == 256 and blk.img_ff.mlp_in is lin["img_ff.mlp_in"]
    with pytest.raises(ValueError, match="missing"):
        QwenTransformerBlock({k: v for k, v in lin.items() if k != "attn.to_k"}, norms, heads=2)
    with pytest.raises(ValueError, match="heads"):
        QwenTransformerBlock(lin, norms, heads=3)


def test_block_from_loaded_checkpoint_tensors():
    flat = {}
    for name, (fo, fi) in LINEAR_SHAPES.items():
        w, s, b = quantize_affine_q6(torch.randn(fo * 256, fi * 256) * 0.02, 64)
        flat.update({f"{name}.weight": w, f"{name}.scales": s, f"{name}.biases": b,
                     f"{name}.bias": torch.zeros(fo * 256, dtype=torch.bfloat16)})
    for n in NORM_NAMES:
        flat[f"{n}.weight"] = torch.ones(128, dtype=torch.bfloat16)
    blk = QwenTransformerBlock.from_block_weights(build_block(flat))
    assert blk.heads == 2 and set(blk.linears) == set(LINEAR_SHAPES)


def test_oracle_block_runs_and_uses_every_weight():
    rng = np.random.default_rng(3)
    d, heads = 256, 2
    lin = {}
    for name, (fo, fi) in ob.BLOCK_LINEARS.items():
        p, s, b = affine_quantize(rng.normal(0, 0.02, (fo * d, fi * d)).astype(np.float32), group_size=64)
        lin[name] = Q6Weights(p, s, b, None, 64)
    w = ob.BlockWeights(lin, {n: np.ones(128, dtype=np.float32) for n in ob.NORMS}, heads)
    img_a, txt_a = ob.qwen_rope_angles([(4, 6)], 8)
    hidden = rng.standard_normal((24, d)).astype(np.float32)
    enc = rng.standard_normal((8, d)).astype(np.float32)
    temb = rng.standard_normal(d).astype(np.float32)
    t_out, i_out = ob.block_forward(w, hidden, enc, temb, np.cos(img_a), np.sin(img_a), np.cos(txt_a),
                                    np.sin(txt_a))
    assert t_out.shape == (8, d) and i_out.shape == (24, d)
    assert np.isfinite(t_out).all() and np.isfinite(i_out).all()
    # both residual branches move the streams
    assert np.abs(i_out - hidden).max() > 1e-3 and np.abs(t_out - enc).max() > 1e-3
