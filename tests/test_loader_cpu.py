"""Checkpoint loading on the CPU: safetensors container, shard plans, block windows.

The shard-plan cases restate the reference's own tests
(tests/test_sweep_profile.py:10-48); the container is cross-checked against
the independent ``safetensors`` package in both directions.
"""

from __future__ import annotations

from dataclasses import FrozenInstanceError
import json

import numpy as np
import pytest
import torch

from qwen_image_shardedit_mlx_b200.qwen_block_loader import (
    LoadedBlock,
    QwenBlockWeights,
    block_layers,
    build_block,
    load_block_window,
    load_safetensors,
    load_transformer_layout,
    plan_transformer_block_shards,
    read_safetensors_header,
    save_safetensors,
)
from qwen_image_shardedit_mlx_b200.quantize import quantize_affine_q6, unpack_codes


def _mixed_tensors() -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(3)
    w, s, b = quantize_affine_q6(torch.randn(96, 128, generator=g) * 0.02, 64)
    return {
        "a.weight": w,                                                  # U32
        "a.scales": s, "a.biases": b,                                   # BF16
        "a.bias": torch.randn(96, generator=g).to(torch.float16),      # F16
        "norm.weight": torch.randn(7, 3, generator=g),                  # F32
        "steps": torch.arange(5, dtype=torch.int64),
        "empty": torch.zeros((0, 4), dtype=torch.float32),
    }


def _same(a: torch.Tensor, b: torch.Tensor) -> bool:
    if a.dtype != b.dtype or a.shape != b.shape:
        return False
    return bool(torch.equal(a.reshape(-1).view(torch.uint8), b.reshape(-1).view(torch.uint8))) if a.numel() else True


def test_safetensors_round_trip_own_writer(tmp_path):
    t = _mixed_tensors()
    p = tmp_path / "x.safetensors"
    save_safetensors(p, t, metadata={"format": "mlx"})
    entries, meta = read_safetensors_header(p)
    assert meta == {"format": "mlx"}
    assert entries["a.weight"].dtype == "U32" and entries["a.scales"].dtype == "BF16"
    got = load_safetensors(p)
    assert set(got) == set(t)
    for name in t:
        assert _same(got[name], t[name]), name
    sub = load_safetensors(p, ["a.scales", "steps"])
    assert set(sub) == {"a.scales", "steps"} and _same(sub["steps"], t["steps"])


def test_safetensors_matches_the_safetensors_package(tmp_path):
    st = pytest.importorskip("safetensors.torch")
    t = _mixed_tensors()
    theirs = tmp_path / "theirs.safetensors"
    st.save_file({k: v.contiguous() for k, v in t.items()}, str(theirs))
    got = load_safetensors(theirs)
    for name in t:
        assert _same(got[name], t[name]), name
    ours = tmp_path / "ours.safetensors"
    save_safetensors(ours, t)
    back = st.load_file(str(ours))
    for name in t:
        assert _same(back[name], t[name]), name


def test_safetensors_rejects_corrupt_files(tmp_path):
    p = tmp_path / "bad.safetensors"
    p.write_bytes(b"\x01\x02")
    with pytest.raises(ValueError, match="short header"):
        read_safetensors_header(p)
    header = json.dumps({"t": {"dtype": "F32", "shape": [4], "data_offsets": [0, 12]}}).encode()
    p.write_bytes(len(header).to_bytes(8, "little") + header + b"\0" * 16)
    with pytest.raises(ValueError, match="do not match"):
        read_safetensors_header(p)
    header = json.dumps({"t": {"dtype": "Q9", "shape": [1], "data_offsets": [0, 1]}}).encode()
    p.write_bytes(len(header).to_bytes(8, "little") + header + b"\0")
    with pytest.raises(ValueError, match="unsupported dtype"):
        read_safetensors_header(p)
    p.write_bytes((1 << 40).to_bytes(8, "little"))
    with pytest.raises(ValueError, match="invalid"):
        read_safetensors_header(p)
    save_safetensors(p, {"t": torch.ones(2)})
    with pytest.raises(KeyError):
        load_safetensors(p, ["u"])


# --- shard plans (reference tests/test_sweep_profile.py) ----------------------------------------

def test_block_shard_plan_counts_tensors_and_shards():
    plans = plan_transformer_block_shards(
        {
            "transformer_blocks.0.attn.weight": "part-1.safetensors",
            "transformer_blocks.0.mlp.weight": "part-1.safetensors",
            "transformer_blocks.1.attn.weight": "part-1.safetensors",
            "transformer_blocks.1.mlp.weight": "part-2.safetensors",
            "proj_out.weight": "part-2.safetensors",
        },
        block_count=2,
    )
    assert plans[0].tensor_count == 2
    assert plans[0].shards == ("part-1.safetensors",)
    assert plans[1].shards == ("part-1.safetensors", "part-2.safetensors")


def test_block_shard_plan_is_immutable():
    plan = plan_transformer_block_shards({"transformer_blocks.0.weight": "part.safetensors"}, block_count=1)[0]
    with pytest.raises(FrozenInstanceError):
        plan.tensor_count = 0  # type: ignore[misc]


def test_block_shard_plan_does_not_confuse_block_1_with_block_10():
    wm = {f"transformer_blocks.{i}.w": "p.safetensors" for i in range(12)}
    wm["transformer_blocks.10.v"] = "q.safetensors"
    plans = plan_transformer_block_shards(wm, block_count=12)
    assert plans[1].tensor_count == 1 and plans[10].tensor_count == 2
    assert plans[10].shards == ("p.safetensors", "q.safetensors")


@pytest.mark.parametrize(("weight_map", "block_count"), [
    ({}, 1),
    ({"transformer_blocks.0.weight": "part.safetensors"}, 0),
    ({"transformer_blocks.0.weight": "part.safetensors"}, 2),
])
def test_block_shard_plan_rejects_incomplete_layouts(weight_map, block_count):
    with pytest.raises(ValueError):
        plan_transformer_block_shards(weight_map, block_count=block_count)


# --- a small synthetic checkpoint -----------------------------------------------------------

D, H = 128, 256


def _block_tensors(i: int, gs: int = 64) -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(100 + i)
    out = {}
    for name, (n, k) in {"img_ff.mlp_in": (H, D), "img_ff.mlp_out": (D, H), "attn.to_q": (D, D)}.items():
        w, s, b = quantize_affine_q6(torch.randn(n, k, generator=g) * 0.02, gs)
        out[f"{name}.weight"], out[f"{name}.scales"], out[f"{name}.biases"] = w, s, b
        out[f"{name}.bias"] = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16)
    out["norm1.weight"] = torch.ones(D, dtype=torch.bfloat16)
    return {f"transformer_blocks.{i}.{k}": v for k, v in out.items()}


def write_checkpoint(root, blocks: int = 3, shards: int = 2, gs: int = 64) -> dict[str, torch.Tensor]:
    tdir = root / "transformer"
    tdir.mkdir(parents=True)
    every: dict[str, torch.Tensor] = {}
    weight_map = {}
    for i in range(blocks):
        t = _block_tensors(i, gs)
        every.update(t)
        names = sorted(t)
        for j, name in enumerate(names):  # spread each block over the shards
            weight_map[name] = f"model-{j % shards + 1:05d}-of-{shards:05d}.safetensors"
    for shard in sorted(set(weight_map.values())):
        save_safetensors(tdir / shard, {n: every[n] for n, s in weight_map.items() if s == shard})
    (tdir / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": weight_map}))
    return every


def test_layout_and_block_window_on_host(tmp_path):
    every = write_checkpoint(tmp_path, blocks=3, shards=2)
    layout = load_transformer_layout(tmp_path, block_count=3)
    assert [p.block_index for p in layout.plans] == [0, 1, 2]
    assert all(p.tensor_count == 13 for p in layout.plans)
    blocks = load_block_window(layout, (1, 2), device="cpu")
    assert [b.block_index for b in blocks] == [1, 2]
    blk = blocks[0].module
    assert isinstance(blocks[0], LoadedBlock) and isinstance(blk, QwenBlockWeights)
    assert set(blk.linears) == {"img_ff.mlp_in", "img_ff.mlp_out", "attn.to_q"}
    assert set(blk.tensors) == {"norm1.weight"}
    lin = blk.linears["img_ff.mlp_in"]
    assert (lin.in_features, lin.out_features, lin.group_size) == (D, H, 64)
    assert torch.equal(unpack_codes(lin.weight, D), unpack_codes(every["transformer_blocks.1.img_ff.mlp_in.weight"], D))
    assert torch.equal(lin.scales, every["transformer_blocks.1.img_ff.mlp_in.scales"])
    assert torch.equal(lin.bias, every["transformer_blocks.1.img_ff.mlp_in.bias"])
    assert blk.img_ff.mlp_in is lin and not hasattr(blk, "txt_ff")
    assert blk.nbytes() > 0
    names = block_layers(blocks)
    assert "transformer_blocks.2.attn.to_q" in names and len(names) == 6


@pytest.mark.parametrize("gs", [32, 128])
def test_group_size_follows_the_shapes(tmp_path, gs):
    write_checkpoint(tmp_path, blocks=1, shards=1, gs=gs)
    layout = load_transformer_layout(tmp_path, block_count=1)
    blk = load_block_window(layout, (0,), device="cpu")[0].module
    assert {lin.group_size for lin in blk.linears.values()} == {gs}
    with pytest.raises(ValueError, match="group size"):
        load_block_window(layout, (0,), device="cpu", group_size=64 if gs != 64 else 32)


def test_layout_errors(tmp_path):
    with pytest.raises(FileNotFoundError, match="missing Transformer index"):
        load_transformer_layout(tmp_path)
    write_checkpoint(tmp_path, blocks=2, shards=2)
    (tmp_path / "transformer" / "model-00002-of-00002.safetensors").unlink()
    with pytest.raises(FileNotFoundError, match="missing Transformer shards"):
        load_transformer_layout(tmp_path, block_count=2)
    (tmp_path / "transformer" / "model.safetensors.index.json").write_text(json.dumps({"weight_map": [1]}))
    with pytest.raises(ValueError, match="invalid weight_map"):
        load_transformer_layout(tmp_path, block_count=2)


def test_block_window_argument_errors(tmp_path):
    write_checkpoint(tmp_path, blocks=3, shards=1)
    layout = load_transformer_layout(tmp_path, block_count=3)
    with pytest.raises(ValueError, match="cannot be empty"):
        load_block_window(layout, (), device="cpu")
    with pytest.raises(ValueError, match="consecutive"):
        load_block_window(layout, (0, 2), device="cpu")
    with pytest.raises(ValueError, match="unknown Transformer block"):
        load_block_window(layout, (2, 3), device="cpu")


def test_build_block_rejects_unpaired_quantized_tensors():
    w, s, b = quantize_affine_q6(torch.randn(64, 64) * 0.02, 64)
    with pytest.raises(ValueError, match="no scales"):
        build_block({"x.weight": w, "x.scales": s})
    with pytest.raises(ValueError, match="do not agree"):
        build_block({"x.weight": w, "x.scales": s, "x.biases": b[:1]})
    with pytest.raises(ValueError, match="bits=6"):
        build_block({"x.weight": w, "x.scales": s, "x.biases": b}, bits=4)
    blk = build_block({"x.weight": w.view(torch.int32), "x.scales": s, "x.biases": b, "y": torch.ones(2)})
    assert blk.linears["x"].weight.dtype == torch.uint32 and np.array_equal(blk.tensors["y"].numpy(), [1, 1])
