"""Host logic of the multi-GPU layouts (qwen_image_shardedit_mlx_b200/sharding.py),
on CPU: token shards, packed-weight slicing at word / group boundaries, and the
tensor-parallel MLP and max-over-ranks timing over a world-size-2 gloo group
(the linears are the oracle's, so no GPU is involved)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle
from qwen_image_shardedit_mlx_b200.sharding import (
    TensorParallelFeedForward,
    max_over_ranks,
    split_k,
    split_rows,
    token_shard,
)


@pytest.mark.parametrize("m", [1, 7, 3456, 3457])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_token_shards_cover_all_tokens_once(m, world):
    shards = [token_shard(m, world, r) for r in range(world)]
    assert shards[0].start == 0 and shards[-1].stop == m
    for a, b in zip(shards, shards[1:]):
        assert a.stop == b.start
    sizes = [s.stop - s.start for s in shards]
    assert max(sizes) - min(sizes) <= 1


def _q6(rng, n, k, gs, bias=True):
    w = rng.normal(0.0, 0.02, size=(n, k)).astype(np.float32)
    packed, scales, biases = oracle.affine_quantize(w, group_size=gs)
    b = oracle.f32_to_bf16_bits(rng.normal(0.0, 0.01, size=(n,)).astype(np.float32)) if bias else None
    return oracle.Q6Weights(packed, scales, biases, b, gs)


def _torch_u32(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.view(np.int32).copy())


def _torch_u16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.view(np.int16).copy())


def _np_q6(weight, scales, biases, bias, gs) -> oracle.Q6Weights:
    return oracle.Q6Weights(weight.numpy().view(np.uint32), scales.numpy().view(np.uint16),
                            biases.numpy().view(np.uint16), None if bias is None else bias.numpy().view(np.uint16), gs)


@pytest.mark.parametrize("k,world,gs", [(12288, 8, 64), (3072, 2, 32), (3072, 4, 128), (1536, 3, 64)])
def test_split_k_cuts_whole_words_and_groups(k, world, gs):
    rng = np.random.default_rng(k + world + gs)
    w = _q6(rng, 24, k, gs)
    codes = oracle.unpack_q6(w.weight, k)
    dense = oracle.dequantize(w.weight, w.scales, w.biases, gs, dtype="f32")
    ks = k // world
    for r in range(world):
        ws, ss, bs = split_k(_torch_u32(w.weight), _torch_u16(w.scales), _torch_u16(w.biases), gs, world, r)
        part = _np_q6(ws, ss, bs, None, gs)
        assert np.array_equal(oracle.unpack_q6(part.weight, ks), codes[:, r * ks:(r + 1) * ks])
        assert np.array_equal(oracle.dequantize(part.weight, part.scales, part.biases, gs, dtype="f32"),
                              dense[:, r * ks:(r + 1) * ks])


def test_split_k_rejects_unaligned_slices():
    w = torch.zeros((4, 3072 * 6 // 32), dtype=torch.int32)
    s = torch.zeros((4, 3072 // 64), dtype=torch.int16)
    with pytest.raises(ValueError):
        split_k(w, s, s, 64, 5, 0)       # 3072 / 5 is not an integer
    with pytest.raises(ValueError):
        split_k(w, s, s, 64, 64, 0)      # 48-code slices cut a 64-code group


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_worker(rank: int, world: int, port: int) -> None:
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(2024)  # same weights and tokens on every rank
        m, d, h, gs = 24, 256, 1024, 64
        fc1 = _q6(rng, h, d, gs)
        fc2 = _q6(rng, d, h, gs)
        x = oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(rng.standard_normal((m, d)).astype(np.float32)))

        w1 = split_rows(_torch_u32(fc1.weight), _torch_u16(fc1.scales), _torch_u16(fc1.biases),
                        _torch_u16(fc1.bias), world, rank)
        w2 = split_k(_torch_u32(fc2.weight), _torch_u16(fc2.scales), _torch_u16(fc2.biases), gs, world, rank)
        fc1_part = _np_q6(*w1, gs)
        fc2_part = _np_q6(*w2, None, gs)

        def fc1_local(t: torch.Tensor) -> torch.Tensor:
            return torch.from_numpy(oracle.linear(t.numpy(), fc1_part, apply_gelu=True, weight_dtype="f32"))

        def fc2_local(t: torch.Tensor) -> torch.Tensor:
            return torch.from_numpy(oracle.linear(t.numpy(), fc2_part, weight_dtype="f32"))

        ff = TensorParallelFeedForward(fc1_local, fc2_local, torch.from_numpy(fc2.bias_f32()))
        got = ff(torch.from_numpy(x)).numpy()
        hidden = oracle.linear(x, fc1, apply_gelu=True, weight_dtype="f32")
        ref = oracle.linear(hidden, fc2, weight_dtype="f32")
        err = float(np.abs(got - ref).max())
        assert err <= 1e-4 * float(np.abs(ref).max()), err

        slowest = max_over_ranks(1.5 + rank)
        assert slowest == 1.5 + (world - 1)
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_mlp_and_max_over_ranks_gloo_world2():
    mp.spawn(_tp_worker, args=(2, _free_port()), nprocs=2, join=True)


def test_max_over_ranks_without_a_group_is_the_value():
    assert max_over_ranks(3.25) == 3.25
