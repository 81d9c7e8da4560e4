"""Tensor-parallel split of the q6 MLP on one GPU: every rank's shard runs
through the real kernels in turn and the partials are summed on the host, which
is what the all-reduce of TensorParallelFeedForward computes across GPUs."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from qwen_image_shardedit_mlx_b200 import ops
from qwen_image_shardedit_mlx_b200.sharding import split_k, split_rows
from tests.helpers import assert_close, f32, from_bits, random_bf16, random_weights, weights_to_torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_shards_sum_to_the_mlp(world):
    rng = np.random.default_rng(world)
    m, d, h, gs = 256, 3072, 12288, 64
    fc1 = weights_to_torch(random_weights(rng, h, d, gs))
    fc2 = weights_to_torch(random_weights(rng, d, h, gs))
    x = from_bits(random_bf16(rng, (m, d)))
    full = ops.q6_mlp(x, fc1, fc2, group_size=gs)
    total = torch.zeros((m, d), dtype=torch.float32, device="cuda")
    for r in range(world):
        w1 = split_rows(*fc1, world, r)
        w2 = split_k(fc2[0], fc2[1], fc2[2], gs, world, r)
        hid = ops.q6_linear(x, *w1, group_size=gs, apply_gelu=True)
        total += ops.q6_linear(hid, *w2, None, group_size=gs).float()
    total += fc2[3].float()
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    assert_close(f32(total.to(torch.bfloat16)), f32(full), max_abs_rel=3e-2, mean_abs_rel=3e-3,
                 what=f"tp{world}")
