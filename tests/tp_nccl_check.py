"""Tensor-parallel q6 MLP over NCCL, one process per GPU (launched by
tests/test_gpu_tp_nccl.py through torch.distributed.run): fc1 column-parallel,
fc2 row-parallel, one all-reduce; checked against the single-GPU MLP."""

import datetime
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
from qwen_image_shardedit_mlx_b200 import ops
from qwen_image_shardedit_mlx_b200.quantize import random_q6
from qwen_image_shardedit_mlx_b200.sharding import TensorParallelFeedForward, split_k, split_rows
rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"]); local = int(os.environ["LOCAL_RANK"])
torch.cuda.set_device(local)
dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
g = torch.Generator(device="cuda").manual_seed(5)
d, h, m = 3072, 12288, 512
fc1 = (*random_q6(h, d, generator=g, device="cuda"), (torch.randn(h, generator=g, device="cuda") * 0.01).to(torch.bfloat16))
fc2 = (*random_q6(d, h, generator=g, device="cuda"), (torch.randn(d, generator=g, device="cuda") * 0.01).to(torch.bfloat16))
x = torch.randn((m, d), generator=g, device="cuda").to(torch.bfloat16)
w1 = split_rows(*fc1, world, rank)
w2 = split_k(fc2[0], fc2[1], fc2[2], 64, world, rank)
ff = TensorParallelFeedForward(lambda t: ops.q6_linear(t, *w1, apply_gelu=True),
                               lambda t: ops.q6_linear(t, *w2, None), fc2[3])
y = ff(x)
full = ops.q6_mlp(x, fc1, fc2)
torch.cuda.synchronize()
err = (y.float() - full.float()).abs()
rel_max = float(err.max() / full.float().abs().max()); rel_mean = float(err.mean() / full.float().pow(2).mean().sqrt())
ok = rel_max < 3e-2 and rel_mean < 3e-3
print(f"rank {rank}: tp{world} vs single-GPU MLP max_rel {rel_max:.2e} mean_rel {rel_mean:.2e} {'OK' if ok else 'FAIL'}", flush=True)
dist.destroy_process_group()
sys.exit(0 if ok else 1)
