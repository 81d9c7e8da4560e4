"""Multi-GPU MMDiT block forms, one process per GPU (launched by
tests/test_gpu_block.py through torch.distributed.run), two samples per call,
each checked against the single-GPU block: the sequence-parallel
tensor-parallel block over NCCL and over peer memory (heads and FF columns
split, joint rows sharded between the GEMMs: all-gather before each
column-parallel GEMM, reduce-scatter after each row-parallel one), and the
context-parallel block (every rank the full weights and 1 / N of each
sample's rows, keys and values all-gathered for the attention), also with the
two samples first split over rank groups (``sample_groups``)."""

import datetime
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
from qwen_image_shardedit_mlx_b200.block import (  # noqa: E402
    ContextParallelQwenBlock,
    QwenTransformerBlock,
    TensorParallelQwenBlock,
    qwen_rope_angles,
    rope_tables,
    sample_groups,
)

rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"]); local = int(os.environ["LOCAL_RANK"])
torch.cuda.set_device(local)
dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
g = torch.Generator(device="cuda").manual_seed(11)
dim, heads = 1024, 8
full = QwenTransformerBlock.random(dim, heads, generator=g)
hidden = torch.randn((2, 600, dim), generator=g, device="cuda").to(torch.bfloat16)
enc = torch.randn((2, 64, dim), generator=g, device="cuda").to(torch.bfloat16)
temb = torch.randn((2, dim), generator=g, device="cuda").to(torch.bfloat16)
ia, ta = qwen_rope_angles([(20, 30)], 64)
rope = rope_tables(ia, ta, "cuda")
ref = full(hidden, enc, temb, rope)
ok = True
for comm in ("nccl", "peer", "cp", "cp-sp"):
    want = ref
    if comm == "cp-sp":  # the two samples split over rank groups, rows split within each group
        samples, size, r_in, grp = sample_groups(world, rank, 2)
        out = ContextParallelQwenBlock(full, size, r_in, group=grp)(hidden[samples], enc[samples], temb[samples],
                                                                    rope)
        want = (ref[0][samples], ref[1][samples])
    elif comm == "cp":
        out = ContextParallelQwenBlock(full, world, rank)(hidden, enc, temb, rope)
    else:
        out = TensorParallelQwenBlock(full, world, rank, comm=comm)(hidden, enc, temb, rope)
    torch.cuda.synchronize()
    for name, a, b in (("text", out[0], want[0]), ("image", out[1], want[1])):
        err = (a.float() - b.float()).abs()
        rel_max = float(err.max() / b.float().abs().max())
        rel_mean = float(err.mean() / b.float().pow(2).mean().sqrt())
        good = rel_max < 3e-2 and rel_mean < 3e-3
        ok = ok and good
        print(f"rank {rank}: tp{world} {comm} {name} stream vs single-GPU block max_rel {rel_max:.2e} "
              f"mean_rel {rel_mean:.2e}", flush=True)
from qwen_image_shardedit_mlx_b200 import ops  # noqa: E402

ok = ok and ops.device_error() == 0
print(f"rank {rank}: {'OK' if ok else 'FAIL'}", flush=True)
dist.destroy_process_group()
sys.exit(0 if ok else 1)
