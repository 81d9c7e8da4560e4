"""Multi-GPU layouts of the q6 feed-forward: token sharding and tensor parallelism.

One process per GPU; torch.distributed (NCCL on GPUs, gloo in the CPU tests)
carries the few host-side collectives.

* Token sharding: every rank runs the whole MLP on its own slice of the
  tokens with replicated weights; the MLP needs no collective (weak scaling
  in ``bench.py``).
* Tensor parallelism: fc1 is column-parallel (each rank holds a contiguous
  block of output rows of the packed codes, scales and biases) and fc2 is
  row-parallel (each rank holds a contiguous K slice of every row, cut at a
  16-code / scale-group boundary so the packed words and groups split
  cleanly: 12288 / 8 = 1536 codes = 288 words = 24 gs64 groups).  Each rank
  computes fc2's partial product without the output bias; an all-reduce sums
  the partials and the bias is added once.
"""

from __future__ import annotations

from typing import Callable

import torch


def token_shard(m: int, world: int, rank: int) -> slice:
    """Contiguous, balanced slice of ``m`` tokens for ``rank`` (the first
    ``m % world`` ranks take one extra token)."""

    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(m, world)
    start = rank * base + min(rank, extra)
    return slice(start, start + base + (1 if rank < extra else 0))


def split_rows(weight: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, bias: torch.Tensor | None,
               world: int, rank: int):
    """Column-parallel slice (output features) of a packed q6 linear: rows
    ``[rank N / world, (rank + 1) N / world)`` of codes, scales, biases and bias."""

    n = weight.shape[0]
    if n % world:
        raise ValueError(f"{n} output rows do not split over {world} ranks")
    rows = slice(rank * (n // world), (rank + 1) * (n // world))
    return (weight[rows].contiguous(), scales[rows].contiguous(), biases[rows].contiguous(),
            None if bias is None else bias[rows].contiguous())


def split_k(weight: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group_size: int, world: int,
            rank: int):
    """Row-parallel slice (input features) of a packed q6 linear: codes
    ``[rank K / world, (rank + 1) K / world)`` of every row, as whole uint32
    words (16 codes = 3 words) and whole scale groups."""

    words = weight.shape[1]
    k = words * 32 // 6
    if k % world:
        raise ValueError(f"K = {k} does not split over {world} ranks")
    ks = k // world
    if ks % 16 or ks % group_size:
        raise ValueError(f"K slice {ks} must be a multiple of 16 codes and of group_size {group_size}")
    w_cols = slice(rank * ks * 6 // 32, (rank + 1) * ks * 6 // 32)
    g_cols = slice(rank * ks // group_size, (rank + 1) * ks // group_size)
    return weight[:, w_cols].contiguous(), scales[:, g_cols].contiguous(), biases[:, g_cols].contiguous()


def max_over_ranks(value: float, device: torch.device | str | None = None) -> float:
    """Max of a per-rank scalar over the default process group (the value
    itself without one).  Timings are reported as the slowest rank's."""

    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class TensorParallelFeedForward(torch.nn.Module):
    """fc2(gelu(fc1(x))) with fc1 column-parallel and fc2 row-parallel.

    ``fc1_local(x)`` must return this rank's slice of gelu(fc1(x) + b1), and
    ``fc2_local(h)`` this rank's partial fc2 product without the output bias
    (for the q6 layers: ``split_rows`` of fc1 run with GELU, and ``split_k`` of
    fc2 run with ``bias=None``).  The partials are summed with an all-reduce
    over ``group`` and ``bias2`` is added once.
    """

    def __init__(self, fc1_local: Callable[[torch.Tensor], torch.Tensor],
                 fc2_local: Callable[[torch.Tensor], torch.Tensor], bias2: torch.Tensor | None = None,
                 group=None) -> None:
        super().__init__()
        self.fc1_local = fc1_local
        self.fc2_local = fc2_local
        self.bias2 = bias2
        self.group = group

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        partial = self.fc2_local(self.fc1_local(x))
        if dist.is_available() and dist.is_initialized() and dist.get_world_size(self.group) > 1:
            dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group)
        if self.bias2 is not None:
            partial = partial + self.bias2.to(partial.dtype)
        return partial
