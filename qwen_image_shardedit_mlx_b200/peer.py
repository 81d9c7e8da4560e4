"""Peer-memory buffers and calls for the sequence-parallel tensor-parallel block.

The tensor-parallel block (``block.TensorParallelQwenBlock`` with
``comm="peer"``) replaces the NCCL reduce-scatter / all-gather pair around
each half of the block by one fused kernel per half
(``q6_sp_add_layernorm_gather_bf16``): it reads every rank's row-parallel
partial sums for its own rows, adds the residual, applies the adaLN
modulate, and writes the modulated rows straight into every rank's gather
buffer.  Those buffers must be addressable from every GPU of the group, so
they are torch symmetric-memory allocations (CUDA peer mappings); a
``q6_sp_barrier`` between the phases orders the ranks.

One ``PeerRows`` serves every block of a stack: its four row buffers
(``gather1`` / ``gather2`` receive the modulated rows before the q/k/v and
feed-forward GEMMs, ``part1`` / ``part2`` hold this rank's partial sums of
the output projection and of the feed-forward) are reused from block to
block, the barriers making each reuse safe.
"""

from __future__ import annotations

import ctypes

import torch

from qwen_image_shardedit_mlx_b200 import _lib, ops

BARRIER_TIMEOUT_NS = 2_000_000_000


class PeerRows:
    """Symmetric row buffers [rows_total, dim] bf16 of one process group."""

    NAMES = ("gather1", "gather2", "part1", "part2")

    def __init__(self, rows_total: int, dim: int, group=None, device: torch.device | str | None = None) -> None:
        import torch.distributed as dist

        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        distributed = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if distributed else 1
        self.rank = dist.get_rank(group) if distributed else 0
        if self.world > 8:
            raise ValueError("the peer kernels take at most 8 ranks")
        if rows_total % self.world:
            raise ValueError(f"{rows_total} rows do not split over {self.world} ranks")
        self.rows_total, self.dim, self.group = int(rows_total), int(dim), group
        self.rows_local = self.rows_total // self.world
        self.buffers: dict[str, torch.Tensor] = {}
        self.ptrs: dict[str, ctypes.Array] = {}
        self._handles = []
        if self.world == 1:
            for name in self.NAMES:
                t = torch.empty((self.rows_total, self.dim), dtype=torch.bfloat16, device=self.device)
                self.buffers[name] = t
                self.ptrs[name] = (ctypes.c_void_p * 1)(t.data_ptr())
            self.signals = torch.zeros(8, dtype=torch.int32, device=self.device)
            self.signal_ptrs = (ctypes.c_void_p * 1)(self.signals.data_ptr())
        else:
            import torch.distributed._symmetric_memory as symm_mem

            gname = group.group_name if group is not None else dist.group.WORLD.group_name
            for name in self.NAMES:
                t = symm_mem.empty((self.rows_total, self.dim), dtype=torch.bfloat16, device=self.device)
                h = symm_mem.rendezvous(t, gname)
                self._handles.append(h)
                self.buffers[name] = t
                self.ptrs[name] = (ctypes.c_void_p * self.world)(*[int(p) for p in h.buffer_ptrs])
            s = symm_mem.empty((8,), dtype=torch.int32, device=self.device)
            h = symm_mem.rendezvous(s, gname)
            self._handles.append(h)
            s.zero_()
            self.signals = s
            self.signal_ptrs = (ctypes.c_void_p * self.world)(*[int(p) for p in h.buffer_ptrs])
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=group)

    def local(self, name: str) -> torch.Tensor:
        """This rank's own-row block of a buffer."""

        r = self.rows_local
        return self.buffers[name][self.rank * r:(self.rank + 1) * r]

    def barrier(self, timeout_ns: int = BARRIER_TIMEOUT_NS) -> None:
        st = _lib.lib().q6_sp_barrier(self.signal_ptrs, self.epoch.data_ptr(), self.world, self.rank, int(timeout_ns),
                                      ops._stream(self.device))
        _lib.check(st, "q6_sp_barrier")

    def add_ln_gather(self, x_local: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, *, dst: str | None,
                      partials: str | None = None, h_out: torch.Tensor | None = None, seq_len: int = 0,
                      text_len: int = 0, eps: float = 1e-6) -> None:
        """h = x_local + sum of every rank's ``partials`` rows (when given) into
        ``h_out``; LayerNorm(h) * (1 + scale) + shift into the own rows of every
        rank's ``dst`` buffer (skipped when ``dst`` is None)."""

        if x_local.shape != (self.rows_local, self.dim) or not x_local.is_contiguous():
            raise ValueError(f"x_local must be contiguous ({self.rows_local}, {self.dim})")
        from qwen_image_shardedit_mlx_b200.block import vector_stride

        vs = 0 if shift is None else vector_stride(shift, scale, self.dim)
        st = _lib.lib().q6_sp_add_layernorm_gather_bf16(
            x_local.data_ptr(), None if partials is None else self.ptrs[partials],
            None if h_out is None else h_out.data_ptr(), None if shift is None else shift.data_ptr(),
            None if scale is None else scale.data_ptr(), vs,
            None if dst is None else self.ptrs[dst], self.world, self.rank, self.rows_local, self.dim, int(seq_len),
            int(text_len), float(eps), ops._stream(self.device))
        _lib.check(st, "q6_sp_add_layernorm_gather_bf16")
