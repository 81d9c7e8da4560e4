"""The context-parallel block layout on CPU over gloo groups.

Each rank keeps rows [r S / W, (r + 1) S / W) of every sample's joint sequence
(S rows, text first) and runs every stage on them with the full weights (the
oracle's linears), in the order ``ContextParallelQwenBlock`` uses: adaLN
modulate with each row's own (sample, stream) vectors, q / k / v of the local
text and image segments, QK-RMSNorm + RoPE at each row's sequence position,
the keys and values of every row all-gathered per sample (the class's own
``_gather_kv``), attention of the local queries over them, the output
projections and the feed-forward with gated residuals on the local rows.  The
rows are the class's own ``local_rows`` / ``local_segments``.  The gathered
output must equal the unsharded oracle block of every sample (no GPU
involved).  Rank boundaries fall inside a sample's text rows, between its text
and image rows, and inside its image rows.
"""

from __future__ import annotations

import os
import types

import numpy as np
import torch
import torch.multiprocessing as mp

import oracle
from oracle import block as ob
from tests.test_block_tp_cpu import _free_port, _full_block, _setup


def _cp_block(w, hidden, enc, temb, rope, world, rank, group=None):
    """This rank's share of the context-parallel block over the ``world``
    ranks of ``group`` (the default group when None); returns the gathered
    joint output [B * S, D]."""

    import torch.distributed as dist

    from qwen_image_shardedit_mlx_b200.block import ContextParallelQwenBlock

    batch, s_img, d = hidden.shape
    s_txt = enc.shape[1]
    seq = s_txt + s_img
    cp = ContextParallelQwenBlock(types.SimpleNamespace(dim=d, heads=w.heads, eps=1e-6), world, rank, group=group)
    r = cp.rows_per_rank(seq)
    r0 = rank * r
    x = np.concatenate([np.concatenate([enc[b], hidden[b]]) for b in range(batch)]).astype(np.float32)
    x_local = cp.local_rows(torch.from_numpy(x), batch, seq).numpy()
    segs = cp.local_segments(batch, seq, s_txt)
    lin = w.linears

    mods = []
    for b in range(batch):
        t = ob.silu(temb[b]).reshape(1, d)
        mods.append((oracle.linear(t, lin["txt_mod_linear"]).reshape(6, d),
                     oracle.linear(t, lin["img_mod_linear"]).reshape(6, d)))

    def modulate(xl, half):
        out = np.empty_like(xl)
        for i in range(xl.shape[0]):
            b, pos = i // r, r0 + i % r
            m = mods[b][int(pos >= s_txt)]
            out[i] = ob.layernorm_modulate(xl[i:i + 1], m[3 * half], m[3 * half + 1])[0]
        return out

    ic, is_, tc, ts = rope
    names = {0: ("attn.add_q_proj", "attn.add_k_proj", "attn.add_v_proj", "attn.norm_added_q", "attn.norm_added_k"),
             1: ("attn.to_q", "attn.to_k", "attn.to_v", "attn.norm_q", "attn.norm_k")}
    z = modulate(x_local, 0)
    q = np.empty_like(x_local)
    k = np.empty_like(x_local)
    v = np.empty_like(x_local)
    for b, s, rows in segs:
        nq, nk, nv, wq, wk = names[s]
        pos = r0 + np.arange(rows.start, rows.stop) - b * r  # positions in the sample's sequence
        c, sn = (tc[pos], ts[pos]) if s == 0 else (ic[pos - s_txt], is_[pos - s_txt])
        q[rows] = ob.qk_rmsnorm_rope(oracle.linear(z[rows], lin[nq]), w.norms[wq], c, sn)
        k[rows] = ob.qk_rmsnorm_rope(oracle.linear(z[rows], lin[nk]), w.norms[wk], c, sn)
        v[rows] = oracle.linear(z[rows], lin[nv])
    kv = cp._gather_kv(torch.from_numpy(np.concatenate([k, v], axis=1)), batch, seq).numpy()
    att = np.empty_like(q)
    for b in range(batch):
        rows = slice(b * r, (b + 1) * r)
        att[rows] = ob.attention(q[rows], kv[b, :, :d], kv[b, :, d:], w.heads).astype(np.float32)
    h = np.empty_like(x_local)
    for b, s, rows in segs:
        h[rows] = oracle.linear(att[rows], lin["attn.to_add_out" if s == 0 else "attn.attn_to_out.0"],
                                residual=x_local[rows], gate=mods[b][s][2])
    z2 = modulate(h, 1)
    y = np.empty_like(x_local)
    for b, s, rows in segs:
        pre = "txt_ff" if s == 0 else "img_ff"
        mid = oracle.linear(z2[rows], lin[f"{pre}.mlp_in"], apply_gelu=True)
        y[rows] = oracle.linear(mid, lin[f"{pre}.mlp_out"], residual=h[rows], gate=mods[b][s][5])
    parts = torch.empty((world * batch * r, d))
    dist.all_gather_into_tensor(parts, torch.from_numpy(y), group=group)
    return parts.view(world, batch, r, d).transpose(0, 1).reshape(batch * seq, d).numpy()


def _worker(rank: int, world: int, port: int, batch: int, s_txt: int) -> None:
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w, hidden, enc, temb, rope = _setup(batch=batch, s_txt=s_txt)
        got = _cp_block(w, hidden, enc, temb, rope, world, rank)
        seq = enc.shape[1] + hidden.shape[1]
        for b in range(batch):
            ref_t, ref_i = _full_block(w, hidden[b], enc[b], temb[b], rope)
            g = got[b * seq:(b + 1) * seq]
            for part, ref in ((g[:s_txt], ref_t), (g[s_txt:], ref_i)):
                err = float(np.abs(part - ref).max())
                assert err <= 1e-4 * float(np.abs(ref).max()), err
    finally:
        dist.destroy_process_group()


def test_context_parallel_block_gloo_world2_one_sample():
    """32 joint rows over 2 ranks: rank 0 holds the 8 text rows and 8 image rows."""

    mp.spawn(_worker, args=(2, _free_port(), 1, 8), nprocs=2, join=True)


def test_context_parallel_block_gloo_world4_two_samples():
    """Two samples of 36 joint rows (12 text) over 4 ranks: 9 rows each, so
    rank 1 starts inside the text rows and ends inside the image rows."""

    mp.spawn(_worker, args=(4, _free_port(), 2, 12), nprocs=4, join=True)


def test_context_parallel_segments():
    """local_segments: the text rows of a rank's share come first, and a
    sequence that does not split over the ranks is refused."""

    from qwen_image_shardedit_mlx_b200.block import ContextParallelQwenBlock

    stub = types.SimpleNamespace(dim=64, heads=1, eps=1e-6)
    segs = [ContextParallelQwenBlock(stub, 4, r).local_segments(2, 36, 12) for r in range(4)]
    assert segs[0] == [(0, 0, slice(0, 9)), (1, 0, slice(9, 18))]
    assert segs[1] == [(0, 0, slice(0, 3)), (0, 1, slice(3, 9)), (1, 0, slice(9, 12)), (1, 1, slice(12, 18))]
    assert segs[3] == [(0, 1, slice(0, 9)), (1, 1, slice(9, 18))]
    try:
        ContextParallelQwenBlock(stub, 5, 0).local_segments(1, 36, 12)
    except ValueError:
        pass
    else:
        raise AssertionError("36 rows over 5 ranks must be refused")


def _groups_worker(rank: int, world: int, port: int, batch: int) -> None:
    import math

    import torch.distributed as dist

    from qwen_image_shardedit_mlx_b200.block import sample_groups

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        samples, size, r_in, group = sample_groups(world, rank, batch)
        g = math.gcd(world, batch)
        assert size == world // g and r_in == rank % size
        per = batch // g
        assert samples == slice((rank // size) * per, (rank // size + 1) * per)
        if size > 1 and g > 1:
            got = torch.empty(size, dtype=torch.float32)
            dist.all_gather_into_tensor(got, torch.tensor([float(rank)]), group=group)
            first = (rank // size) * size
            assert got.tolist() == [float(first + j) for j in range(size)]
        else:
            assert group is None
    finally:
        dist.destroy_process_group()


def test_sample_groups_split_the_batch_then_the_rows():
    """4 ranks, a batch of 2: two groups of 2 ranks, one sample each, whose
    collectives stay inside the group; 2 ranks, a batch of 2: one sample per
    rank and no group; 4 ranks, one sample: every rank in one group."""

    mp.spawn(_groups_worker, args=(4, _free_port(), 2), nprocs=4, join=True)
    mp.spawn(_groups_worker, args=(2, _free_port(), 2), nprocs=2, join=True)
    mp.spawn(_groups_worker, args=(4, _free_port(), 1), nprocs=4, join=True)


def _groups_block_worker(rank: int, world: int, port: int, batch: int, s_txt: int) -> None:
    import torch.distributed as dist

    from qwen_image_shardedit_mlx_b200.block import sample_groups

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w, hidden, enc, temb, rope = _setup(batch=batch, s_txt=s_txt)
        samples, size, r_in, group = sample_groups(world, rank, batch)
        got = _cp_block(w, hidden[samples], enc[samples], temb[samples], rope, size, r_in, group=group)
        seq = enc.shape[1] + hidden.shape[1]
        for i, b in enumerate(range(batch)[samples]):
            ref_t, ref_i = _full_block(w, hidden[b], enc[b], temb[b], rope)
            g = got[i * seq:(i + 1) * seq]
            for part, ref in ((g[:s_txt], ref_t), (g[s_txt:], ref_i)):
                err = float(np.abs(part - ref).max())
                assert err <= 1e-4 * float(np.abs(ref).max()), err
    finally:
        dist.destroy_process_group()


def test_sample_groups_block_gloo_world8_cfg_pair():
    """The 8-GPU layout of the CFG pair: two groups of four ranks, one sample
    each, every sample's 36 joint rows (12 text) split 9 per rank inside its
    group, keys and values gathered over the group only.  Every rank's sample
    must equal the unsharded oracle block."""

    mp.spawn(_groups_block_worker, args=(8, _free_port(), 2, 12), nprocs=8, join=True)
