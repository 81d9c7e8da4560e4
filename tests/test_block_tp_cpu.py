"""The sequence-parallel tensor-parallel block layout on CPU over gloo groups.

Each rank runs the block's stages with the oracle's linears on its shard of
the weights (``split_rows`` for q / k / v and mlp_in, ``split_k`` for the
output projections and mlp_out), in the order ``TensorParallelQwenBlock``
uses: the joint rows [B * S, D] (each sample's text rows, then its image
rows) split into contiguous row shards; adaLN modulate on the local rows
with each row's own (sample, stream) vectors; all-gather of the modulated
rows; local heads; row-parallel partials carrying the gate on every rank and
the output bias on rank 0; reduce-scatter back to the local rows; residual
adds on the local rows.  The gathered output must equal the unsharded oracle
block of every sample (no GPU involved).  Shard boundaries fall inside a
sample's text / image rows and between samples.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import torch
import torch.multiprocessing as mp

import oracle
from oracle import block as ob
from qwen_image_shardedit_mlx_b200.sharding import split_k, split_rows


def _u32(a):
    return torch.from_numpy(a.view(np.int32).copy())


def _u16(a):
    return torch.from_numpy(a.view(np.int16).copy())


def _np(weight, scales, biases, bias, gs):
    return oracle.Q6Weights(weight.numpy().view(np.uint32), scales.numpy().view(np.uint16),
                            biases.numpy().view(np.uint16), None if bias is None else bias.numpy().view(np.uint16),
                            gs)


def _setup(seed=31, d=512, heads=4, s_img=24, s_txt=8, batch=1):
    rng = np.random.default_rng(seed)
    lin = {}
    for name, (fo, fi) in ob.BLOCK_LINEARS.items():
        w = rng.normal(0, 0.02, (fo * d, fi * d)).astype(np.float32)
        p, s, b = oracle.affine_quantize(w, group_size=64)
        bias = oracle.f32_to_bf16_bits(rng.normal(0, 0.01, fo * d).astype(np.float32))
        lin[name] = oracle.Q6Weights(p, s, b, bias, 64)
    norms = {n: (1 + 0.1 * rng.standard_normal(128)).astype(np.float32) for n in ob.NORMS}
    w = ob.BlockWeights(lin, norms, heads)
    hidden = rng.standard_normal((batch, s_img, d)).astype(np.float32)
    enc = rng.standard_normal((batch, s_txt, d)).astype(np.float32)
    temb = rng.standard_normal((batch, d)).astype(np.float32)
    ia, ta = ob.qwen_rope_angles([(4, 6)], s_txt)
    rope = (np.cos(ia), np.sin(ia), np.cos(ta), np.sin(ta))
    return w, hidden, enc, temb, rope


def _tp_block(w, hidden, enc, temb, rope, world, rank):
    """The sequence-parallel layout on this rank; returns the gathered joint output [B * S, D]."""

    import torch.distributed as dist

    batch, s_img, d = hidden.shape
    s_txt = enc.shape[1]
    seq = s_txt + s_img
    lead = rank == 0
    heads = w.heads // world
    rows_local = batch * seq // world
    row0 = rank * rows_local

    def rows(name):
        q = w.linears[name]
        return _np(*split_rows(_u32(q.weight), _u16(q.scales), _u16(q.biases), _u16(q.bias), world, rank), 64)

    def cols(name):
        q = w.linears[name]
        ws, ss, bs = split_k(_u32(q.weight), _u16(q.scales), _u16(q.biases), 64, world, rank)
        return _np(ws, ss, bs, _u16(q.bias) if lead else None, 64)

    def all_gather(local):
        parts = [torch.zeros_like(torch.from_numpy(local)) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(local, dtype=np.float32)))
        return torch.cat(parts).numpy()

    def reduce_scatter(full):
        t = torch.from_numpy(np.ascontiguousarray(full, dtype=np.float32))
        dist.all_reduce(t)  # reduce-scatter's sum, then this rank's rows
        return t.numpy()[row0:row0 + rows_local]

    mods = []
    for b in range(batch):
        t = ob.silu(temb[b]).reshape(1, d)
        mods.append((oracle.linear(t, w.linears["txt_mod_linear"]).reshape(6, d),
                     oracle.linear(t, w.linears["img_mod_linear"]).reshape(6, d)))

    def stream_of(g):  # global joint row -> (sample, stream)
        return g // seq, int(g % seq >= s_txt)

    def modulate(x_local, half):
        out = np.empty_like(x_local)
        for i in range(rows_local):
            b, s = stream_of(row0 + i)
            m = mods[b][s]
            out[i] = ob.layernorm_modulate(x_local[i:i + 1], m[3 * half], m[3 * half + 1])[0]
        return out

    x = np.concatenate([np.concatenate([enc[b], hidden[b]]) for b in range(batch)])
    x_local = x[row0:row0 + rows_local]
    z = all_gather(modulate(x_local, 0))
    ic, is_, tc, ts = rope
    segs = [(b, s, slice(b * seq, b * seq + s_txt) if s == 0 else slice(b * seq + s_txt, (b + 1) * seq))
            for b in range(batch) for s in (0, 1)]
    names = {0: ("attn.add_q_proj", "attn.add_k_proj", "attn.add_v_proj", "attn.norm_added_q", "attn.norm_added_k"),
             1: ("attn.to_q", "attn.to_k", "attn.to_v", "attn.norm_q", "attn.norm_k")}
    dl = heads * 128
    q = np.empty((batch * seq, dl), np.float32)
    k = np.empty_like(q)
    v = np.empty_like(q)
    for b, s, r in segs:
        nq, nk, nv, wq, wk = names[s]
        c, sn = (tc, ts) if s == 0 else (ic, is_)
        q[r] = ob.qk_rmsnorm_rope(oracle.linear(z[r], rows(nq)), w.norms[wq], c, sn)
        k[r] = ob.qk_rmsnorm_rope(oracle.linear(z[r], rows(nk)), w.norms[wk], c, sn)
        v[r] = oracle.linear(z[r], rows(nv))
    att = np.empty_like(q)
    for b in range(batch):
        r = slice(b * seq, (b + 1) * seq)
        att[r] = ob.attention(q[r], k[r], v[r], heads).astype(np.float32)
    part = np.empty((batch * seq, d), np.float32)
    for b, s, r in segs:
        part[r] = oracle.linear(att[r], cols("attn.to_add_out" if s == 0 else "attn.attn_to_out.0"),
                                gate=mods[b][s][2])
    h_local = x_local + reduce_scatter(part)
    z2 = all_gather(modulate(h_local, 1))
    part2 = np.empty((batch * seq, d), np.float32)
    for b, s, r in segs:
        pre = "txt_ff" if s == 0 else "img_ff"
        mid = oracle.linear(z2[r], rows(f"{pre}.mlp_in"), apply_gelu=True)
        part2[r] = oracle.linear(mid, cols(f"{pre}.mlp_out"), gate=mods[b][s][5])
    return all_gather(h_local + reduce_scatter(part2))


def _full_block(w, hidden, enc, temb, rope):
    """The unsharded block with the same (unrounded) arithmetic."""

    d = hidden.shape[1]
    t = ob.silu(temb).reshape(1, d)
    im = oracle.linear(t, w.linears["img_mod_linear"]).reshape(6, d)
    tm = oracle.linear(t, w.linears["txt_mod_linear"]).reshape(6, d)
    img_in = ob.layernorm_modulate(hidden, im[0], im[1])
    txt_in = ob.layernorm_modulate(enc, tm[0], tm[1])
    ic, is_, tc, ts = rope
    lin = w.linears
    q = np.concatenate([ob.qk_rmsnorm_rope(oracle.linear(txt_in, lin["attn.add_q_proj"]), w.norms["attn.norm_added_q"], tc, ts),
                        ob.qk_rmsnorm_rope(oracle.linear(img_in, lin["attn.to_q"]), w.norms["attn.norm_q"], ic, is_)])
    k = np.concatenate([ob.qk_rmsnorm_rope(oracle.linear(txt_in, lin["attn.add_k_proj"]), w.norms["attn.norm_added_k"], tc, ts),
                        ob.qk_rmsnorm_rope(oracle.linear(img_in, lin["attn.to_k"]), w.norms["attn.norm_k"], ic, is_)])
    v = np.concatenate([oracle.linear(txt_in, lin["attn.add_v_proj"]), oracle.linear(img_in, lin["attn.to_v"])])
    joint = ob.attention(q, k, v, w.heads).astype(np.float32)
    s_txt = enc.shape[0]
    txt_h = oracle.linear(joint[:s_txt], lin["attn.to_add_out"], residual=enc, gate=tm[2])
    img_h = oracle.linear(joint[s_txt:], lin["attn.attn_to_out.0"], residual=hidden, gate=im[2])
    img_mid = oracle.linear(ob.layernorm_modulate(img_h, im[3], im[4]), lin["img_ff.mlp_in"], apply_gelu=True)
    txt_mid = oracle.linear(ob.layernorm_modulate(txt_h, tm[3], tm[4]), lin["txt_ff.mlp_in"], apply_gelu=True)
    return (oracle.linear(txt_mid, lin["txt_ff.mlp_out"], residual=txt_h, gate=tm[5]),
            oracle.linear(img_mid, lin["img_ff.mlp_out"], residual=img_h, gate=im[5]))


def _worker(rank: int, world: int, port: int, batch: int) -> None:
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w, hidden, enc, temb, rope = _setup(batch=batch)
        got = _tp_block(w, hidden, enc, temb, rope, world, rank)
        seq = enc.shape[1] + hidden.shape[1]
        for b in range(batch):
            ref_t, ref_i = _full_block(w, hidden[b], enc[b], temb[b], rope)
            g = got[b * seq:(b + 1) * seq]
            for part, r in ((g[:enc.shape[1]], ref_t), (g[enc.shape[1]:], ref_i)):
                err = float(np.abs(part - r).max())
                assert err <= 1e-4 * float(np.abs(r).max()), err
        # the oracle block with bf16 roundings stays close to the unrounded one
        rounded = ob.block_forward(w, hidden[0], enc[0], temb[0], *rope)
        for g, r in zip(rounded, _full_block(w, hidden[0], enc[0], temb[0], rope)):
            assert float(np.abs(g - r).max()) <= 3e-2 * float(np.abs(r).max())
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sequence_parallel_block_gloo_world2_one_sample():
    """32 joint rows over 2 ranks: rank 0 holds the 8 text rows and 8 image rows."""

    mp.spawn(_worker, args=(2, _free_port(), 1), nprocs=2, join=True)


def test_sequence_parallel_block_gloo_world4_two_samples():
    """Two samples (CFG cond / uncond) of 32 joint rows over 4 ranks: shards of
    16 rows, one starting in a sample's text rows, one in its image rows."""

    mp.spawn(_worker, args=(4, _free_port(), 2), nprocs=4, join=True)


class _StubBlock:
    """A block whose modulation vectors are a known function of its index."""

    def __init__(self, i: int, d: int) -> None:
        self.i, self.dim = i, d

    def modulation_joint(self, temb: torch.Tensor) -> torch.Tensor:
        b = temb.shape[0]
        base = torch.arange(b * 2 * 6 * self.dim, dtype=torch.float32).reshape(b, 2, 6, self.dim)
        return (base * 0.001 + self.i + temb.float().sum()).to(torch.bfloat16)


def _mod_worker(rank: int, world: int, port: int, n: int) -> None:
    import torch.distributed as dist

    from qwen_image_shardedit_mlx_b200.block import stack_modulations

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        d = 16
        blocks = [_StubBlock(i, d) for i in range(n)]
        temb = torch.full((2, d), 0.25, dtype=torch.bfloat16)
        got = stack_modulations(blocks, temb, world, rank)
        assert got.shape == (n, 2, 2, 6, d)
        for i, blk in enumerate(blocks):
            assert torch.equal(got[i], blk.modulation_joint(temb)), (rank, i)
    finally:
        dist.destroy_process_group()


def test_stack_modulations_split_over_ranks_gloo():
    """Every rank ends with every block's modulation vectors, each computed
    once somewhere (7 blocks over 4 ranks leave the last rank a short run)."""

    mp.spawn(_mod_worker, args=(4, _free_port(), 7), nprocs=4, join=True)
