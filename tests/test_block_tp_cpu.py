"""The tensor-parallel block layout on CPU over a world-size-2 gloo group.

Each rank runs the block's stages with the oracle's linears on its shard of
the weights (``split_rows`` for q / k / v and mlp_in, ``split_k`` for the
output projections and mlp_out), in the order ``TensorParallelQwenBlock``
uses: local heads, row-parallel partials carrying the residual and bias on
rank 0 and the gate on every rank, an all-reduce after the attention output
and after the feed-forward.  The summed streams must equal the unsharded
oracle block (no GPU involved).
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


def _setup(seed=31, d=256, heads=2, s_img=24, s_txt=8):
    rng = np.random.default_rng(seed)
    lin = {}
    for name, (fo, fi) in ob.BLOCK_LINEARS.items():
        w = rng.normal(0, 0.02, (fo * d, fi * d)).astype(np.float32)
        p, s, b = oracle.affine_quantize(w, group_size=64)
        bias = oracle.f32_to_bf16_bits(rng.normal(0, 0.01, fo * d).astype(np.float32))
        lin[name] = oracle.Q6Weights(p, s, b, bias, 64)
    norms = {n: (1 + 0.1 * rng.standard_normal(128)).astype(np.float32) for n in ob.NORMS}
    w = ob.BlockWeights(lin, norms, heads)
    hidden = rng.standard_normal((s_img, d)).astype(np.float32)
    enc = rng.standard_normal((s_txt, d)).astype(np.float32)
    temb = rng.standard_normal(d).astype(np.float32)
    ia, ta = ob.qwen_rope_angles([(4, 6)], s_txt)
    rope = (np.cos(ia), np.sin(ia), np.cos(ta), np.sin(ta))
    return w, hidden, enc, temb, rope


def _tp_block(w, hidden, enc, temb, rope, world, rank):
    import torch.distributed as dist

    d, lead = hidden.shape[1], rank == 0
    heads = w.heads // world

    def rows(name):
        q = w.linears[name]
        return _np(*split_rows(_u32(q.weight), _u16(q.scales), _u16(q.biases), _u16(q.bias), world, rank), 64)

    def cols(name):
        q = w.linears[name]
        ws, ss, bs = split_k(_u32(q.weight), _u16(q.scales), _u16(q.biases), 64, world, rank)
        return _np(ws, ss, bs, _u16(q.bias) if lead else None, 64)

    def allreduce(a):
        t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
        dist.all_reduce(t)
        return t.numpy()

    t = ob.silu(temb).reshape(1, d)
    im = oracle.linear(t, w.linears["img_mod_linear"]).reshape(6, d)
    tm = oracle.linear(t, w.linears["txt_mod_linear"]).reshape(6, d)
    img_in = ob.layernorm_modulate(hidden, im[0], im[1])
    txt_in = ob.layernorm_modulate(enc, tm[0], tm[1])
    ic, is_, tc, ts = rope
    q = np.concatenate([ob.qk_rmsnorm_rope(oracle.linear(txt_in, rows("attn.add_q_proj")), w.norms["attn.norm_added_q"], tc, ts),
                        ob.qk_rmsnorm_rope(oracle.linear(img_in, rows("attn.to_q")), w.norms["attn.norm_q"], ic, is_)])
    k = np.concatenate([ob.qk_rmsnorm_rope(oracle.linear(txt_in, rows("attn.add_k_proj")), w.norms["attn.norm_added_k"], tc, ts),
                        ob.qk_rmsnorm_rope(oracle.linear(img_in, rows("attn.to_k")), w.norms["attn.norm_k"], ic, is_)])
    v = np.concatenate([oracle.linear(txt_in, rows("attn.add_v_proj")), oracle.linear(img_in, rows("attn.to_v"))])
    joint = ob.attention(q, k, v, heads).astype(np.float32)
    s_txt = enc.shape[0]
    streams = np.concatenate([
        oracle.linear(joint[:s_txt], cols("attn.to_add_out"), residual=enc if lead else None, gate=tm[2]),
        oracle.linear(joint[s_txt:], cols("attn.attn_to_out.0"), residual=hidden if lead else None, gate=im[2]),
    ])
    streams = allreduce(streams)
    txt_h, img_h = streams[:s_txt], streams[s_txt:]
    img_mid = oracle.linear(ob.layernorm_modulate(img_h, im[3], im[4]), rows("img_ff.mlp_in"), apply_gelu=True)
    txt_mid = oracle.linear(ob.layernorm_modulate(txt_h, tm[3], tm[4]), rows("txt_ff.mlp_in"), apply_gelu=True)
    outs = np.concatenate([
        oracle.linear(txt_mid, cols("txt_ff.mlp_out"), residual=txt_h if lead else None, gate=tm[5]),
        oracle.linear(img_mid, cols("img_ff.mlp_out"), residual=img_h if lead else None, gate=im[5]),
    ])
    outs = allreduce(outs)
    return outs[:s_txt], outs[s_txt:]


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


def _worker(rank: int, world: int, port: int) -> None:
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        args = _setup()
        got = _tp_block(*args, world, rank)
        ref = _full_block(*args)
        for g, r in zip(got, ref):
            err = float(np.abs(g - r).max())
            assert err <= 1e-4 * float(np.abs(r).max()), err
        # the oracle block with bf16 roundings stays close to the unrounded one
        rounded = ob.block_forward(*args[:4], *args[4])
        for g, r in zip(rounded, ref):
            assert float(np.abs(g - r).max()) <= 3e-2 * float(np.abs(r).max())
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_tensor_parallel_block_gloo_world2():
    mp.spawn(_worker, args=(2, _free_port()), nprocs=2, join=True)
