"""GPU parity of the MMDiT block pieces and of whole blocks against the block oracle.

* ``q6_layernorm_modulate_bf16`` and ``q6_qk_rmsnorm_rope_bf16`` against the
  oracle's float64 restatements, rounded to bf16 once;
* whole blocks (every q6 linear, the fused epilogues, the attention) at
  reduced widths against ``oracle.block.block_forward``, which rounds to bf16
  where the GPU path stores bf16 (north-star matmul tolerance on the outputs);
* the full Qwen-Image block shape (3072 wide, 24 heads, 3456 + 256 tokens)
  runs and stays finite.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_close, f32, from_bits, random_bf16, random_weights, weights_to_torch
from oracle import block as ob
from qwen_image_shardedit_mlx_b200 import _lib
from qwen_image_shardedit_mlx_b200.block import (
    QwenTransformerBlock,
    layernorm_modulate,
    qk_rmsnorm_rope_,
    qwen_rope_angles,
    rope_tables,
)
from qwen_image_shardedit_mlx_b200.q6_metal_mlp import QuantizedLinear

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,d", [(1, 256), (37, 768), (130, 3072), (3456, 3072)])
def test_layernorm_modulate_vs_oracle(m, d):
    rng = np.random.default_rng(m + d)
    x = random_bf16(rng, (m, d), 2.0)
    shift = random_bf16(rng, (d,), 0.5)
    scale = random_bf16(rng, (d,), 0.5)
    got = layernorm_modulate(from_bits(x), from_bits(shift), from_bits(scale))
    torch.cuda.synchronize()
    ref = ob.layernorm_modulate(oracle.bf16_bits_to_f32(x), oracle.bf16_bits_to_f32(shift),
                                oracle.bf16_bits_to_f32(scale))
    refb = oracle.round_bf16(ref)
    g = f32(got)
    # one fp32 pass vs float64: equal after the bf16 rounding but for rare one-unit flips
    assert np.mean(g == refb) > 0.99
    assert np.all(np.abs(g - refb) <= 2.0 ** -7 * np.abs(refb) + 1e-6)


def test_layernorm_modulate_rejects_bad_arguments():
    x = torch.zeros((4, 320), dtype=torch.bfloat16, device="cuda")
    v = torch.zeros(320, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.Q6Error):  # D not a multiple of 256
        layernorm_modulate(x, v, v)
    x = torch.zeros((4, 1280), dtype=torch.bfloat16, device="cuda")
    v = torch.zeros(1280, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.Q6Error):  # 5 x 256: no instantiation
        layernorm_modulate(x, v, v)


def test_add_layernorm_modulate_strided_vectors_match_contiguous():
    """Modulation vectors read in place from the [B, 2, 6, D] modulation
    output (rows 6 D apart) give the same bits as contiguous copies."""

    from qwen_image_shardedit_mlx_b200.block import ModulationVectors, add_layernorm_modulate

    g = torch.Generator(device="cuda").manual_seed(5)
    b, seq, txt, d = 2, 40, 9, 768
    both = torch.randn((b, 2, 6, d), generator=g, device="cuda").to(torch.bfloat16)
    x = torch.randn((b * seq, d), generator=g, device="cuda").to(torch.bfloat16)
    add = torch.randn((b * seq, d), generator=g, device="cuda").to(torch.bfloat16)
    vec = ModulationVectors(both)
    assert vec.shift2.stride(0) == 6 * d
    h1, h2 = torch.empty_like(x), torch.empty_like(x)
    y1 = add_layernorm_modulate(x, vec.shift2, vec.scale2, add=add, h_out=h1, seq_len=seq, text_len=txt)
    y2 = add_layernorm_modulate(x, vec.shift2.contiguous(), vec.scale2.contiguous(), add=add, h_out=h2,
                                seq_len=seq, text_len=txt)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2) and torch.equal(h1, h2)
    # row 0 of sample 1 is a text row: vector 2 (sample 1, text)
    row = seq
    hrow = h1[row].float()
    ln = (hrow - hrow.mean()) / torch.sqrt(hrow.var(unbiased=False) + 1e-6)
    want = ln * (1 + both[1, 0, 4].float()) + both[1, 0, 3].float()
    assert torch.allclose(y1[row].float(), want, atol=3e-2, rtol=2e-2)


@pytest.mark.parametrize("m,heads,extra", [(1, 2, 0), (45, 6, 64), (3456, 24, 0), (256, 24, 256), (37, 3, 0),
                                            (100, 5, 8), (9, 1, 0), (7, 11, 128)])
def test_qk_rmsnorm_rope_vs_oracle(m, heads, extra):
    rng = np.random.default_rng(m * heads + extra)
    width = heads * 128
    buf = from_bits(random_bf16(rng, (m, width + extra), 1.5))
    before = buf.clone()
    w = oracle.f32_to_bf16_bits((1.0 + 0.1 * rng.standard_normal(128)).astype(np.float32))
    ang = rng.uniform(-20, 20, (m, 64))
    cos, sin = torch.tensor(np.cos(ang), dtype=torch.float32), torch.tensor(np.sin(ang), dtype=torch.float32)
    qk_rmsnorm_rope_(buf[:, :width], from_bits(w), cos, sin)
    torch.cuda.synchronize()
    ref = oracle.round_bf16(ob.qk_rmsnorm_rope(f32(before[:, :width]), oracle.bf16_bits_to_f32(w),
                                               np.float32(np.cos(ang)), np.float32(np.sin(ang))))
    g = f32(buf[:, :width])
    assert np.all(np.abs(g - ref) <= 2.0 ** -7 * np.abs(ref) + 2e-3)
    assert np.mean(np.abs(g - ref) <= 2.0 ** -8 * np.abs(ref) + 1e-6) > 0.98
    if extra:  # columns past the heads are untouched
        assert torch.equal(buf[:, width:], before[:, width:])


def _block_pair(rng, dim: int, heads: int, gs: int = 64):
    lin_o, lin_t = {}, {}
    for name, (fo, fi) in ob.BLOCK_LINEARS.items():
        w = random_weights(rng, fo * dim, fi * dim, gs)
        lin_o[name] = w
        wt, st, bt, bias = weights_to_torch(w)
        lin_t[name] = QuantizedLinear(wt, st, bt, bias, group_size=gs)
    norms_bits = {n: oracle.f32_to_bf16_bits((1.0 + 0.1 * rng.standard_normal(128)).astype(np.float32))
                  for n in ob.NORMS}
    ow = ob.BlockWeights(lin_o, {n: oracle.bf16_bits_to_f32(b) for n, b in norms_bits.items()}, heads)
    tb = QwenTransformerBlock(lin_t, {n: from_bits(b) for n, b in norms_bits.items()}, heads=heads)
    return ow, tb


@pytest.mark.parametrize("dim,heads,img_hw,txt", [(256, 2, (8, 12), 32), (768, 6, (10, 20), 40)])
def test_block_vs_oracle(dim, heads, img_hw, txt):
    rng = np.random.default_rng(dim + txt)
    ow, tb = _block_pair(rng, dim, heads)
    s_img = img_hw[0] * img_hw[1]
    hidden = random_bf16(rng, (s_img, dim))
    enc = random_bf16(rng, (txt, dim))
    temb = random_bf16(rng, (dim,))
    ia, ta = qwen_rope_angles([img_hw], txt)
    rope = rope_tables(ia, ta, "cuda")
    t_out, i_out = tb(from_bits(hidden)[None], from_bits(enc)[None], from_bits(temb)[None], rope)
    torch.cuda.synchronize()
    rf = [f32(r) for r in rope]
    t_ref, i_ref = ob.block_forward(ow, oracle.bf16_bits_to_f32(hidden), oracle.bf16_bits_to_f32(enc),
                                    oracle.bf16_bits_to_f32(temb), *rf)
    assert_close(f32(i_out[0]), i_ref, what=f"block image stream d{dim}")
    assert_close(f32(t_out[0]), t_ref, what=f"block text stream d{dim}")


def _block_pair_gpu(seed: int, dim: int, heads: int, gs: int = 64):
    """A random block quantised on the GPU (torch quantiser, bit-identical to
    the oracle's) and the oracle's view of the same weights."""

    from qwen_image_shardedit_mlx_b200.quantize import quantize_affine_q6

    from helpers import to_bits

    g = torch.Generator(device="cuda").manual_seed(seed)
    lin_o, lin_t = {}, {}
    for name, (fo, fi) in ob.BLOCK_LINEARS.items():
        w = torch.randn((fo * dim, fi * dim), generator=g, device="cuda") * 0.02
        q, s, b = quantize_affine_q6(w, gs)
        bias = (torch.randn((fo * dim,), generator=g, device="cuda") * 0.01).to(torch.bfloat16)
        lin_t[name] = QuantizedLinear(q, s, b, bias, group_size=gs)
        lin_o[name] = oracle.Q6Weights(q.view(torch.int32).cpu().numpy().view(np.uint32), to_bits(s), to_bits(b),
                                       to_bits(bias), gs)
    norms_t = {n: (1.0 + 0.1 * torch.randn((128,), generator=g, device="cuda")).to(torch.bfloat16) for n in ob.NORMS}
    ow = ob.BlockWeights(lin_o, {n: f32(v) for n, v in norms_t.items()}, heads)
    return ow, QwenTransformerBlock(lin_t, norms_t, heads=heads)


def test_full_size_block_vs_oracle_on_sampled_rows():
    """The Qwen-Image block at its real shape (3072 wide, 24 heads, 3456 image
    + 256 text tokens), checked on 16 sampled image rows and 8 text rows (keys
    and values always come from every row).

    * Stage by stage: each stage of the GPU block, fed the GPU's own input to
      that stage, matches the oracle's stage within the matmul bar
      (max 2e-2 of the largest value, mean 1e-3 of the rms).
    * End to end: the whole chain (ten bf16 roundings, the library attention)
      against the oracle run from the block inputs.  A one-unit bf16 rounding
      flip early in the chain moves later stages by about a unit too, so the
      mean bar of the chain is 2e-3 of the rms; the max bar stays 2e-2.
    """

    from qwen_image_shardedit_mlx_b200.block import (
        ModulationVectors,
        add_layernorm_modulate,
        batched_joint_attention,
        joint_rope,
        project_qkv_joint,
        rope_qk_joint,
        segments,
    )

    ow, tb = _block_pair_gpu(3072, 3072, 24)
    rng = np.random.default_rng(3712)
    s_img, s_txt, d = 3456, 256, 3072
    seq = s_img + s_txt
    hidden = random_bf16(rng, (s_img, d))
    enc = random_bf16(rng, (s_txt, d))
    temb = random_bf16(rng, (d,))
    ia, ta = qwen_rope_angles([(36, 48), (36, 48)], s_txt)
    rope = rope_tables(ia, ta, "cuda")
    rf = [f32(r) for r in rope]
    t_out, i_out = tb(from_bits(hidden)[None], from_bits(enc)[None], from_bits(temb)[None], rope)
    ir = np.unique(np.concatenate([[0, s_img - 1], rng.choice(s_img, 14, replace=False)]))
    tr = np.unique(np.concatenate([[0, s_txt - 1], rng.choice(s_txt, 6, replace=False)]))
    jr = np.concatenate([tr, s_txt + ir])  # sampled joint rows
    hf, ef, tf = (oracle.bf16_bits_to_f32(a) for a in (hidden, enc, temb))

    # ---- stage by stage, every stage fed the GPU's own input
    x = torch.cat([from_bits(enc), from_bits(hidden)]).contiguous()
    xf = np.concatenate([ef, hf])
    both = tb.modulation_joint(from_bits(temb)[None])  # one GEMV over [txt_mod; img_mod]
    mod_img, mod_txt = both[:, 1], both[:, 0]
    t = oracle.round_bf16(ob.silu(tf).reshape(1, d))
    assert_close(f32(mod_img[0]).reshape(6 * d), ob._lin(ow, "img_mod_linear", t)[0], what="img modulation")
    mi, mt = f32(mod_img[0]), f32(mod_txt[0])
    vec = ModulationVectors(both)  # strided views: vectors 6 D apart
    z = add_layernorm_modulate(x, vec.shift1, vec.scale1, seq_len=seq, text_len=s_txt)
    mod_of = lambda j, k: mt[k] if j < s_txt else mi[k]  # noqa: E731
    ref = np.stack([ob.layernorm_modulate(xf[j], mod_of(j, 0), mod_of(j, 1)) for j in jr])
    assert_close(f32(z)[jr], ref, what="adaLN modulate 1")
    qkv = torch.empty((seq, 3 * d), dtype=torch.bfloat16, device="cuda")
    project_qkv_joint(tb, z, qkv, 1, seq, s_txt)
    zf = f32(z)
    for names, rows, off in ((("attn.add_q_proj", "attn.add_k_proj", "attn.add_v_proj"), tr, 0),
                             (("attn.to_q", "attn.to_k", "attn.to_v"), ir, s_txt)):
        for j, name in enumerate(names):
            ref = ob._lin(ow, name, zf[off + rows], launch_rows=seq)
            assert_close(f32(qkv[torch.as_tensor(off + rows, device="cuda"), j * d:(j + 1) * d]), ref, what=name)
    qkv_f = f32(qkv)
    rope_qk_joint(tb, qkv, d, joint_rope(rope), seq, s_txt)
    cos_j, sin_j = np.concatenate([rf[2], rf[0]]), np.concatenate([rf[3], rf[1]])
    for j, (nt, ni) in enumerate((("attn.norm_added_q", "attn.norm_q"), ("attn.norm_added_k", "attn.norm_k"))):
        for rows, off, norm in ((tr, 0, nt), (ir, s_txt, ni)):
            ref = ob.qk_rmsnorm_rope(qkv_f[off + rows, j * d:(j + 1) * d], ow.norms[norm], cos_j[off + rows],
                                     sin_j[off + rows])
            assert_close(f32(qkv[torch.as_tensor(off + rows, device="cuda"), j * d:(j + 1) * d]), ref, what=norm)
    qkv_f = f32(qkv)
    att = batched_joint_attention(qkv, d, 1, seq, 24, s_txt)
    ref = ob.attention(qkv_f[jr, :d], qkv_f[:, d:2 * d], qkv_f[:, 2 * d:], 24).astype(np.float32)
    assert_close(f32(att)[jr], ref, what="joint attention")
    h = torch.empty_like(x)
    att_f = f32(att)
    for b, stream, r in segments(1, seq, s_txt):
        name = "attn.to_add_out" if stream == 0 else "attn.attn_to_out.0"
        tb._linear(name, att[r], residual=x[r], gate=vec.gate1(b, stream), out=h[r])
    for rows, off, name, m in ((tr, 0, "attn.to_add_out", mt), (ir, s_txt, "attn.attn_to_out.0", mi)):
        ref = ob._lin(ow, name, att_f[off + rows], residual=xf[off + rows], gate=m[2], launch_rows=seq)
        assert_close(f32(h)[off + rows], ref, what=name)
    z2 = add_layernorm_modulate(h, vec.shift2, vec.scale2, seq_len=seq, text_len=s_txt)
    hf2 = f32(h)
    ref = np.stack([ob.layernorm_modulate(hf2[j], mod_of(j, 3), mod_of(j, 4)) for j in jr])
    assert_close(f32(z2)[jr], ref, what="adaLN modulate 2")
    y = torch.empty_like(x)
    for b, stream, r in segments(1, seq, s_txt):
        tb._mlp("txt_ff" if stream == 0 else "img_ff", z2[r], h[r], vec.gate2(b, stream), y[r])
    torch.cuda.synchronize()
    z2f = f32(z2)
    for rows, off, pre, m in ((tr, 0, "txt_ff", mt), (ir, s_txt, "img_ff", mi)):
        mid = ob._lin(ow, f"{pre}.mlp_in", z2f[off + rows], apply_gelu=True, launch_rows=seq)
        ref = ob._lin(ow, f"{pre}.mlp_out", mid, residual=hf2[off + rows], gate=m[5], launch_rows=seq)
        assert_close(f32(y)[off + rows], ref, what=f"{pre} (fused MLP)")
    # the stage-by-stage run is the block's forward
    assert torch.equal(y[s_txt:], i_out[0]) and torch.equal(y[:s_txt], t_out[0])

    # ---- end to end from the block inputs
    t_ref, i_ref = ob.block_forward_rows(ow, hf, ef, tf, *rf, img_rows=ir, txt_rows=tr)
    assert_close(f32(i_out[0])[ir], i_ref, mean_abs_rel=2e-3, what="full-size block chain, image rows")
    assert_close(f32(t_out[0])[tr], t_ref, mean_abs_rel=2e-3, what="full-size block chain, text rows")


def test_block_with_padded_text_mask_vs_oracle():
    """A padded prompt: the last text tokens are padding (mask 0), so no query
    may attend to them as keys; image and text outputs follow the masked
    oracle and differ from the unmasked block."""

    rng = np.random.default_rng(41)
    dim, heads, img_hw, txt = 768, 6, (10, 20), 40
    ow, tb = _block_pair(rng, dim, heads)
    s_img = img_hw[0] * img_hw[1]
    hidden = random_bf16(rng, (s_img, dim))
    enc = random_bf16(rng, (txt, dim))
    temb = random_bf16(rng, (dim,))
    mask = np.ones(txt, dtype=np.float32)
    mask[27:] = 0.0
    ia, ta = qwen_rope_angles([img_hw], txt)
    rope = rope_tables(ia, ta, "cuda")
    args = (from_bits(hidden)[None], from_bits(enc)[None], from_bits(temb)[None], rope)
    t_m, i_m = tb(*args, encoder_mask=torch.from_numpy(mask)[None].cuda())
    t_u, i_u = tb(*args)
    torch.cuda.synchronize()
    rf = [f32(r) for r in rope]
    t_ref, i_ref = ob.block_forward(ow, oracle.bf16_bits_to_f32(hidden), oracle.bf16_bits_to_f32(enc),
                                    oracle.bf16_bits_to_f32(temb), *rf, text_mask=mask)
    assert_close(f32(i_m[0]), i_ref, what="masked block image stream")
    assert_close(f32(t_m[0]), t_ref, what="masked block text stream")
    assert float((i_m.float() - i_u.float()).abs().max()) > 1e-2  # the mask changes the image stream
    # an all-ones mask is the unmasked block
    t_1, i_1 = tb(*args, encoder_mask=torch.ones((1, txt), device="cuda"))
    torch.cuda.synchronize()
    assert_close(f32(i_1[0]), f32(i_u[0]), what="all-ones mask", bf16_output=False)


def test_full_size_block_runs():
    g = torch.Generator(device="cuda").manual_seed(5)
    blk = QwenTransformerBlock.random(generator=g)
    hidden = torch.randn((1, 3456, 3072), generator=g, device="cuda").to(torch.bfloat16)
    enc = torch.randn((1, 256, 3072), generator=g, device="cuda").to(torch.bfloat16)
    temb = torch.randn((1, 3072), generator=g, device="cuda").to(torch.bfloat16)
    ia, ta = qwen_rope_angles([(36, 48), (36, 48)], 256)
    t_out, i_out = blk(hidden, enc, temb, rope_tables(ia, ta, "cuda"))
    torch.cuda.synchronize()
    assert t_out.shape == (1, 256, 3072) and i_out.shape == (1, 3456, 3072)
    assert bool(torch.isfinite(t_out).all()) and bool(torch.isfinite(i_out).all())


def test_tensor_parallel_block_world1_matches_the_block():
    """One rank holds every head, column and row: the sequence-parallel block
    (residual added after the row-parallel GEMM instead of in its epilogue)
    agrees with the single-GPU block to bf16 rounding."""

    from qwen_image_shardedit_mlx_b200.block import TensorParallelQwenBlock

    rng = np.random.default_rng(77)
    _, tb = _block_pair(rng, 512, 4)
    tp = TensorParallelQwenBlock(tb, 1, 0)
    hidden = from_bits(random_bf16(rng, (2, 96, 512)))
    enc = from_bits(random_bf16(rng, (2, 24, 512)))
    temb = from_bits(random_bf16(rng, (2, 512)))
    ia, ta = qwen_rope_angles([(8, 12)], 24)
    rope = rope_tables(ia, ta, "cuda")
    a = tb(hidden, enc, temb, rope)
    b = tp(hidden, enc, temb, rope)
    torch.cuda.synchronize()
    for x, y in zip(a, b):
        assert_close(f32(y), f32(x), bf16_output=False, what="tp world 1")


def test_context_parallel_block_world1_matches_the_block():
    """One rank holds every row: the context-parallel block (per-sample adaLN
    and QK-norm launches placed by row0, keys and values copied out for the
    attention) agrees with the single-GPU block, batch 2 with a padded text
    mask."""

    from qwen_image_shardedit_mlx_b200.block import ContextParallelQwenBlock

    rng = np.random.default_rng(78)
    _, tb = _block_pair(rng, 512, 4)
    cp = ContextParallelQwenBlock(tb, 1, 0)
    hidden = from_bits(random_bf16(rng, (2, 96, 512)))
    enc = from_bits(random_bf16(rng, (2, 24, 512)))
    temb = from_bits(random_bf16(rng, (2, 512)))
    mask = torch.ones((2, 24), device="cuda")
    mask[1, 20:] = 0
    ia, ta = qwen_rope_angles([(8, 12)], 24)
    rope = rope_tables(ia, ta, "cuda")
    a = tb(hidden, enc, temb, rope, encoder_mask=mask)
    b = cp(hidden, enc, temb, rope, encoder_mask=mask)
    torch.cuda.synchronize()
    for x, y in zip(a, b):
        assert_close(f32(y), f32(x), bf16_output=False, what="cp world 1")


def test_batched_block_vs_oracle_per_sample():
    """Two samples (CFG cond / uncond) through one block call: the joint rows
    of both go through each batched kernel, and every sample matches the
    oracle block run on it alone (its own timestep embedding)."""

    rng = np.random.default_rng(2)
    dim, heads, img_hw, txt = 512, 4, (8, 12), 24
    ow, tb = _block_pair(rng, dim, heads)
    s_img = img_hw[0] * img_hw[1]
    hidden = random_bf16(rng, (2, s_img, dim))
    enc = random_bf16(rng, (2, txt, dim))
    temb = random_bf16(rng, (2, dim))
    ia, ta = qwen_rope_angles([img_hw], txt)
    rope = rope_tables(ia, ta, "cuda")
    t_out, i_out = tb(from_bits(hidden), from_bits(enc), from_bits(temb), rope)
    torch.cuda.synchronize()
    rf = [f32(r) for r in rope]
    for b in range(2):
        t_ref, i_ref = ob.block_forward(ow, oracle.bf16_bits_to_f32(hidden[b]), oracle.bf16_bits_to_f32(enc[b]),
                                        oracle.bf16_bits_to_f32(temb[b]), *rf)
        assert_close(f32(i_out[b]), i_ref, what=f"batched block image stream, sample {b}")
        assert_close(f32(t_out[b]), t_ref, what=f"batched block text stream, sample {b}")


def test_peer_comm_block_world1_matches_nccl_layout():
    """The peer-memory form of the sequence-parallel block (fused reduce +
    residual + modulate + gather kernels, barriers) on one rank against the
    NCCL form: the same rows through the same GEMMs, the residual sums formed
    by two different kernels (fp32, one bf16 rounding each)."""

    from qwen_image_shardedit_mlx_b200.block import TensorParallelQwenBlock

    rng = np.random.default_rng(78)
    _, tb = _block_pair(rng, 512, 4)
    hidden = from_bits(random_bf16(rng, (2, 96, 512)))
    enc = from_bits(random_bf16(rng, (2, 24, 512)))
    temb = from_bits(random_bf16(rng, (2, 512)))
    ia, ta = qwen_rope_angles([(8, 12)], 24)
    rope = rope_tables(ia, ta, "cuda")
    a = TensorParallelQwenBlock(tb, 1, 0, comm="nccl")(hidden, enc, temb, rope)
    b = TensorParallelQwenBlock(tb, 1, 0, comm="peer")(hidden, enc, temb, rope)
    torch.cuda.synchronize()
    for x, y in zip(a, b):
        assert_close(f32(y), f32(x), bf16_output=False, what="peer vs nccl layout, world 1")


def test_peer_barrier_gives_up_on_a_missing_peer():
    """The barrier's bounded wait: a two-rank signal table whose second
    rank never arrives (both entries are this GPU's memory, and nothing writes
    the slot this rank waits on) ends after the 2 ms limit with
    Q6_SITE_PEER_BARRIER in the device error word instead of hanging."""

    import ctypes

    from qwen_image_shardedit_mlx_b200 import ops

    sig = torch.zeros(16, dtype=torch.int32, device="cuda")
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    table = (ctypes.c_void_p * 2)(sig.data_ptr(), sig[8:].data_ptr())
    ops.clear_device_error()
    try:
        st = _lib.lib().q6_sp_barrier(table, epoch.data_ptr(), 2, 0, 2_000_000, ops._stream(sig.device))
        assert st == _lib.Q6_OK
        assert ops.device_error() == _lib.Q6_SITE_PEER_BARRIER
    finally:
        ops.clear_device_error()
    assert ops.device_error() == 0
    assert int(epoch.item()) == 1  # the barrier advanced its epoch counter


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tensor_parallel_block_over_nccl_world2():
    import os
    import socket
    import subprocess
    import sys
    from pathlib import Path

    with socket.socket() as sck:
        sck.bind(("127.0.0.1", 0))
        port = sck.getsockname()[1]
    script = Path(__file__).with_name("tp_block_check.py")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), str(script)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert r.stdout.count("OK") == 2


def test_two_stream_block_matches_one_stream():
    """The text- and image-stream launches on two CUDA streams give the same
    bits as both in order on one stream (batch 2, so each stage forks four
    GEMMs over two streams), eagerly and replayed from a CUDA graph."""

    from qwen_image_shardedit_mlx_b200.block import QwenTransformerBlock, joint_rope

    g = torch.Generator(device="cuda").manual_seed(44)
    blk = QwenTransformerBlock.random(512, 4, generator=g)
    x = torch.randn((2 * (96 + 24), 512), generator=g, device="cuda").to(torch.bfloat16)
    temb = torch.randn((2, 512), generator=g, device="cuda").to(torch.bfloat16)
    ia, ta = qwen_rope_angles([(8, 12)], 24)
    rope = joint_rope(rope_tables(ia, ta, "cuda"))
    blk.overlap_streams = False
    ref = blk.forward_joint(x, temb, rope, 2, 24)
    blk.overlap_streams = True
    got = blk.forward_joint(x, temb, rope, 2, 24)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    out = torch.empty_like(x)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        blk.forward_joint(x, temb, rope, 2, 24, out=out)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        blk.forward_joint(x, temb, rope, 2, 24, out=out)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    del graph
