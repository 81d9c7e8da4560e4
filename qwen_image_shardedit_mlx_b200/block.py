"""One Qwen-Image MMDiT dual-stream block on the q6 kernels.

The block the reference profiles stage by stage
(benchmarks/profile_qwen_block.py:163-301; mflux ``QwenTransformerBlock``):

=====================================  =========================================================
reference stage                         here
=====================================  =========================================================
img/txt_mod_linear(silu(temb))         ``q6_linear`` on the few-row streaming GEMV
_modulate(norm1(x), mod1)              ``q6_layernorm_modulate_bf16`` (one fused kernel)
to_q/k/v, add_q/k/v_proj               ``q6_linear`` writing straight into the joint
                                        [text; image] q / k / v buffers
norm_q/k, norm_added_q/k + rope        ``q6_qk_rmsnorm_rope_bf16`` in place on those buffers
joint attention (_compute_attention)   torch scaled_dot_product_attention (library kernel)
attn_to_out[0] / to_add_out + gate1    ``q6_linear`` with the residual and gate in its epilogue
_modulate(norm2(x), mod2)              ``q6_layernorm_modulate_bf16``
img_ff / txt_ff + gate2 residual       ``q6_mlp`` with the residual and gate in fc2's epilogue
=====================================  =========================================================

Tensor names follow the reference's checkpoint layout (``img_mod_linear``,
``attn.to_q``, ``attn.attn_to_out.0``, ``img_ff.mlp_in``, ``attn.norm_q``
...), so ``from_block_weights`` builds a block from a loaded checkpoint block.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from qwen_image_shardedit_mlx_b200 import _lib, ops
from qwen_image_shardedit_mlx_b200.q6_metal_mlp import QuantizedLinear, QwenFeedForward
from qwen_image_shardedit_mlx_b200.quantize import quantize_affine_q6

HEAD_DIM = 128
LINEAR_SHAPES = {
    # name: (out_features, in_features) as multiples of the hidden size D (FF hidden = 4 D)
    "img_mod_linear": (6, 1), "txt_mod_linear": (6, 1),
    "attn.to_q": (1, 1), "attn.to_k": (1, 1), "attn.to_v": (1, 1),
    "attn.add_q_proj": (1, 1), "attn.add_k_proj": (1, 1), "attn.add_v_proj": (1, 1),
    "attn.attn_to_out.0": (1, 1), "attn.to_add_out": (1, 1),
    "img_ff.mlp_in": (4, 1), "img_ff.mlp_out": (1, 4),
    "txt_ff.mlp_in": (4, 1), "txt_ff.mlp_out": (1, 4),
}
NORM_NAMES = ("attn.norm_q", "attn.norm_k", "attn.norm_added_q", "attn.norm_added_k")


def layernorm_modulate(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, *, eps: float = 1e-6,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """``LayerNorm(x) * (1 + scale) + shift`` over the last axis (bf16 in and out)."""

    d = x.shape[-1]
    xb = x.reshape(-1, d)
    if xb.dtype != torch.bfloat16 or not xb.is_contiguous():
        xb = xb.to(torch.bfloat16).contiguous()
    sh = shift.reshape(d).to(torch.bfloat16).contiguous()
    sc = scale.reshape(d).to(torch.bfloat16).contiguous()
    y = out if out is not None else torch.empty_like(xb)
    st = _lib.lib().q6_layernorm_modulate_bf16(xb.data_ptr(), sh.data_ptr(), sc.data_ptr(), y.data_ptr(),
                                               xb.shape[0], d, float(eps), ops._stream(xb.device))
    _lib.check(st, "q6_layernorm_modulate_bf16")
    return y.reshape(x.shape)


def qk_rmsnorm_rope_(qk: torch.Tensor, weight: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, *,
                     eps: float = 1e-6) -> torch.Tensor:
    """In place on rows [M, H * 128] (row stride may exceed H * 128): per head
    RMSNorm with ``weight`` then the interleaved-pair rotation by cos / sin [M, 64]."""

    if qk.dtype != torch.bfloat16 or qk.dim() != 2 or qk.stride(1) != 1:
        raise ValueError("qk must be a 2-D bf16 view with unit column stride")
    m, width = qk.shape
    if width % HEAD_DIM:
        raise ValueError(f"row width {width} is not a multiple of {HEAD_DIM}")
    c = cos.to(device=qk.device, dtype=torch.float32).contiguous()
    s = sin.to(device=qk.device, dtype=torch.float32).contiguous()
    if c.shape != (m, HEAD_DIM // 2) or s.shape != (m, HEAD_DIM // 2):
        raise ValueError(f"cos/sin must be ({m}, {HEAD_DIM // 2})")
    w = weight.to(device=qk.device, dtype=torch.bfloat16).contiguous()
    st = _lib.lib().q6_qk_rmsnorm_rope_bf16(qk.data_ptr(), qk.stride(0), m, width // HEAD_DIM, HEAD_DIM,
                                            w.data_ptr(), c.data_ptr(), s.data_ptr(), float(eps),
                                            ops._stream(qk.device))
    _lib.check(st, "q6_qk_rmsnorm_rope_bf16")
    return qk


def qwen_rope_angles(img_shapes: list[tuple[int, int]], txt_len: int, *, theta: float = 10000.0,
                     axes: tuple[int, int, int] = (16, 56, 56), device: torch.device | str = "cpu"):
    """Rotary angles (radians, float64) [S_img, 64] and [S_txt, 64].

    Three axes (frame, height, width) of 16 / 56 / 56 dimensions with base
    ``theta``: image ``f`` of (h, w) patches takes frame position f and
    centred grid positions; text positions continue after the largest image
    position on all three axes (the published Qwen-Image rotary layout).
    """

    def freqs(dim: int) -> torch.Tensor:
        return 1.0 / theta ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim)

    fr, fh, fw = (freqs(a) for a in axes)
    rows, max_pos = [], 0
    for f, (h, w) in enumerate(img_shapes):
        hp = torch.arange(h, dtype=torch.float64) - h // 2
        wp = torch.arange(w, dtype=torch.float64) - w // 2
        hh, ww = torch.meshgrid(hp, wp, indexing="ij")
        rows.append(torch.cat([(f * fr).expand(h * w, -1), hh.reshape(-1, 1) * fh, ww.reshape(-1, 1) * fw], dim=1))
        max_pos = max(max_pos, h // 2, w // 2)
    img = torch.cat(rows, dim=0)
    tp = (max_pos + torch.arange(txt_len, dtype=torch.float64)).reshape(-1, 1)
    txt = torch.cat([tp * fr, tp * fh, tp * fw], dim=1)
    return img.to(device), txt.to(device)


def rope_tables(img_angles: torch.Tensor, txt_angles: torch.Tensor, device: torch.device | str):
    """(img_cos, img_sin, txt_cos, txt_sin) fp32 on ``device``."""

    return tuple(t.to(device=device, dtype=torch.float32).contiguous()
                 for t in (img_angles.cos(), img_angles.sin(), txt_angles.cos(), txt_angles.sin()))


class QwenTransformerBlock(torch.nn.Module):
    """Dual-stream MMDiT block: q6 linears by reference name, bf16 norm weights."""

    def __init__(self, linears: dict[str, QuantizedLinear], norms: dict[str, torch.Tensor], *,
                 heads: int, eps: float = 1e-6) -> None:
        super().__init__()
        missing = [n for n in LINEAR_SHAPES if n not in linears] + [n for n in NORM_NAMES if n not in norms]
        if missing:
            raise ValueError(f"block is missing {missing}")
        self.linears = linears
        self.norms = {k: v.to(torch.bfloat16).contiguous() for k, v in norms.items()}
        self.heads = int(heads)
        self.dim = linears["attn.to_q"].out_features
        if self.dim != self.heads * HEAD_DIM:
            raise ValueError(f"hidden size {self.dim} != heads {heads} x {HEAD_DIM}")
        self.eps = float(eps)
        self.img_ff = QwenFeedForward(linears["img_ff.mlp_in"], linears["img_ff.mlp_out"])
        self.txt_ff = QwenFeedForward(linears["txt_ff.mlp_in"], linears["txt_ff.mlp_out"])
        self._ws: torch.Tensor | None = None

    @classmethod
    def random(cls, dim: int = 3072, heads: int = 24, *, group_size: int = 64, std: float = 0.02,
               bias_std: float = 0.01, generator: torch.Generator | None = None,
               device: torch.device | str = "cuda") -> "QwenTransformerBlock":
        linears = {}
        for name, (fo, fi) in LINEAR_SHAPES.items():
            w = torch.randn((fo * dim, fi * dim), generator=generator, device=device) * std
            q, s, b = quantize_affine_q6(w, group_size)
            bias = (torch.randn((fo * dim,), generator=generator, device=device) * bias_std).to(torch.bfloat16)
            linears[name] = QuantizedLinear(q, s, b, bias, group_size=group_size)
        norms = {n: (1.0 + 0.1 * torch.randn((HEAD_DIM,), generator=generator, device=device)).to(torch.bfloat16)
                 for n in NORM_NAMES}
        return cls(linears, norms, heads=heads)

    @classmethod
    def from_block_weights(cls, block, *, heads: int | None = None) -> "QwenTransformerBlock":
        """From a loaded checkpoint block (``qwen_block_loader.QwenBlockWeights``)."""

        norms = {n: block.tensors[f"{n}.weight"] for n in NORM_NAMES}
        dim = block.linears["attn.to_q"].out_features
        return cls(dict(block.linears), norms, heads=heads or dim // HEAD_DIM)

    def _workspace(self, m: int, device: torch.device) -> torch.Tensor:
        need = int(ops.mlp_workspace_bytes(m, 4 * self.dim, self.dim))
        if self._ws is None or self._ws.numel() < need or self._ws.device != device:
            self._ws = torch.empty(need, dtype=torch.uint8, device=device)
        return self._ws

    def _mlp(self, ff: QwenFeedForward, x: torch.Tensor, residual: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
        if ff.mlp_in.lora is not None or ff.mlp_out.lora is not None:
            mid = ops.q6_linear(x, ff.mlp_in.weight, ff.mlp_in.scales, ff.mlp_in.biases, ff.mlp_in.bias,
                                group_size=ff.mlp_in.group_size, apply_gelu=True, lora=ff.mlp_in.lora)
            lo = ff.mlp_out
            return ops.q6_linear(mid, lo.weight, lo.scales, lo.biases, lo.bias, group_size=lo.group_size,
                                 residual=residual, gate=gate, lora=lo.lora)
        w1 = (ff.mlp_in.weight, ff.mlp_in.scales, ff.mlp_in.biases, ff.mlp_in.bias)
        w2 = (ff.mlp_out.weight, ff.mlp_out.scales, ff.mlp_out.biases, ff.mlp_out.bias)
        return ops.q6_mlp(x, w1, w2, group_size=ff.mlp_in.group_size, residual=residual, gate=gate,
                          workspace=self._workspace(x.shape[0], x.device))

    def _linear(self, name: str, x: torch.Tensor, **kw) -> torch.Tensor:
        lin = self.linears[name]
        return ops.q6_linear(x, lin.weight, lin.scales, lin.biases, lin.bias, group_size=lin.group_size,
                             lora=lin.lora, **kw)

    def forward_sample(self, hidden: torch.Tensor, encoder: torch.Tensor, mod_img: torch.Tensor,
                       mod_txt: torch.Tensor, rope: tuple[torch.Tensor, ...],
                       text_mask: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """One sample: hidden [S_img, D], encoder [S_txt, D], modulation
        vectors [6, D] per stream, optional text mask [S_txt] (1 = token,
        0 = padding); returns (text out, image out)."""

        img_cos, img_sin, txt_cos, txt_sin = rope
        s_img, s_txt, d = hidden.shape[0], encoder.shape[0], self.dim
        ish1, isc1, ig1, ish2, isc2, ig2 = mod_img
        tsh1, tsc1, tg1, tsh2, tsc2, tg2 = mod_txt
        img_in = layernorm_modulate(hidden, ish1, isc1, eps=self.eps)
        txt_in = layernorm_modulate(encoder, tsh1, tsc1, eps=self.eps)
        # joint [text; image] projections, written in place
        s = s_txt + s_img
        q = torch.empty((s, d), dtype=torch.bfloat16, device=hidden.device)
        k = torch.empty_like(q)
        v = torch.empty_like(q)
        project_qkv(self, txt_in, img_in, q, k, v)
        qk_rmsnorm_rope_(q[:s_txt], self.norms["attn.norm_added_q"], txt_cos, txt_sin, eps=self.eps)
        qk_rmsnorm_rope_(q[s_txt:], self.norms["attn.norm_q"], img_cos, img_sin, eps=self.eps)
        qk_rmsnorm_rope_(k[:s_txt], self.norms["attn.norm_added_k"], txt_cos, txt_sin, eps=self.eps)
        qk_rmsnorm_rope_(k[s_txt:], self.norms["attn.norm_k"], img_cos, img_sin, eps=self.eps)
        joint = joint_attention(q, k, v, self.heads, s_txt, text_mask)
        img_h = self._linear("attn.attn_to_out.0", joint[s_txt:], residual=hidden, gate=ig1)
        txt_h = self._linear("attn.to_add_out", joint[:s_txt], residual=encoder, gate=tg1)
        img_ff_in = layernorm_modulate(img_h, ish2, isc2, eps=self.eps)
        txt_ff_in = layernorm_modulate(txt_h, tsh2, tsc2, eps=self.eps)
        img_out = self._mlp(self.img_ff, img_ff_in, img_h, ig2)
        txt_out = self._mlp(self.txt_ff, txt_ff_in, txt_h, tg2)
        return txt_out, img_out

    def modulation(self, temb: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """(img, txt) modulation vectors [B, 6, D] from the timestep embedding [B, D]."""

        t = F.silu(temb.to(torch.bfloat16))
        b = t.shape[0]
        return (self._linear("img_mod_linear", t).reshape(b, 6, self.dim),
                self._linear("txt_mod_linear", t).reshape(b, 6, self.dim))

    def forward(self, hidden: torch.Tensor, encoder: torch.Tensor, temb: torch.Tensor,
                rope: tuple[torch.Tensor, ...],
                encoder_mask: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """hidden [B, S_img, D], encoder [B, S_txt, D], temb [B, D] (bf16);
        ``rope`` = (img_cos, img_sin, txt_cos, txt_sin) fp32 [S, 64];
        ``encoder_mask`` [B, S_txt] (1 = text token, 0 = padding; None = no
        padding).  Returns (encoder_out, hidden_out) like the reference block."""

        mod_img, mod_txt = self.modulation(temb)
        outs = [self.forward_sample(hidden[b], encoder[b], mod_img[b], mod_txt[b], rope,
                                    None if encoder_mask is None else encoder_mask[b])
                for b in range(hidden.shape[0])]
        return torch.stack([o[0] for o in outs]), torch.stack([o[1] for o in outs])


def joint_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, s_txt: int,
                    text_mask: torch.Tensor | None = None) -> torch.Tensor:
    """Joint [text; image] attention of one sample over rows [S, heads * 128]
    (torch scaled_dot_product_attention).  ``text_mask`` [S_txt] (1 = token,
    0 = padding) removes padded text tokens as keys, every image token stays
    a key: the joint mask the reference builds from
    ``encoder_hidden_states_mask`` (benchmarks/profile_qwen_block.py:228-248).
    Without a mask the library's unmasked flash kernel runs."""

    s = q.shape[0]
    shape = (1, s, heads, HEAD_DIM)
    mask = None
    if text_mask is not None:
        keep = torch.ones(s, dtype=torch.bool, device=q.device)
        keep[:s_txt] = text_mask.reshape(-1).to(q.device) > 0.5
        mask = keep.view(1, 1, 1, s)
    att = F.scaled_dot_product_attention(q.view(shape).transpose(1, 2), k.view(shape).transpose(1, 2),
                                         v.view(shape).transpose(1, 2), attn_mask=mask,
                                         scale=1.0 / math.sqrt(HEAD_DIM))
    return att.transpose(1, 2).reshape(s, heads * HEAD_DIM)


_TXT_QKV = ("attn.add_q_proj", "attn.add_k_proj", "attn.add_v_proj")


def fused_rows(owner: torch.nn.Module, names: tuple[str, ...]) -> QuantizedLinear | None:
    """Row concatenation of q6 linears of ``owner.linears`` that read the same
    input (the text stream's q, k and v projections): one GEMM whose output
    columns are theirs side by side.  At a few hundred tokens the three
    3072-row GEMMs each fill a third of the GPU's tiles (and need split-K);
    their concatenation fills it alone.  The members' tensors are rebound to
    views of the concatenation, so no weight is held twice.  None when a
    member carries a LoRA delta or the members differ in input or group size."""

    lins = [owner.linears[n] for n in names]
    if any(lin.lora is not None for lin in lins):
        return None
    if len({(lin.in_features, lin.group_size, lin.weight.device) for lin in lins}) != 1:
        return None
    cache = owner.__dict__.setdefault("_fused_rows", {})
    hit = cache.get(names)
    if hit is not None and all(lin.weight.data_ptr() == ptr for lin, ptr in zip(lins, hit[0])):
        return hit[1]
    w = torch.cat([lin.weight for lin in lins])
    sc = torch.cat([lin.scales for lin in lins])
    bi = torch.cat([lin.biases for lin in lins])
    bias = torch.cat([lin.bias if lin.bias is not None else
                      torch.zeros(lin.out_features, dtype=torch.bfloat16, device=w.device) for lin in lins])
    fused = QuantizedLinear(w, sc, bi, bias, group_size=lins[0].group_size)
    off = 0
    for lin in lins:
        n = lin.out_features
        lin.weight, lin.scales, lin.biases = w[off:off + n], sc[off:off + n], bi[off:off + n]
        if lin.bias is not None:
            lin.bias = bias[off:off + n]
        off += n
    cache[names] = (tuple(lin.weight.data_ptr() for lin in lins), fused)
    return fused


def project_qkv(owner: torch.nn.Module, txt_in: torch.Tensor, img_in: torch.Tensor, q: torch.Tensor,
                k: torch.Tensor, v: torch.Tensor) -> None:
    """Joint [text; image] q, k, v projections written in place: the image
    rows by three GEMMs, the text rows by one GEMM of the concatenated text
    projections (``fused_rows``) copied into place."""

    s_txt = txt_in.shape[0]
    fused = fused_rows(owner, _TXT_QKV) if s_txt else None
    if fused is not None:
        t = ops.q6_linear(txt_in, fused.weight, fused.scales, fused.biases, fused.bias,
                          group_size=fused.group_size)
        width = q.shape[1]
        for j, buf in enumerate((q, k, v)):
            buf[:s_txt].copy_(t[:, j * width:(j + 1) * width])
    for buf, img_name, txt_name in ((q, "attn.to_q", "attn.add_q_proj"), (k, "attn.to_k", "attn.add_k_proj"),
                                    (v, "attn.to_v", "attn.add_v_proj")):
        if fused is None:
            owner._linear(txt_name, txt_in, out=buf[:s_txt])
        owner._linear(img_name, img_in, out=buf[s_txt:])


def block_flops(s_img: int, s_txt: int, dim: int) -> int:
    """FLOPs of one block forward (one sample): per token 8 D^2 for q, k, v
    and the output projection and 16 D^2 for the 4x feed-forward, 4 S^2 D for
    the joint attention (q k^T and p v), 24 D^2 for the two modulation linears."""

    s = s_img + s_txt
    return 24 * s * dim * dim + 4 * s * s * dim + 24 * dim * dim


class TensorParallelQwenBlock(torch.nn.Module):
    """The block split over the ranks of a process group (one rank per GPU).

    Heads and the feed-forward hidden columns are divided: q / k / v and
    mlp_in are column-parallel (each rank holds its heads' / columns' rows of
    codes, scales and biases), the output projections and mlp_out are
    row-parallel (each rank holds the matching K slice).  The modulation
    linears, the norms and the residual streams are replicated.  A
    row-parallel partial carries the residual and the output bias on rank 0
    only and the gate on every rank, so that the all-reduce sum of the
    partials is ``residual + gate * (x W^T + bias)`` exactly as the
    single-GPU epilogue computes it.  Two all-reduces per block, each over
    the joint [text; image] rows.
    """

    def __init__(self, full: QwenTransformerBlock, world: int, rank: int, group=None) -> None:
        super().__init__()
        from qwen_image_shardedit_mlx_b200.sharding import split_k, split_rows

        if full.heads % world:
            raise ValueError(f"{full.heads} heads do not split over {world} ranks")
        if any(lin.lora is not None for lin in full.linears.values()):
            raise ValueError("fold LoRA adapters before sharding the block")
        self.world, self.rank, self.group = int(world), int(rank), group
        self.dim, self.heads_local, self.eps = full.dim, full.heads // world, full.eps
        self.norms = full.norms

        def rows(name: str) -> QuantizedLinear:
            lin = full.linears[name]
            return QuantizedLinear(*split_rows(lin.weight, lin.scales, lin.biases, lin.bias, world, rank),
                                   group_size=lin.group_size)

        def cols(name: str) -> QuantizedLinear:
            lin = full.linears[name]
            w, s, b = split_k(lin.weight, lin.scales, lin.biases, lin.group_size, world, rank)
            return QuantizedLinear(w, s, b, lin.bias if rank == 0 else None, group_size=lin.group_size)

        self.linears = {"img_mod_linear": full.linears["img_mod_linear"],
                        "txt_mod_linear": full.linears["txt_mod_linear"]}
        for name in ("attn.to_q", "attn.to_k", "attn.to_v", "attn.add_q_proj", "attn.add_k_proj",
                     "attn.add_v_proj", "img_ff.mlp_in", "txt_ff.mlp_in"):
            self.linears[name] = rows(name)
        for name in ("attn.attn_to_out.0", "attn.to_add_out", "img_ff.mlp_out", "txt_ff.mlp_out"):
            self.linears[name] = cols(name)
        self._ws: torch.Tensor | None = None

    def _linear(self, name: str, x: torch.Tensor, **kw) -> torch.Tensor:
        lin = self.linears[name]
        return ops.q6_linear(x, lin.weight, lin.scales, lin.biases, lin.bias, group_size=lin.group_size, **kw)

    def _all_reduce(self, t: torch.Tensor) -> None:
        import torch.distributed as dist

        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def _mlp(self, prefix: str, x: torch.Tensor, residual: torch.Tensor | None, gate: torch.Tensor,
             out: torch.Tensor) -> None:
        l1, l2 = self.linears[f"{prefix}.mlp_in"], self.linears[f"{prefix}.mlp_out"]
        need = int(ops.mlp_workspace_bytes(x.shape[0], l1.out_features, l1.in_features))
        if self._ws is None or self._ws.numel() < need or self._ws.device != x.device:
            self._ws = torch.empty(need, dtype=torch.uint8, device=x.device)
        ops.q6_mlp(x, (l1.weight, l1.scales, l1.biases, l1.bias), (l2.weight, l2.scales, l2.biases, l2.bias),
                   group_size=l1.group_size, residual=residual, gate=gate, workspace=self._ws, out=out)

    def modulation(self, temb: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        t = F.silu(temb.to(torch.bfloat16))
        b = t.shape[0]
        return (self._linear("img_mod_linear", t).reshape(b, 6, self.dim),
                self._linear("txt_mod_linear", t).reshape(b, 6, self.dim))

    def forward_sample(self, hidden: torch.Tensor, encoder: torch.Tensor, mod_img: torch.Tensor,
                       mod_txt: torch.Tensor, rope: tuple[torch.Tensor, ...],
                       text_mask: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        img_cos, img_sin, txt_cos, txt_sin = rope
        s_img, s_txt = hidden.shape[0], encoder.shape[0]
        s, dl, lead = s_txt + s_img, self.heads_local * HEAD_DIM, self.rank == 0
        ish1, isc1, ig1, ish2, isc2, ig2 = mod_img
        tsh1, tsc1, tg1, tsh2, tsc2, tg2 = mod_txt
        img_in = layernorm_modulate(hidden, ish1, isc1, eps=self.eps)
        txt_in = layernorm_modulate(encoder, tsh1, tsc1, eps=self.eps)
        q = torch.empty((s, dl), dtype=torch.bfloat16, device=hidden.device)
        k = torch.empty_like(q)
        v = torch.empty_like(q)
        project_qkv(self, txt_in, img_in, q, k, v)
        qk_rmsnorm_rope_(q[:s_txt], self.norms["attn.norm_added_q"], txt_cos, txt_sin, eps=self.eps)
        qk_rmsnorm_rope_(q[s_txt:], self.norms["attn.norm_q"], img_cos, img_sin, eps=self.eps)
        qk_rmsnorm_rope_(k[:s_txt], self.norms["attn.norm_added_k"], txt_cos, txt_sin, eps=self.eps)
        qk_rmsnorm_rope_(k[s_txt:], self.norms["attn.norm_k"], img_cos, img_sin, eps=self.eps)
        joint = joint_attention(q, k, v, self.heads_local, s_txt, text_mask)
        # row-parallel output projections into one joint [text; image] buffer, one all-reduce
        streams = torch.empty((s, self.dim), dtype=torch.bfloat16, device=hidden.device)
        self._linear("attn.attn_to_out.0", joint[s_txt:], residual=hidden if lead else None, gate=ig1,
                     out=streams[s_txt:])
        self._linear("attn.to_add_out", joint[:s_txt], residual=encoder if lead else None, gate=tg1,
                     out=streams[:s_txt])
        self._all_reduce(streams)
        txt_h, img_h = streams[:s_txt], streams[s_txt:]
        img_ff_in = layernorm_modulate(img_h, ish2, isc2, eps=self.eps)
        txt_ff_in = layernorm_modulate(txt_h, tsh2, tsc2, eps=self.eps)
        outs = torch.empty_like(streams)
        self._mlp("img_ff", img_ff_in, img_h if lead else None, ig2, outs[s_txt:])
        self._mlp("txt_ff", txt_ff_in, txt_h if lead else None, tg2, outs[:s_txt])
        self._all_reduce(outs)
        return outs[:s_txt], outs[s_txt:]

    def forward(self, hidden: torch.Tensor, encoder: torch.Tensor, temb: torch.Tensor,
                rope: tuple[torch.Tensor, ...],
                encoder_mask: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        mod_img, mod_txt = self.modulation(temb)
        outs = [self.forward_sample(hidden[b], encoder[b], mod_img[b], mod_txt[b], rope,
                                    None if encoder_mask is None else encoder_mask[b])
                for b in range(hidden.shape[0])]
        return torch.stack([o[0] for o in outs]), torch.stack([o[1] for o in outs])
