"""One Qwen-Image MMDiT dual-stream block on the q6 kernels.

The block the reference profiles stage by stage
(benchmarks/profile_qwen_block.py:163-301; mflux ``QwenTransformerBlock``):

=====================================  =========================================================
reference stage                         here
=====================================  =========================================================
img/txt_mod_linear(silu(temb))         ``q6_linear`` on the few-row streaming GEMV (M = batch)
_modulate(norm1(x), mod1)              ``q6_add_layernorm_modulate_bf16``: one launch over the
                                        joint rows of every sample and stream
to_q/k/v, add_q/k/v_proj               one GEMM per (sample, stream) of the concatenated q, k, v
                                        projections, writing a joint [text; image] qkv buffer
norm_q/k, norm_added_q/k + rope        ``q6_qk_rmsnorm_rope_joint_bf16`` in place, one launch
                                        for q and one for k over all rows
joint attention (_compute_attention)   torch scaled_dot_product_attention over the batch
                                        (library kernel), text padding masked as keys
attn_to_out[0] / to_add_out + gate1    ``q6_linear`` with the residual and gate in its epilogue
_modulate(norm2(x), mod2)              ``q6_add_layernorm_modulate_bf16``
img_ff / txt_ff + gate2 residual       ``q6_mlp`` with the residual and gate in fc2's epilogue
=====================================  =========================================================

Rows of a batch live in one joint buffer [B * S, D], each sample's S rows
text first ([text; image], the order of the reference's joint attention).
``TensorParallelQwenBlock`` splits the block over the GPUs of a process
group: heads and feed-forward columns per rank, and the rows between the
GEMMs (adaLN modulate, residuals) sequence-parallel, with an all-gather
before each column-parallel GEMM and a reduce-scatter after each
row-parallel one.

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

    overlap_streams = True  # text- and image-stream GEMMs on two CUDA streams (both_streams)

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

    def _workspace(self, m: int, h: int, d: int, device: torch.device, slot: int = 0) -> torch.Tensor:
        """MLP workspace; one per stream that runs MLPs concurrently (``slot``)."""

        need = int(ops.mlp_workspace_bytes(m, h, d))
        slots = self.__dict__.setdefault("_ws_slots", {})
        ws = slots.get(slot)
        if ws is None or ws.numel() < need or ws.device != device:
            ws = torch.empty(need, dtype=torch.uint8, device=device)
            slots[slot] = ws
        return ws

    def _linear(self, name: str, x: torch.Tensor, **kw) -> torch.Tensor:
        lin = self.linears[name]
        return ops.q6_linear(x, lin.weight, lin.scales, lin.biases, lin.bias, group_size=lin.group_size,
                             lora=lin.lora, lora_b_nmajor=getattr(lin, "lora_b_nmajor", None), **kw)

    def _mlp(self, prefix: str, x: torch.Tensor, residual: torch.Tensor | None, gate: torch.Tensor,
             out: torch.Tensor, slot: int = 0) -> torch.Tensor:
        l1, l2 = self.linears[f"{prefix}.mlp_in"], self.linears[f"{prefix}.mlp_out"]
        if l1.lora is not None or l2.lora is not None:
            mid = ops.q6_linear(x, l1.weight, l1.scales, l1.biases, l1.bias, group_size=l1.group_size,
                                apply_gelu=True, lora=l1.lora, lora_b_nmajor=getattr(l1, "lora_b_nmajor", None))
            return ops.q6_linear(mid, l2.weight, l2.scales, l2.biases, l2.bias, group_size=l2.group_size,
                                 residual=residual, gate=gate, lora=l2.lora, out=out,
                                 lora_b_nmajor=getattr(l2, "lora_b_nmajor", None))
        ws = self._workspace(x.shape[0], l1.out_features, l1.in_features, x.device, slot)
        return ops.q6_mlp(x, (l1.weight, l1.scales, l1.biases, l1.bias), (l2.weight, l2.scales, l2.biases, l2.bias),
                          group_size=l1.group_size, residual=residual, gate=gate, workspace=ws, out=out)

    def modulation_joint(self, temb: torch.Tensor) -> torch.Tensor:
        """Modulation vectors [B, 2, 6, D] (text stream first) from the
        timestep embedding [B, D]: txt_mod_linear and img_mod_linear read the
        same silu(temb), so one GEMV over their row concatenation writes both
        in the layout the joint-row kernels index (no copies)."""

        t = F.silu(temb.to(torch.bfloat16))
        b = t.shape[0]
        fused = fused_rows(self, _MOD)
        if fused is not None:
            y = ops.q6_linear(t, fused.weight, fused.scales, fused.biases, fused.bias, group_size=fused.group_size)
            return y.view(b, 2, 6, self.dim)
        return torch.stack([self._linear(name, t).view(b, 6, self.dim) for name in _MOD], dim=1)

    def modulation(self, temb: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """(img, txt) modulation vectors [B, 6, D] from the timestep embedding [B, D]."""

        both = self.modulation_joint(temb)
        return both[:, 1], both[:, 0]

    def forward_joint(self, x: torch.Tensor, temb: torch.Tensor, rope_joint: tuple[torch.Tensor, torch.Tensor],
                      batch: int, text_len: int, text_mask: torch.Tensor | None = None,
                      out: torch.Tensor | None = None) -> torch.Tensor:
        """The block over joint rows ``x`` [B * S, D] (each sample's S rows text
        first); ``rope_joint`` = (cos, sin) fp32 [S, 64] with the text rows
        first; ``text_mask`` [B, S_txt] or None.  Returns the joint output rows."""

        rows, d = x.shape
        seq = rows // batch
        vec = ModulationVectors(self.modulation_joint(temb))
        z = add_layernorm_modulate(x, vec.shift1, vec.scale1, seq_len=seq, text_len=text_len, eps=self.eps)
        qkv = torch.empty((rows, 3 * d), dtype=torch.bfloat16, device=x.device)
        both_streams(self, x.device,
                     lambda: project_qkv_joint(self, z, qkv, batch, seq, text_len, which=0),
                     lambda: project_qkv_joint(self, z, qkv, batch, seq, text_len, which=1))
        rope_qk_joint(self, qkv, d, rope_joint, seq, text_len)
        att = batched_joint_attention(qkv, d, batch, seq, self.heads, text_len, text_mask)
        h = torch.empty_like(x)

        def out_proj(which: int) -> None:
            for b, stream, r in segments(batch, seq, text_len):
                if stream == which:
                    name = "attn.to_add_out" if stream == 0 else "attn.attn_to_out.0"
                    self._linear(name, att[r], residual=x[r], gate=vec.gate1(b, stream), out=h[r])

        both_streams(self, x.device, lambda: out_proj(0), lambda: out_proj(1))
        z2 = add_layernorm_modulate(h, vec.shift2, vec.scale2, seq_len=seq, text_len=text_len, eps=self.eps)
        y = out if out is not None else torch.empty_like(x)

        def ff(which: int) -> None:
            for b, stream, r in segments(batch, seq, text_len):
                if stream == which:
                    self._mlp("txt_ff" if stream == 0 else "img_ff", z2[r], h[r], vec.gate2(b, stream), y[r],
                              slot=stream)

        both_streams(self, x.device, lambda: ff(0), lambda: ff(1))
        return y

    def forward(self, hidden: torch.Tensor, encoder: torch.Tensor, temb: torch.Tensor,
                rope: tuple[torch.Tensor, ...],
                encoder_mask: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """hidden [B, S_img, D], encoder [B, S_txt, D], temb [B, D] (bf16);
        ``rope`` = (img_cos, img_sin, txt_cos, txt_sin) fp32 [S, 64];
        ``encoder_mask`` [B, S_txt] (1 = text token, 0 = padding; None = no
        padding).  Returns (encoder_out, hidden_out) like the reference block."""

        x, batch, s_txt = joint_rows(hidden, encoder)
        y = self.forward_joint(x, temb, joint_rope(rope), batch, s_txt, encoder_mask)
        return split_joint(y, batch, s_txt)


# ------------------------------------------------------------------- joint-row helpers


class ModulationVectors:
    """A block's adaLN vectors per (sample, stream) as views of the
    [B, 2 streams (text, image), 6, D] modulation output: shift / scale of
    the attention half (1) and of the feed-forward half (2) as [2 B, D] views
    whose rows lie 6 D apart (the joint-row kernels take that vector stride),
    and the gates as [D] views.  Nothing is copied."""

    def __init__(self, both: torch.Tensor) -> None:
        if both.dim() != 4 or both.shape[1:3] != (2, 6) or not both.is_contiguous():
            raise ValueError("modulation vectors must be a contiguous [B, 2, 6, D] tensor")
        self.shift1 = both[:, :, 0].flatten(0, 1)
        self.scale1 = both[:, :, 1].flatten(0, 1)
        self.shift2 = both[:, :, 3].flatten(0, 1)
        self.scale2 = both[:, :, 4].flatten(0, 1)
        self._both = both

    @classmethod
    def from_streams(cls, mod_img: torch.Tensor, mod_txt: torch.Tensor) -> "ModulationVectors":
        """From separate [B, 6, D] image and text modulation outputs."""

        return cls(torch.stack([mod_txt, mod_img], dim=1).contiguous())

    def gate1(self, b: int, stream: int) -> torch.Tensor:
        return self._both[b, stream, 2]

    def gate2(self, b: int, stream: int) -> torch.Tensor:
        return self._both[b, stream, 5]


def segments(batch: int, seq: int, text_len: int):
    """(sample, stream, row slice) of the joint rows: stream 0 text, 1 image."""

    for b in range(batch):
        if text_len:
            yield b, 0, slice(b * seq, b * seq + text_len)
        if seq > text_len:
            yield b, 1, slice(b * seq + text_len, (b + 1) * seq)


def joint_rows(hidden: torch.Tensor, encoder: torch.Tensor) -> tuple[torch.Tensor, int, int]:
    """[B * S, D] joint rows (each sample's text rows, then its image rows)."""

    batch, s_txt, d = encoder.shape
    x = torch.cat([encoder.to(torch.bfloat16), hidden.to(torch.bfloat16)], dim=1)
    return x.reshape(batch * (s_txt + hidden.shape[1]), d).contiguous(), batch, s_txt


def split_joint(y: torch.Tensor, batch: int, s_txt: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(text rows [B, S_txt, D], image rows [B, S_img, D]) views of joint rows."""

    v = y.view(batch, -1, y.shape[-1])
    return v[:, :s_txt], v[:, s_txt:]


def joint_rope(rope: tuple[torch.Tensor, ...]) -> tuple[torch.Tensor, torch.Tensor]:
    """(cos, sin) [S, 64] of the joint sequence (text rows first) from
    (img_cos, img_sin, txt_cos, txt_sin)."""

    img_cos, img_sin, txt_cos, txt_sin = rope
    return torch.cat([txt_cos, img_cos]).contiguous(), torch.cat([txt_sin, img_sin]).contiguous()


def vector_stride(shift: torch.Tensor, scale: torch.Tensor, d: int) -> int:
    """Element stride between the modulation vectors of ``shift`` / ``scale``
    ([V, D] views with unit column stride, the same row stride; or [D])."""

    for t in (shift, scale):
        if t.dtype != torch.bfloat16 or t.shape[-1] != d or t.dim() not in (1, 2) or t.stride(-1) != 1:
            raise ValueError(f"modulation vectors must be bf16 [V, {d}] with unit column stride")
    if shift.dim() != scale.dim() or (shift.dim() == 2 and (shift.shape[0] != scale.shape[0]
                                                             or shift.stride(0) != scale.stride(0))):
        raise ValueError("shift and scale must have the same layout")
    return d if shift.dim() == 1 or shift.shape[0] == 1 else int(shift.stride(0))


def add_layernorm_modulate(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, *,
                           add: torch.Tensor | None = None, h_out: torch.Tensor | None = None,
                           out: torch.Tensor | None = None, row0: int = 0, seq_len: int = 0, text_len: int = 0,
                           eps: float = 1e-6) -> torch.Tensor:
    """y = LayerNorm(x [+ add]) * (1 + scale[v]) + shift[v] over joint rows
    (q6_add_layernorm_modulate_bf16): row m is row row0 + m of sequences of
    ``seq_len`` rows whose first ``text_len`` are text; shift / scale are
    [samples * 2, D] vectors (text, image per sample), or [D] for one vector,
    whose rows may lie any multiple of 8 elements apart (``vector_stride``),
    e.g. one chunk of the [B, 2, 6, D] modulation output.  ``h_out`` receives
    x + add."""

    d = x.shape[-1]
    if x.dtype != torch.bfloat16 or not x.is_contiguous():
        raise ValueError("x must be contiguous bf16 rows")
    if add is not None and (add.dtype != torch.bfloat16 or not add.is_contiguous() or add.shape != x.shape):
        raise ValueError("add must match x")
    vs = vector_stride(shift, scale, d)
    y = out if out is not None else torch.empty_like(x)
    st = _lib.lib().q6_add_layernorm_modulate_bf16(
        x.data_ptr(), None if add is None else add.data_ptr(), None if h_out is None else h_out.data_ptr(),
        shift.data_ptr(), scale.data_ptr(), vs, y.data_ptr(), x.shape[0], d, int(row0), int(seq_len),
        int(text_len), float(eps), ops._stream(x.device))
    _lib.check(st, "q6_add_layernorm_modulate_bf16")
    return y


def qk_rmsnorm_rope_joint_(qk: torch.Tensor, w_text: torch.Tensor, w_image: torch.Tensor, cos: torch.Tensor,
                           sin: torch.Tensor, *, row0: int = 0, seq_len: int = 0, text_len: int = 0,
                           eps: float = 1e-6) -> torch.Tensor:
    """In place on joint rows [M, H * 128] (row stride may exceed the width):
    text rows take ``w_text``, image rows ``w_image``; row m uses angle-table
    row (row0 + m) % seq_len of cos / sin [seq_len, 64]."""

    if qk.dtype != torch.bfloat16 or qk.dim() != 2 or qk.stride(1) != 1:
        raise ValueError("qk must be a 2-D bf16 view with unit column stride")
    m, width = qk.shape
    st = _lib.lib().q6_qk_rmsnorm_rope_joint_bf16(
        qk.data_ptr(), qk.stride(0), m, width // HEAD_DIM, HEAD_DIM, w_text.data_ptr(), w_image.data_ptr(),
        cos.data_ptr(), sin.data_ptr(), int(row0), int(seq_len), int(text_len), float(eps), ops._stream(qk.device))
    _lib.check(st, "q6_qk_rmsnorm_rope_joint_bf16")
    return qk


def rope_qk_joint(owner, qkv: torch.Tensor, width: int, rope_joint: tuple[torch.Tensor, torch.Tensor], seq: int,
                  text_len: int) -> None:
    """QK-RMSNorm and rotary embedding on the q and k columns of a joint qkv buffer."""

    cos, sin = rope_joint
    n = owner.norms
    qk_rmsnorm_rope_joint_(qkv[:, :width], n["attn.norm_added_q"], n["attn.norm_q"], cos, sin, seq_len=seq,
                           text_len=text_len, eps=owner.eps)
    qk_rmsnorm_rope_joint_(qkv[:, width:2 * width], n["attn.norm_added_k"], n["attn.norm_k"], cos, sin,
                           seq_len=seq, text_len=text_len, eps=owner.eps)


def batched_joint_attention(qkv: torch.Tensor, width: int, batch: int, seq: int, heads: int, text_len: int,
                            text_mask: torch.Tensor | None = None) -> torch.Tensor:
    """Joint [text; image] attention of every sample from a qkv buffer [B * S,
    3 * width] (torch scaled_dot_product_attention over [B, heads, S, 128]).
    ``text_mask`` [B, S_txt] (1 = token, 0 = padding) removes padded text
    tokens as keys while every image token stays a key: the joint mask the
    reference builds from ``encoder_hidden_states_mask``
    (benchmarks/profile_qwen_block.py:228-248).  Without a mask the library's
    unmasked flash kernel runs.  Returns [B * S, width] rows."""

    def view(j: int) -> torch.Tensor:
        return qkv[:, j * width:(j + 1) * width].view(batch, seq, heads, HEAD_DIM).transpose(1, 2)

    mask = None
    if text_mask is not None:
        keep = torch.ones((batch, seq), dtype=torch.bool, device=qkv.device)
        keep[:, :text_len] = text_mask.reshape(batch, text_len).to(qkv.device) > 0.5
        mask = keep.view(batch, 1, 1, seq)
    att = F.scaled_dot_product_attention(view(0), view(1), view(2), attn_mask=mask, scale=1.0 / math.sqrt(HEAD_DIM))
    return att.transpose(1, 2).reshape(batch * seq, width)


_MOD = ("txt_mod_linear", "img_mod_linear")  # text first: the [B, 2, 6, D] stream order
_TXT_QKV = ("attn.add_q_proj", "attn.add_k_proj", "attn.add_v_proj")
_IMG_QKV = ("attn.to_q", "attn.to_k", "attn.to_v")


def fused_rows(owner: torch.nn.Module, names: tuple[str, ...]) -> QuantizedLinear | None:
    """Row concatenation of q6 linears of ``owner.linears`` that read the same
    input (one stream's q, k and v projections): one GEMM whose output
    columns are theirs side by side, written straight into the joint qkv
    buffer.  At a few hundred tokens the three 3072-row GEMMs each fill a
    third of the GPU's tiles (and need split-K); their concatenation fills it
    alone.  The members' tensors are rebound to views of the concatenation,
    so no weight is held twice.  None when a member carries a LoRA delta or
    the members differ in input or group size."""

    lins = [owner.linears[n] for n in names]
    if any(lin.lora is not None for lin in lins):
        return None
    if len({(lin.in_features, lin.group_size, lin.weight.device) for lin in lins}) != 1:
        return None
    # the cache lives on the first member, so every owner sharing the members
    # (a block and its tensor-parallel form) shares one concatenation
    cache = lins[0].__dict__.setdefault("_fused_rows", {})
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


def both_streams(owner, device: torch.device, text_fn, image_fn) -> None:
    """Run a stage's text-stream launches (``text_fn``) and image-stream
    launches (``image_fn``), which touch disjoint rows and weights, on two CUDA
    streams: the text work on a side stream that first waits for everything
    queued so far, the image work on the caller's stream, which then waits
    for the side stream.  The small text GEMMs (256 rows) fill SMs that the
    image GEMM's last wave leaves idle.  With ``owner.overlap_streams`` False
    both run in order on the caller's stream.  CUDA graph capture records the
    fork and the join."""

    if not getattr(owner, "overlap_streams", True):
        text_fn()
        image_fn()
        return
    side = owner.__dict__.get("_side_stream")
    if side is None or side.device != device:
        side = torch.cuda.Stream(device)
        owner.__dict__["_side_stream"] = side
    main = torch.cuda.current_stream(device)
    side.wait_stream(main)
    with torch.cuda.stream(side):
        text_fn()
    image_fn()
    main.wait_stream(side)


def project_qkv_joint(owner: torch.nn.Module, z: torch.Tensor, qkv: torch.Tensor, batch: int, seq: int,
                      text_len: int, which: int | None = None, segs=None) -> None:
    """q, k, v of every joint row into qkv [B * S, 3 * width]: one GEMM per
    (sample, stream) of the stream's concatenated projections (``fused_rows``);
    a stream with a LoRA delta on one of them runs its three GEMMs and copies.
    ``which`` (0 text, 1 image) limits the launches to one stream; ``segs``
    ((sample, stream, row slice) triples) replaces the joint rows' segments."""

    fused = {0: fused_rows(owner, _TXT_QKV), 1: fused_rows(owner, _IMG_QKV)}
    width = qkv.shape[1] // 3
    for _, stream, r in (segments(batch, seq, text_len) if segs is None else segs):
        if which is not None and stream != which:
            continue
        f = fused[stream]
        if f is not None:
            ops.q6_linear(z[r], f.weight, f.scales, f.biases, f.bias, group_size=f.group_size, out=qkv[r])
            continue
        for j, name in enumerate(_TXT_QKV if stream == 0 else _IMG_QKV):
            qkv[r, j * width:(j + 1) * width].copy_(owner._linear(name, z[r]))


def block_flops(s_img: int, s_txt: int, dim: int) -> int:
    """FLOPs of one block forward (one sample): per token 8 D^2 for q, k, v
    and the output projection and 16 D^2 for the 4x feed-forward, 4 S^2 D for
    the joint attention (q k^T and p v), 24 D^2 for the two modulation linears."""

    s = s_img + s_txt
    return 24 * s * dim * dim + 4 * s * s * dim + 24 * dim * dim


# ------------------------------------------------------------------- tensor parallel

_PEER_ROWS: dict = {}


class TensorParallelQwenBlock(torch.nn.Module):
    """The block split over the ranks of a process group (one rank per GPU).

    Heads and the feed-forward hidden columns are divided: q / k / v and
    mlp_in are column-parallel (each rank holds its heads' / columns' rows of
    codes, scales and biases), the output projections and mlp_out are
    row-parallel (each rank holds the matching K slice).  Between the GEMMs
    the joint rows are sequence-parallel: rank r holds rows [r R, (r + 1) R)
    of the [B * S, D] joint rows (R = B S / world) and runs the adaLN
    modulate and the residual adds on them alone.  So each half of the block
    is all-gather (modulated rows) -> column-parallel GEMM -> local work ->
    row-parallel GEMM -> reduce-scatter (partial sums, gate and rank-0 bias
    applied in the epilogue) -> residual add + next modulate on local rows.
    The modulation linears (M = batch) are replicated.
    """

    def __init__(self, full: QwenTransformerBlock, world: int, rank: int, group=None, comm: str = "nccl") -> None:
        super().__init__()
        from qwen_image_shardedit_mlx_b200.sharding import split_k, split_rows

        if comm not in ("nccl", "peer"):
            raise ValueError(f"comm must be 'nccl' or 'peer', got {comm!r}")
        self.comm = comm

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

    overlap_streams = True  # text- and image-stream GEMMs on two CUDA streams (both_streams)
    _linear = QwenTransformerBlock._linear
    _workspace = QwenTransformerBlock._workspace
    _mlp = QwenTransformerBlock._mlp
    modulation = QwenTransformerBlock.modulation
    modulation_joint = QwenTransformerBlock.modulation_joint

    # collectives over the rows of the joint buffer
    def _gather(self, local: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return local
        import torch.distributed as dist

        full = torch.empty((local.shape[0] * self.world, local.shape[1]), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(full, local, group=self.group)
        return full

    def _reduce_scatter(self, full: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return full
        import torch.distributed as dist

        local = torch.empty((full.shape[0] // self.world, full.shape[1]), dtype=full.dtype, device=full.device)
        dist.reduce_scatter_tensor(local, full, op=dist.ReduceOp.SUM, group=self.group)
        return local

    def _peer(self, rows_total: int, device: torch.device):
        """The peer-memory row buffers of this group (one set shared by every
        block of the group with the same shape)."""

        from qwen_image_shardedit_mlx_b200.peer import PeerRows

        key = (id(self.group), int(rows_total), self.dim, str(device))
        pr = _PEER_ROWS.get(key)
        if pr is None:
            pr = PeerRows(rows_total, self.dim, self.group, device)
            _PEER_ROWS[key] = pr
        return pr

    def forward_local(self, x_local: torch.Tensor, temb: torch.Tensor,
                      rope_joint: tuple[torch.Tensor, torch.Tensor], batch: int, seq: int, text_len: int,
                      text_mask: torch.Tensor | None = None,
                      mod: torch.Tensor | None = None) -> tuple[torch.Tensor, object]:
        """This rank's joint rows through the block: x_local [R, D] are rows
        [rank R, (rank + 1) R) of the [B * S, D] joint rows.  Returns a
        pending pair: the block's output rows are h + ff (``finish``); a stack
        may instead hand the pair to the next block, whose first modulate
        adds them in the same pass.  ``mod``: this block's modulation vectors
        [B, 2, 6, D] when computed beforehand (``stack_modulations``)."""

        rows_local, d = x_local.shape
        row0 = self.rank * rows_local
        vec = ModulationVectors(self.modulation_joint(temb) if mod is None else mod)
        if self.comm == "peer":
            pr = self._peer(rows_local * self.world, x_local.device)
            pr.add_ln_gather(x_local, vec.shift1, vec.scale1, dst="gather1", seq_len=seq, text_len=text_len,
                             eps=self.eps)
            pr.barrier()
            return self._rest_peer(pr, x_local, vec, rope_joint, batch, seq, text_len, text_mask)
        z = self._gather(add_layernorm_modulate(x_local, vec.shift1, vec.scale1, row0=row0, seq_len=seq,
                                                text_len=text_len, eps=self.eps))
        return self._rest(x_local, z, vec, rope_joint, batch, seq, text_len, text_mask, row0)

    def forward_local_pending(self, pending: tuple[torch.Tensor, torch.Tensor], temb: torch.Tensor,
                              rope_joint: tuple[torch.Tensor, torch.Tensor], batch: int, seq: int,
                              text_len: int, text_mask: torch.Tensor | None = None,
                              mod: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """``forward_local`` of the output (h, ff) of the previous block: its
        residual add x = h + ff is formed in the same pass as this block's
        first modulate."""

        h_prev, ff_prev = pending
        rows_local = h_prev.shape[0]
        row0 = self.rank * rows_local
        vec = ModulationVectors(self.modulation_joint(temb) if mod is None else mod)
        x_local = torch.empty_like(h_prev)
        if self.comm == "peer":
            pr = self._peer(rows_local * self.world, h_prev.device)
            pr.add_ln_gather(h_prev, vec.shift1, vec.scale1, dst="gather1", partials=ff_prev, h_out=x_local,
                             seq_len=seq, text_len=text_len, eps=self.eps)
            pr.barrier()
            return self._rest_peer(pr, x_local, vec, rope_joint, batch, seq, text_len, text_mask)
        z_local = add_layernorm_modulate(h_prev, vec.shift1, vec.scale1, add=ff_prev, h_out=x_local, row0=row0,
                                         seq_len=seq, text_len=text_len, eps=self.eps)
        return self._rest(x_local, self._gather(z_local), vec, rope_joint, batch, seq, text_len, text_mask, row0)

    def _rest_peer(self, pr, x_local, vec, rope_joint, batch, seq, text_len, text_mask):
        """The block after the first modulate, with the fused peer kernels:
        partial sums land in this rank's ``part`` buffers, the next kernel
        reduces them onto their owners and gathers the modulated rows."""

        dl = self.heads_local * HEAD_DIM
        z = pr.buffers["gather1"]
        rows = z.shape[0]
        qkv = torch.empty((rows, 3 * dl), dtype=torch.bfloat16, device=z.device)
        both_streams(self, z.device,
                     lambda: project_qkv_joint(self, z, qkv, batch, seq, text_len, which=0),
                     lambda: project_qkv_joint(self, z, qkv, batch, seq, text_len, which=1))
        rope_qk_joint(self, qkv, dl, rope_joint, seq, text_len)
        att = batched_joint_attention(qkv, dl, batch, seq, self.heads_local, text_len, text_mask)
        part = pr.buffers["part1"]

        def out_proj(which: int) -> None:
            for b, stream, r in segments(batch, seq, text_len):
                if stream == which:
                    name = "attn.to_add_out" if stream == 0 else "attn.attn_to_out.0"
                    self._linear(name, att[r], gate=vec.gate1(b, stream), out=part[r])

        both_streams(self, z.device, lambda: out_proj(0), lambda: out_proj(1))
        pr.barrier()
        h_local = torch.empty_like(x_local)
        pr.add_ln_gather(x_local, vec.shift2, vec.scale2, dst="gather2", partials="part1", h_out=h_local,
                         seq_len=seq, text_len=text_len, eps=self.eps)
        pr.barrier()
        z2 = pr.buffers["gather2"]
        part2 = pr.buffers["part2"]

        def ff(which: int) -> None:
            for b, stream, r in segments(batch, seq, text_len):
                if stream == which:
                    self._mlp("txt_ff" if stream == 0 else "img_ff", z2[r], None, vec.gate2(b, stream), part2[r],
                              slot=stream)

        both_streams(self, z2.device, lambda: ff(0), lambda: ff(1))
        pr.barrier()
        return h_local, "part2"

    def _rest(self, x_local, z, vec, rope_joint, batch, seq, text_len, text_mask, row0):
        d, dl = self.dim, self.heads_local * HEAD_DIM
        rows = z.shape[0]
        qkv = torch.empty((rows, 3 * dl), dtype=torch.bfloat16, device=z.device)
        project_qkv_joint(self, z, qkv, batch, seq, text_len)
        rope_qk_joint(self, qkv, dl, rope_joint, seq, text_len)
        att = batched_joint_attention(qkv, dl, batch, seq, self.heads_local, text_len, text_mask)
        part = torch.empty((rows, d), dtype=torch.bfloat16, device=z.device)
        for b, stream, r in segments(batch, seq, text_len):
            name = "attn.to_add_out" if stream == 0 else "attn.attn_to_out.0"
            self._linear(name, att[r], gate=vec.gate1(b, stream), out=part[r])
        attn_local = self._reduce_scatter(part)
        h_local = torch.empty_like(x_local)
        z2 = self._gather(add_layernorm_modulate(x_local, vec.shift2, vec.scale2, add=attn_local, h_out=h_local,
                                                 row0=row0, seq_len=seq, text_len=text_len, eps=self.eps))
        part2 = torch.empty((rows, d), dtype=torch.bfloat16, device=z.device)
        for b, stream, r in segments(batch, seq, text_len):
            self._mlp("txt_ff" if stream == 0 else "img_ff", z2[r], None, vec.gate2(b, stream), part2[r])
        return h_local, self._reduce_scatter(part2)

    def finish(self, pending: tuple[torch.Tensor, object]) -> torch.Tensor:
        """The output rows h + ff of a pending pair."""

        h, ff = pending
        if isinstance(ff, str):  # peer path: ff is every rank's partial-sum buffer
            pr = self._peer(h.shape[0] * self.world, h.device)
            out = torch.empty_like(h)
            pr.add_ln_gather(h, None, None, dst=None, partials=ff, h_out=out)
            return out
        return h + ff

    def forward(self, hidden: torch.Tensor, encoder: torch.Tensor, temb: torch.Tensor,
                rope: tuple[torch.Tensor, ...],
                encoder_mask: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """Full inputs and outputs on every rank (each rank computes its row
        shard, then the output rows are all-gathered)."""

        x, batch, s_txt = joint_rows(hidden, encoder)
        rows = x.shape[0]
        if rows % self.world:
            raise ValueError(f"{rows} joint rows do not split over {self.world} ranks")
        r = rows // self.world
        x_local = x[self.rank * r:(self.rank + 1) * r].contiguous()
        seq = rows // batch
        y_local = self.finish(self.forward_local(x_local, temb, joint_rope(rope), batch, seq, s_txt, encoder_mask))
        return split_joint(self._gather(y_local), batch, s_txt)



class ContextParallelQwenBlock(torch.nn.Module):
    """The block with its joint rows split over the ranks (context
    parallelism): rank r of W keeps rows [r S / W, (r + 1) S / W) of every
    sample's joint sequence (S rows, text first) through the whole block and
    holds every weight (the full block, replicated), and only keys and values
    cross GPUs: one all-gather per sample before the joint attention, whose
    queries are the rank's rows.  Every GEMM keeps all its output columns and
    all of K, so at 8 GPUs the image GEMMs run on 464 rows at the tensor
    path's full tile widths, where the tensor-parallel form's out-projection
    (K = 384) and q / k / v (1152 columns) leave most SMs idle.  A stack keeps
    the rows sharded from block to block.  The per-rank weights are the whole
    model's (16.6 GB for 60 blocks).  Requires S divisible by W."""

    overlap_streams = True  # text- and image-stream GEMMs on two CUDA streams (both_streams)

    def __init__(self, full: QwenTransformerBlock, world: int, rank: int, group=None) -> None:
        super().__init__()
        self.full = full
        self.world, self.rank, self.group = int(world), int(rank), group
        self.dim, self.heads, self.eps = full.dim, full.heads, full.eps

    def modulation_joint(self, temb: torch.Tensor) -> torch.Tensor:
        return self.full.modulation_joint(temb)

    def rows_per_rank(self, seq: int) -> int:
        if seq % self.world:
            raise ValueError(f"{seq} joint rows per sample do not split over {self.world} ranks")
        return seq // self.world

    def local_rows(self, x: torch.Tensor, batch: int, seq: int) -> torch.Tensor:
        """This rank's rows [B * R, D] of joint rows x [B * S, D]."""

        r = self.rows_per_rank(seq)
        return x.view(batch, seq, -1)[:, self.rank * r:(self.rank + 1) * r].reshape(batch * r, -1).contiguous()

    def local_segments(self, batch: int, seq: int, text_len: int):
        """(sample, stream, local row slice) of this rank's rows: stream 0 text, 1 image."""

        r = self.rows_per_rank(seq)
        t = min(max(text_len - self.rank * r, 0), r)
        out = []
        for b in range(batch):
            if t:
                out.append((b, 0, slice(b * r, b * r + t)))
            if t < r:
                out.append((b, 1, slice(b * r + t, (b + 1) * r)))
        return out

    def _comm_stream(self, device: torch.device) -> torch.cuda.Stream:
        side = self.__dict__.get("_comm")
        if side is None or side.device != device:
            side = torch.cuda.Stream(device)
            self.__dict__["_comm"] = side
        return side

    def _gather_kv(self, kv_local: torch.Tensor, batch: int, seq: int) -> torch.Tensor:
        """Keys and values of every row of every sample, [B, S, 2D], from this
        rank's [B * R, 2D] (one all-gather per sample)."""

        if self.world == 1:
            return kv_local.view(batch, seq, -1)
        import torch.distributed as dist

        r = seq // self.world
        full = torch.empty((batch, seq, kv_local.shape[1]), dtype=kv_local.dtype, device=kv_local.device)
        for b in range(batch):
            dist.all_gather_into_tensor(full[b], kv_local[b * r:(b + 1) * r], group=self.group)
        return full

    def forward_local(self, x_local: torch.Tensor, temb: torch.Tensor, rope_joint: tuple[torch.Tensor, torch.Tensor],
                      batch: int, seq: int, text_len: int, text_mask: torch.Tensor | None = None,
                      mod: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's output rows [B * R, D] from its input rows ``x_local``
        (``local_rows`` of the joint rows); ``rope_joint`` covers the whole
        sequence; ``mod`` = the block's [B, 2, 6, D] modulation vectors when
        precomputed (``stack_modulations``)."""

        full, d = self.full, self.dim
        r = self.rows_per_rank(seq)
        r0 = self.rank * r
        dev = x_local.device
        vec = ModulationVectors(full.modulation_joint(temb) if mod is None else mod)
        segs = self.local_segments(batch, seq, text_len)
        cos, sin = rope_joint
        n = full.norms

        def modulate(src: torch.Tensor, shift, scale, dst: torch.Tensor) -> None:
            for b in range(batch):  # row0 places each sample's rows in its sequence
                rows = slice(b * r, (b + 1) * r)
                add_layernorm_modulate(src[rows], shift, scale, out=dst[rows], row0=b * seq + r0, seq_len=seq,
                                       text_len=text_len, eps=self.eps)

        z = torch.empty_like(x_local)
        modulate(x_local, vec.shift1, vec.scale1, z)
        qkv = torch.empty((batch * r, 3 * d), dtype=torch.bfloat16, device=dev)
        kv_src = torch.empty((batch * r, 2 * d), dtype=torch.bfloat16, device=dev)
        kv = torch.empty((batch, seq, 2 * d), dtype=torch.bfloat16, device=dev) if self.world > 1 else None
        main = torch.cuda.current_stream(dev)
        comm = self._comm_stream(dev) if self.world > 1 else None
        landed = []
        # Sample by sample: q / k / v, QK-norm + RoPE, then its keys and values
        # leave on the communication stream while the next sample's GEMMs run.
        for b in range(batch):
            rows = slice(b * r, (b + 1) * r)
            mine = [sg for sg in segs if sg[0] == b]
            both_streams(self, dev,
                         lambda: project_qkv_joint(full, z, qkv, batch, seq, text_len, which=0, segs=mine),
                         lambda: project_qkv_joint(full, z, qkv, batch, seq, text_len, which=1, segs=mine))
            for j, (w_txt, w_img) in enumerate((("attn.norm_added_q", "attn.norm_q"),
                                                ("attn.norm_added_k", "attn.norm_k"))):
                qk_rmsnorm_rope_joint_(qkv[rows, j * d:(j + 1) * d], n[w_txt], n[w_img], cos, sin, row0=b * seq + r0,
                                       seq_len=seq, text_len=text_len, eps=self.eps)
            kv_src[rows].copy_(qkv[rows, d:])
            if comm is not None:
                import torch.distributed as dist

                comm.wait_stream(main)
                with torch.cuda.stream(comm):
                    dist.all_gather_into_tensor(kv[b], kv_src[rows], group=self.group)
                    ev = torch.cuda.Event()
                    ev.record(comm)
                landed.append(ev)
        if kv is None:
            kv = kv_src.view(batch, seq, 2 * d)
        att = torch.empty((batch * r, d), dtype=torch.bfloat16, device=dev)
        keep = None
        if text_mask is not None:
            keep = torch.ones((batch, seq), dtype=torch.bool, device=dev)
            keep[:, :text_len] = text_mask.reshape(batch, text_len).to(dev) > 0.5
        for b in range(batch):  # each sample's attention as soon as its keys and values are in
            if landed:
                main.wait_event(landed[b])
            rows = slice(b * r, (b + 1) * r)
            q = qkv[rows, :d].view(1, r, self.heads, HEAD_DIM).transpose(1, 2)
            k = kv[b:b + 1, :, :d].view(1, seq, self.heads, HEAD_DIM).transpose(1, 2)
            v = kv[b:b + 1, :, d:].view(1, seq, self.heads, HEAD_DIM).transpose(1, 2)
            mask = None if keep is None else keep[b].view(1, 1, 1, seq)
            o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, scale=1.0 / math.sqrt(HEAD_DIM))
            att[rows].copy_(o.transpose(1, 2).reshape(r, d))
        h = torch.empty_like(x_local)

        def out_proj(which: int) -> None:
            for b, stream, rows in segs:
                if stream == which:
                    name = "attn.to_add_out" if stream == 0 else "attn.attn_to_out.0"
                    full._linear(name, att[rows], residual=x_local[rows], gate=vec.gate1(b, stream), out=h[rows])

        both_streams(self, dev, lambda: out_proj(0), lambda: out_proj(1))
        z2 = torch.empty_like(x_local)
        modulate(h, vec.shift2, vec.scale2, z2)
        y = out if out is not None else torch.empty_like(x_local)

        def ff(which: int) -> None:
            for b, stream, rows in segs:
                if stream == which:
                    full._mlp("txt_ff" if stream == 0 else "img_ff", z2[rows], h[rows], vec.gate2(b, stream), y[rows],
                              slot=stream)

        both_streams(self, dev, lambda: ff(0), lambda: ff(1))
        return y

    def forward(self, hidden: torch.Tensor, encoder: torch.Tensor, temb: torch.Tensor,
                rope: tuple[torch.Tensor, ...],
                encoder_mask: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """Every rank passes the full inputs (as the reference block takes them)
        and gets the full (encoder_out, hidden_out): local rows in, one
        all-gather of the output rows at the end."""

        x, batch, s_txt = joint_rows(hidden, encoder)
        seq = x.shape[0] // batch
        y_local = self.forward_local(self.local_rows(x, batch, seq), temb, joint_rope(rope), batch, seq, s_txt,
                                     encoder_mask)
        if self.world == 1:
            y = y_local
        else:
            import torch.distributed as dist

            r = seq // self.world
            parts = torch.empty((self.world * batch * r, self.dim), dtype=y_local.dtype, device=y_local.device)
            dist.all_gather_into_tensor(parts, y_local, group=self.group)
            y = parts.view(self.world, batch, r, self.dim).transpose(0, 1).reshape(batch * seq, self.dim)
        return split_joint(y, batch, s_txt)


_SAMPLE_GROUPS: dict = {}


def sample_groups(world: int, rank: int, batch: int):
    """Split a batch of independent samples (the CFG cond / uncond pair run
    through the same blocks) over the ranks before splitting rows: with
    g = gcd(world, batch) groups, group i takes samples [i B / g, (i + 1) B / g)
    on ranks [i W / g, (i + 1) W / g), and a ContextParallelQwenBlock over the
    group's ranks splits those samples' rows.  Two GPUs then run one sample
    each with no communication; eight run each sample context-parallel over
    four.  Returns (sample slice, group size, rank in group, process group or
    None).  Every rank must call it with the same arguments (the groups are
    created collectively, once per (world, g))."""

    g = math.gcd(world, batch)
    size = world // g
    i = rank // size
    group = None
    if g > 1 and size > 1:
        import torch.distributed as dist

        key = (world, g)
        if key not in _SAMPLE_GROUPS:
            _SAMPLE_GROUPS[key] = [dist.new_group(list(range(j * size, (j + 1) * size))) for j in range(g)]
        group = _SAMPLE_GROUPS[key][i]
    per = batch // g
    return slice(i * per, (i + 1) * per), size, rank % size, group


def stack_modulations(blocks, temb: torch.Tensor, world: int = 1, rank: int = 0, group=None) -> torch.Tensor:
    """Modulation vectors [n, B, 2, 6, D] of every block of a stack for one
    timestep embedding, the work split over the ranks of a tensor-parallel
    group: rank r computes a contiguous run of ceil(n / world) blocks and one
    all-gather shares them.  The modulation linears read only silu(temb), so
    a denoising step can compute them all before its first block and each
    block then skips its replicated modulation GEMV."""

    n = len(blocks)
    per = -(-n // world)
    b = temb.shape[0]
    d = blocks[0].dim
    local = torch.zeros((per, b, 2, 6, d), dtype=torch.bfloat16, device=temb.device)
    for j in range(per):
        i = rank * per + j
        if i < n:
            local[j].copy_(blocks[i].modulation_joint(temb))
    if world == 1:
        return local[:n]
    import torch.distributed as dist

    everything = torch.empty((per * world, b, 2, 6, d), dtype=torch.bfloat16, device=temb.device)
    dist.all_gather_into_tensor(everything, local, group=group)
    return everything[:n]
