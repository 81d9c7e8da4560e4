"""CPU oracle (test infrastructure only) for the Qwen-Image MMDiT block around the q6 linears.

Restates the block's stages as the reference profiles them
(benchmarks/profile_qwen_block.py:163-301), in float64 with a bf16 rounding
at every point where the GPU path stores bf16:

* modulation  - ``img_mod_linear(silu(temb))``, split into (shift, scale,
  gate) x 2 (:163-172);
* adaLN       - ``_modulate(LayerNorm(x), mod)``: LayerNorm without affine
  parameters (eps 1e-6), ``x * (1 + scale) + shift`` (:174-181, :262-263);
* attention   - q/k/v projections per stream, RMSNorm over each head
  (``norm_q`` / ``norm_k`` / ``norm_added_q`` / ``norm_added_k``), rotary
  embedding, joint [text; image] softmax attention (:183-240), output
  projections (:242-251);
* residuals   - ``x + gate1 * attn_out`` and ``x + gate2 * ff(x')`` (:253-301).

The rotary embedding acts on interleaved pairs (x[2i], x[2i+1]) with
per-token angles, the complex form of the published Qwen-Image rotary scheme;
``qwen_rope_angles`` restates its table: three axes (frame, height, width) of
16 / 56 / 56 dimensions, base 10000, image positions centred on the patch
grid, text positions continuing after the largest image position.  mflux's
own tables (the reference's ``image_rotary_emb``) are not vendored here, so
the table itself is parity unpinned; the block computations take the tables
as inputs and are checked with the same tables on both sides.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from oracle.oracle import Q6Weights, bf16_bits_to_f32, gelu, linear, round_bf16


def silu(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float64)
    return (x / (1.0 + np.exp(-x))).astype(np.float32)


def layernorm_modulate(x: np.ndarray, shift: np.ndarray, scale: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """LayerNorm over the last axis (no affine), then ``* (1 + scale) + shift``; fp32 result."""

    x = np.asarray(x, dtype=np.float64)
    mu = x.mean(axis=-1, keepdims=True)
    var = ((x - mu) ** 2).mean(axis=-1, keepdims=True)
    n = (x - mu) / np.sqrt(var + eps)
    return (n * (1.0 + np.asarray(scale, dtype=np.float64)) + np.asarray(shift, dtype=np.float64)).astype(np.float32)


def rmsnorm_heads(x: np.ndarray, weight: np.ndarray, head_dim: int = 128, eps: float = 1e-6) -> np.ndarray:
    """RMSNorm over each head of ``head_dim`` values of rows [M, H * head_dim]."""

    x = np.asarray(x, dtype=np.float64)
    m = x.shape[0]
    h = x.reshape(m, -1, head_dim)
    r = 1.0 / np.sqrt((h * h).mean(axis=-1, keepdims=True) + eps)
    return (h * r * np.asarray(weight, dtype=np.float64)).reshape(m, -1)


def rope_pairs(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, head_dim: int = 128) -> np.ndarray:
    """Rotate interleaved pairs of every head by per-row angles (cos/sin [M, head_dim / 2])."""

    x = np.asarray(x, dtype=np.float64)
    m = x.shape[0]
    h = x.reshape(m, -1, head_dim // 2, 2)
    c = np.asarray(cos, dtype=np.float64)[:, None, :]
    s = np.asarray(sin, dtype=np.float64)[:, None, :]
    a, b = h[..., 0], h[..., 1]
    out = np.stack([a * c - b * s, a * s + b * c], axis=-1)
    return out.reshape(m, -1)


def qk_rmsnorm_rope(x: np.ndarray, weight: np.ndarray, cos: np.ndarray, sin: np.ndarray,
                    eps: float = 1e-6) -> np.ndarray:
    return rope_pairs(rmsnorm_heads(x, weight, 128, eps), cos, sin).astype(np.float32)


def _axis_freqs(dim: int, theta: float) -> np.ndarray:
    return 1.0 / theta ** (np.arange(0, dim, 2, dtype=np.float64) / dim)


def qwen_rope_angles(img_shapes: list[tuple[int, int]], txt_len: int, *, theta: float = 10000.0,
                     axes: tuple[int, int, int] = (16, 56, 56)) -> tuple[np.ndarray, np.ndarray]:
    """Angles [S_img, 64] and [S_txt, 64] (radians) for images of (h, w)
    patches, frame index = image index, followed by ``txt_len`` text tokens."""

    fr, fh, fw = (_axis_freqs(a, theta) for a in axes)
    rows = []
    max_pos = 0
    for f, (h, w) in enumerate(img_shapes):
        hp = np.arange(h) - h // 2
        wp = np.arange(w) - w // 2
        hh, ww = np.meshgrid(hp, wp, indexing="ij")
        ang = np.concatenate([
            np.broadcast_to(f * fr, (h * w, fr.size)),
            hh.reshape(-1, 1) * fh,
            ww.reshape(-1, 1) * fw,
        ], axis=1)
        rows.append(ang)
        max_pos = max(max_pos, h // 2, w // 2)
    img = np.concatenate(rows, axis=0)
    tp = (max_pos + np.arange(txt_len, dtype=np.float64)).reshape(-1, 1)
    txt = np.concatenate([tp * fr, tp * fh, tp * fw], axis=1)
    return img, txt


def joint_key_mask(text_mask: np.ndarray | None, s_img: int) -> np.ndarray | None:
    """Keys a joint [text; image] query may attend to, from the encoder's text
    mask [S_txt] (1 = real token, 0 = padding): padded text tokens are masked
    out as keys, every image token stays (the reference converts its
    ``encoder_hidden_states_mask`` this way before SDPA,
    benchmarks/profile_qwen_block.py:228-248)."""

    if text_mask is None:
        return None
    return np.concatenate([np.asarray(text_mask).reshape(-1) > 0.5, np.ones(s_img, dtype=bool)])


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, heads: int,
              key_mask: np.ndarray | None = None) -> np.ndarray:
    """softmax(q k^T / sqrt(d)) v per head; rows [S, H * d]; ``key_mask``
    [S_k] bool drops the keys it marks False."""

    s = q.shape[0]
    d = q.shape[1] // heads
    qh = np.asarray(q, dtype=np.float64).reshape(s, heads, d).transpose(1, 0, 2)
    kh = np.asarray(k, dtype=np.float64).reshape(-1, heads, d).transpose(1, 0, 2)
    vh = np.asarray(v, dtype=np.float64).reshape(-1, heads, d).transpose(1, 0, 2)
    logits = qh @ kh.transpose(0, 2, 1) / np.sqrt(d)
    if key_mask is not None:
        logits = np.where(np.asarray(key_mask, dtype=bool)[None, None, :], logits, -np.inf)
    logits -= logits.max(axis=-1, keepdims=True)
    p = np.exp(logits)
    p /= p.sum(axis=-1, keepdims=True)
    return (p @ vh).transpose(1, 0, 2).reshape(s, heads * d)


@dataclass
class BlockWeights:
    """One block's q6 linears (by the reference's layer names) and norm weights (fp32 values)."""

    linears: dict[str, Q6Weights]
    norms: dict[str, np.ndarray]  # attn.norm_q / norm_k / norm_added_q / norm_added_k, [128]
    heads: int


def kernel_weight_dtype(rows: int, n: int, k: int, group_size: int) -> str:
    """Weight precision of the library kernel that runs a linear launch of
    ``rows`` token rows on an n x k weight: fp32 dequantised weights on the
    few-row kernels (the streaming GEMV for 1-2 rows; the warp-MMA kernel for
    2-16 rows when the weight holds at least 2^24 codes, K is a multiple of
    512 and, at group size 32, for at most 8 rows), bf16 on the tensor-core
    path (MLX qmm semantics).  Mirrors the library's auto-path policy."""

    if rows <= 2:
        return "f32"
    warp_mma = (rows <= 16 and n * k >= 1 << 24 and k % 512 == 0 and (k // group_size) % 8 == 0
                and (group_size != 32 or rows <= 8))
    return "f32" if warp_mma else "bf16"


def _lin(w: BlockWeights, name: str, x: np.ndarray, *, launch_rows: int | None = None, **kw) -> np.ndarray:
    """One q6 linear with the weight precision of the kernel path that runs it
    for ``launch_rows`` token rows (default: the rows of ``x``;
    kernel_weight_dtype): the modulation linears at M = batch run on the
    few-row kernels, which keep the reference kernel's fp32
    ``scale * code + qbias``.  ``x`` may hold a subset of the launch's rows."""

    rows = np.asarray(x).shape[0] if launch_rows is None else launch_rows
    lin = w.linears[name]
    kw.setdefault("weight_dtype", kernel_weight_dtype(rows, lin.out_features, lin.in_features, lin.group_size))
    return round_bf16(linear(x, w.linears[name], **kw))


def block_forward(w: BlockWeights, hidden: np.ndarray, encoder: np.ndarray, temb: np.ndarray,
                  img_cos: np.ndarray, img_sin: np.ndarray, txt_cos: np.ndarray, txt_sin: np.ndarray,
                  eps: float = 1e-6, text_mask: np.ndarray | None = None) -> tuple[np.ndarray, np.ndarray]:
    """One sample through the block: returns (text stream out, image stream out), fp32 values of bf16.

    ``hidden`` [S_img, D], ``encoder`` [S_txt, D], ``temb`` [D] hold the
    values of bf16 inputs; ``text_mask`` [S_txt] (optional) marks real text
    tokens with 1 and padding with 0.
    """

    return block_forward_rows(w, hidden, encoder, temb, img_cos, img_sin, txt_cos, txt_sin, eps=eps,
                              text_mask=text_mask)


def block_forward_rows(w: BlockWeights, hidden: np.ndarray, encoder: np.ndarray, temb: np.ndarray,
                       img_cos: np.ndarray, img_sin: np.ndarray, txt_cos: np.ndarray, txt_sin: np.ndarray,
                       eps: float = 1e-6, text_mask: np.ndarray | None = None,
                       img_rows: np.ndarray | None = None,
                       txt_rows: np.ndarray | None = None) -> tuple[np.ndarray, np.ndarray]:
    """``block_forward`` restricted to the output rows ``txt_rows`` /
    ``img_rows`` (all rows when None).  Keys and values still come from every
    row; only the query side (attention output, output projections, feed
    forward) is computed for the selected rows, each of which depends on its
    own input row and on all keys and values.  Returns the selected rows."""

    d = hidden.shape[1]
    s_txt, s_img = encoder.shape[0], hidden.shape[0]
    ir = np.arange(s_img) if img_rows is None else np.asarray(img_rows)
    tr = np.arange(s_txt) if txt_rows is None else np.asarray(txt_rows)
    t = round_bf16(silu(temb).reshape(1, d))
    img_mod = _lin(w, "img_mod_linear", t).reshape(6, d)
    txt_mod = _lin(w, "txt_mod_linear", t).reshape(6, d)
    ish1, isc1, ig1, ish2, isc2, ig2 = img_mod
    tsh1, tsc1, tg1, tsh2, tsc2, tg2 = txt_mod

    img_in = round_bf16(layernorm_modulate(hidden, ish1, isc1, eps))
    txt_in = round_bf16(layernorm_modulate(encoder, tsh1, tsc1, eps))
    # keys and values of every row
    k_i = round_bf16(qk_rmsnorm_rope(_lin(w, "attn.to_k", img_in), w.norms["attn.norm_k"], img_cos, img_sin, eps))
    k_t = round_bf16(qk_rmsnorm_rope(_lin(w, "attn.add_k_proj", txt_in), w.norms["attn.norm_added_k"], txt_cos,
                                     txt_sin, eps))
    v_i = _lin(w, "attn.to_v", img_in)
    v_t = _lin(w, "attn.add_v_proj", txt_in)
    # queries of the selected rows only
    q_i = round_bf16(qk_rmsnorm_rope(_lin(w, "attn.to_q", img_in[ir], launch_rows=s_img), w.norms["attn.norm_q"], img_cos[ir],
                                     img_sin[ir], eps))
    q_t = round_bf16(qk_rmsnorm_rope(_lin(w, "attn.add_q_proj", txt_in[tr], launch_rows=s_txt), w.norms["attn.norm_added_q"],
                                     txt_cos[tr], txt_sin[tr], eps))
    key_mask = joint_key_mask(text_mask, s_img)
    keys, vals = np.concatenate([k_t, k_i]), np.concatenate([v_t, v_i])
    att_t = round_bf16(attention(q_t, keys, vals, w.heads, key_mask).astype(np.float32))
    att_i = round_bf16(attention(q_i, keys, vals, w.heads, key_mask).astype(np.float32))
    img_h = _lin(w, "attn.attn_to_out.0", att_i, residual=hidden[ir], gate=ig1, launch_rows=s_img)
    txt_h = _lin(w, "attn.to_add_out", att_t, residual=encoder[tr], gate=tg1, launch_rows=s_txt)

    img_ff_in = round_bf16(layernorm_modulate(img_h, ish2, isc2, eps))
    txt_ff_in = round_bf16(layernorm_modulate(txt_h, tsh2, tsc2, eps))
    img_mid = _lin(w, "img_ff.mlp_in", img_ff_in, apply_gelu=True, launch_rows=s_img)
    txt_mid = _lin(w, "txt_ff.mlp_in", txt_ff_in, apply_gelu=True, launch_rows=s_txt)
    img_out = _lin(w, "img_ff.mlp_out", img_mid, residual=img_h, gate=ig2, launch_rows=s_img)
    txt_out = _lin(w, "txt_ff.mlp_out", txt_mid, residual=txt_h, gate=tg2, launch_rows=s_txt)
    return txt_out, img_out


def _block_forward_full(w: BlockWeights, hidden: np.ndarray, encoder: np.ndarray, temb: np.ndarray,
                        img_cos: np.ndarray, img_sin: np.ndarray, txt_cos: np.ndarray, txt_sin: np.ndarray,
                        eps: float = 1e-6) -> tuple[np.ndarray, np.ndarray]:
    """The whole-sequence form of the block (every row through every stage),
    kept as the plain statement of the stage order that block_forward_rows
    restricts to selected rows."""

    d = hidden.shape[1]
    t = round_bf16(silu(temb).reshape(1, d))
    img_mod = _lin(w, "img_mod_linear", t).reshape(6, d)
    txt_mod = _lin(w, "txt_mod_linear", t).reshape(6, d)
    # (shift, scale, gate) for the attention half, then for the MLP half
    ish1, isc1, ig1, ish2, isc2, ig2 = img_mod
    tsh1, tsc1, tg1, tsh2, tsc2, tg2 = txt_mod

    img_in = round_bf16(layernorm_modulate(hidden, ish1, isc1, eps))
    txt_in = round_bf16(layernorm_modulate(encoder, tsh1, tsc1, eps))
    q_i, k_i, v_i = (_lin(w, f"attn.{n}", img_in) for n in ("to_q", "to_k", "to_v"))
    q_t, k_t, v_t = (_lin(w, f"attn.{n}", txt_in) for n in ("add_q_proj", "add_k_proj", "add_v_proj"))
    q_i = round_bf16(qk_rmsnorm_rope(q_i, w.norms["attn.norm_q"], img_cos, img_sin, eps))
    k_i = round_bf16(qk_rmsnorm_rope(k_i, w.norms["attn.norm_k"], img_cos, img_sin, eps))
    q_t = round_bf16(qk_rmsnorm_rope(q_t, w.norms["attn.norm_added_q"], txt_cos, txt_sin, eps))
    k_t = round_bf16(qk_rmsnorm_rope(k_t, w.norms["attn.norm_added_k"], txt_cos, txt_sin, eps))
    s_txt = encoder.shape[0]
    joint = round_bf16(attention(np.concatenate([q_t, q_i]), np.concatenate([k_t, k_i]),
                                 np.concatenate([v_t, v_i]), w.heads).astype(np.float32))
    img_h = _lin(w, "attn.attn_to_out.0", joint[s_txt:], residual=hidden, gate=ig1)
    txt_h = _lin(w, "attn.to_add_out", joint[:s_txt], residual=encoder, gate=tg1)

    img_ff_in = round_bf16(layernorm_modulate(img_h, ish2, isc2, eps))
    txt_ff_in = round_bf16(layernorm_modulate(txt_h, tsh2, tsc2, eps))
    img_mid = _lin(w, "img_ff.mlp_in", img_ff_in, apply_gelu=True)
    txt_mid = _lin(w, "txt_ff.mlp_in", txt_ff_in, apply_gelu=True)
    img_out = _lin(w, "img_ff.mlp_out", img_mid, residual=img_h, gate=ig2)
    txt_out = _lin(w, "txt_ff.mlp_out", txt_mid, residual=txt_h, gate=tg2)
    return txt_out, img_out


BLOCK_LINEARS = {
    # name: (out_features factor of D, in_features factor of D); D = hidden size, FF hidden = 4 D
    "img_mod_linear": (6, 1), "txt_mod_linear": (6, 1),
    "attn.to_q": (1, 1), "attn.to_k": (1, 1), "attn.to_v": (1, 1),
    "attn.add_q_proj": (1, 1), "attn.add_k_proj": (1, 1), "attn.add_v_proj": (1, 1),
    "attn.attn_to_out.0": (1, 1), "attn.to_add_out": (1, 1),
    "img_ff.mlp_in": (4, 1), "img_ff.mlp_out": (1, 4),
    "txt_ff.mlp_in": (4, 1), "txt_ff.mlp_out": (1, 4),
}
NORMS = ("attn.norm_q", "attn.norm_k", "attn.norm_added_q", "attn.norm_added_k")

__all__ = [
    "BLOCK_LINEARS", "NORMS", "BlockWeights", "attention", "block_forward", "block_forward_rows", "gelu",
    "joint_key_mask", "layernorm_modulate",
    "qk_rmsnorm_rope", "qwen_rope_angles", "rmsnorm_heads", "rope_pairs", "silu", "bf16_bits_to_f32",
]
