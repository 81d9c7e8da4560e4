"""LoRA adapters on the q6 linears: additive delta, multi-adapter fold, checkpoint keys.

Reference behaviour followed here:

* One adapter stays additive, ``y += s * ((x @ A) @ B)`` with A [in, r] and
  B [r, out] (shardedit_mlx/dense_img_ff_window.py:48-60, :93-118).
* Several adapters on one layer: the reference folds ``sum_i s_i (A_i @ B_i)``
  into the dense weight (:121-131, :134-153).  That fold stays available for
  dense weights (``lora_delta_weight``), but the q6 path cannot add a delta to
  packed codes, so ``fold_lora_adapters`` stacks the adapters into ONE fused
  delta of rank sum(r_i): A = [A_1 | A_2 | ...], B = [B'_1; B'_2; ...] with
  B'_i = bf16(s_i * B_i) and scale 1 (or the B_i unscaled and the common
  scale, when all scales agree).  The tensor-core kernel forms
  bf16(scale * B) for its MMA operand, so each adapter contributes exactly
  what a single-adapter call with (A_i, B_i, s_i) contributes, summed in the
  same fp32 accumulator as the q6 product.
* Checkpoint keys: ``plan_qwen_lora_keys`` / ``select_lora_keys`` index LoRA
  keys by transformer block (shardedit_mlx/lora_plan.py:8-87), and
  ``apply_lora_weights`` patches adapters onto the q6 layers of loaded blocks
  (the role of ``apply_window_loras``, shardedit_mlx/shard_runtime.py:247-300).
"""

from __future__ import annotations

from collections.abc import Iterable, Mapping, Sequence
from dataclasses import dataclass
import re

import torch

RANK_ALIGN = 32          # the fused delta's rank is padded to a multiple of this
MAX_FUSED_RANK = 256     # two LoRA stages of up to 128 rank columns each


@dataclass(frozen=True)
class LoRAAdapter:
    """One low-rank adapter: delta = scale * (x @ lora_A) @ lora_B."""

    lora_A: torch.Tensor  # [in_features, r]
    lora_B: torch.Tensor  # [r, out_features]
    scale: float = 1.0

    @property
    def rank(self) -> int:
        return int(self.lora_A.shape[-1])


def _check_adapter(ad: LoRAAdapter, in_features: int | None, out_features: int | None) -> tuple[int, int]:
    a, b = ad.lora_A, ad.lora_B
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0] or a.shape[1] == 0:
        raise ValueError(f"LoRA A must be (in, r) and B (r, out); got {tuple(a.shape)}, {tuple(b.shape)}")
    k, n = int(a.shape[0]), int(b.shape[1])
    if (in_features is not None and k != in_features) or (out_features is not None and n != out_features):
        raise ValueError(f"LoRA A must be ({in_features}, r) and B (r, {out_features}); "
                         f"got {tuple(a.shape)}, {tuple(b.shape)}")
    return k, n


def fold_lora_adapters(
    adapters: Sequence[LoRAAdapter],
    *,
    in_features: int | None = None,
    out_features: int | None = None,
) -> tuple[torch.Tensor, torch.Tensor, float] | None:
    """Stack adapters into one fused (A, B, scale) delta for the q6 kernel.

    Returns None for no adapters, the adapter itself (bf16) for one, and for
    several the rank-concatenated pair described in the module docstring.
    Raises ValueError when shapes disagree or the total rank exceeds
    MAX_FUSED_RANK (the q6 path has no second delta pass).
    """

    if not adapters:
        return None
    k = n = None
    for ad in adapters:
        k, n = _check_adapter(ad, in_features if k is None else k, out_features if n is None else n)
    total = sum(ad.rank for ad in adapters)
    if total > MAX_FUSED_RANK:
        raise ValueError(f"fused LoRA rank {total} exceeds {MAX_FUSED_RANK}; fold the adapters into dense "
                         "weights (lora_delta_weight) instead")
    if len(adapters) == 1:
        ad = adapters[0]
        return (ad.lora_A.to(torch.bfloat16).contiguous(), ad.lora_B.to(torch.bfloat16).contiguous(),
                float(ad.scale))
    dev = adapters[0].lora_A.device
    a = torch.cat([ad.lora_A.to(device=dev, dtype=torch.bfloat16) for ad in adapters], dim=1)
    scales = {float(ad.scale) for ad in adapters}
    if len(scales) == 1:
        b = torch.cat([ad.lora_B.to(device=dev, dtype=torch.bfloat16) for ad in adapters], dim=0)
        return a.contiguous(), b.contiguous(), scales.pop()
    # B'_i = bf16(fp32(s_i) * fp32(B_i)): the product the kernel forms for a
    # single adapter, so the kernel's own bf16(1 * B'_i) reproduces it exactly.
    parts = []
    for ad in adapters:
        s = torch.tensor(float(ad.scale), dtype=torch.float32, device=dev)
        parts.append((ad.lora_B.to(device=dev, dtype=torch.bfloat16).to(torch.float32) * s).to(torch.bfloat16))
    return a.contiguous(), torch.cat(parts, dim=0).contiguous(), 1.0


def pad_lora_rank(a: torch.Tensor, b: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Zero-pad A's columns and B's rows to a multiple of RANK_ALIGN.

    Exact: the padded rank columns of x @ A are zero and meet zero rows of B.
    """

    r = int(a.shape[1])
    rp = -(-r // RANK_ALIGN) * RANK_ALIGN
    if rp == r:
        return a, b
    a_p = torch.zeros((a.shape[0], rp), dtype=a.dtype, device=a.device)
    a_p[:, :r] = a
    b_p = torch.zeros((rp, b.shape[1]), dtype=b.dtype, device=b.device)
    b_p[:r] = b
    return a_p, b_p


def lora_delta_weight(adapters: Sequence[LoRAAdapter], *, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor | None:
    """Dense fold ``sum_i s_i (A_i @ B_i)`` in [out, in] layout (fp32 sums,
    cast once), the reference's multi-adapter fuse for dense weights
    (shardedit_mlx/dense_img_ff_window.py:121-131).  None without adapters."""

    if not adapters:
        return None
    delta = None
    for ad in adapters:
        piece = float(ad.scale) * (ad.lora_A.to(torch.float32) @ ad.lora_B.to(torch.float32))
        delta = piece if delta is None else delta + piece
    return delta.T.contiguous().to(dtype)


# --- checkpoint key plan (shardedit_mlx/lora_plan.py) ------------------------------------------

_BLOCK_PATTERNS = (
    re.compile(r"(?:^|\.)transformer_blocks\.(\d+)\."),
    re.compile(r"(?:^|_)transformer_blocks_(\d+)_"),
)


@dataclass(frozen=True)
class LoRAKeyPlan:
    block_count: int
    keys_by_block: tuple[tuple[str, ...], ...]
    key_count: int


def lora_key_block_index(key: str) -> int | None:
    """Transformer block a LoRA key belongs to, in dotted or underscored form."""

    for pattern in _BLOCK_PATTERNS:
        m = pattern.search(key)
        if m:
            return int(m.group(1))
    return None


def plan_qwen_lora_keys(keys: tuple[str, ...], *, block_count: int = 60) -> LoRAKeyPlan:
    """Index LoRA keys by block without loading tensors (lora_plan.py:31-72)."""

    if block_count <= 0:
        raise ValueError("block_count must be positive")
    if not keys:
        raise ValueError("LoRA keys cannot be empty")
    if len(set(keys)) != len(keys):
        raise ValueError("LoRA keys must be unique")
    indexed = [(key, lora_key_block_index(key)) for key in keys]
    unknown = tuple(key for key, i in indexed if i is None)
    if unknown:
        raise ValueError(f"LoRA keys without a Transformer block index: {unknown[:5]}")
    outside = tuple(key for key, i in indexed if not 0 <= i < block_count)
    if outside:
        raise ValueError(f"LoRA keys outside the model block range: {outside[:5]}")
    by_block: list[list[str]] = [[] for _ in range(block_count)]
    for key, i in indexed:
        by_block[i].append(key)
    return LoRAKeyPlan(block_count=block_count, keys_by_block=tuple(tuple(sorted(b)) for b in by_block),
                       key_count=len(keys))


def select_lora_keys(plan: LoRAKeyPlan, block_indices: tuple[int, ...]) -> tuple[str, ...]:
    """Keys of the selected blocks, block order then key order (lora_plan.py:75-87)."""

    if any(i < 0 or i >= plan.block_count for i in block_indices):
        raise ValueError("block index is outside the LoRA plan")
    if len(set(block_indices)) != len(block_indices):
        raise ValueError("block indices must be unique")
    return tuple(key for i in block_indices for key in plan.keys_by_block[i])


# --- checkpoint adapters onto q6 layers ---------------------------------------------------------

# (suffix, role): PEFT ``lora_A``/``lora_B`` and kohya ``lora_down``/``lora_up``
# (also ``lora.down``/``lora.up``) store torch-Linear layouts: down/A is
# [r, in], up/B is [out, r].  ``alpha`` rescales by alpha / r.
_SUFFIXES = (
    (".lora_A.weight", "down"), (".lora_B.weight", "up"),
    (".lora_down.weight", "down"), (".lora_up.weight", "up"),
    (".lora.down.weight", "down"), (".lora.up.weight", "up"),
    (".alpha", "alpha"),
)
_PREFIXES = ("transformer.", "diffusion_model.", "base_model.model.", "lora_unet_", "lora_transformer_")

# diffusers QwenImageTransformerBlock module names -> the q6 block's layer names
LAYER_ALIASES = {
    "img_mlp.net.0.proj": "img_ff.mlp_in",
    "img_mlp.net.2": "img_ff.mlp_out",
    "txt_mlp.net.0.proj": "txt_ff.mlp_in",
    "txt_mlp.net.2": "txt_ff.mlp_out",
    "attn.to_out.0": "attn.attn_to_out.0",
    "img_mod.1": "img_mod_linear",
    "txt_mod.1": "txt_mod_linear",
}


def _split_lora_key(key: str) -> tuple[str, str] | None:
    for suffix, role in _SUFFIXES:
        if key.endswith(suffix):
            path = key[: -len(suffix)]
            for prefix in _PREFIXES:
                if path.startswith(prefix):
                    path = path[len(prefix):]
                    break
            return path, role
    return None


def _resolve_layer(path: str, layers: Mapping[str, object], underscored: Mapping[str, str]) -> str | None:
    if path in layers:
        return path
    m = re.match(r"(transformer_blocks\.\d+\.)(.*)$", path)
    if m and m.group(2) in LAYER_ALIASES:
        alias = m.group(1) + LAYER_ALIASES[m.group(2)]
        if alias in layers:
            return alias
    flat = path.replace(".", "_")
    if flat in underscored:
        return underscored[flat]
    return None


def apply_lora_weights(
    layers: Mapping[str, object],
    weights: Mapping[str, torch.Tensor],
    scale: float = 1.0,
) -> tuple[int, set[str]]:
    """Attach one LoRA checkpoint's adapters to q6 layers (additively, so a
    second checkpoint adds a second adapter that the fold stacks).

    ``layers`` maps full layer names (``transformer_blocks.3.img_ff.mlp_in``)
    to modules with ``add_lora`` and ``in_features``/``out_features``;
    ``weights`` maps checkpoint keys to tensors.  Returns (layers patched,
    keys matched).  Raises ValueError when a layer has only one of its
    down/up pair or its shapes do not fit the layer, like the reference's
    window patcher refuses partial matches (shard_runtime.py:279-288).
    """

    underscored = {}
    for name in layers:
        underscored[name.replace(".", "_")] = name
        m = re.match(r"(transformer_blocks\.\d+\.)(.*)$", name)
        if m:
            for src, dst in LAYER_ALIASES.items():
                if dst == m.group(2):
                    underscored[(m.group(1) + src).replace(".", "_")] = name
    pending: dict[str, dict[str, tuple[str, torch.Tensor]]] = {}
    for key, value in weights.items():
        split = _split_lora_key(key)
        if split is None:
            continue
        path, role = split
        layer = _resolve_layer(path, layers, underscored)
        if layer is None:
            continue
        pending.setdefault(layer, {})[role] = (key, value)
    matched: set[str] = set()
    applied = 0
    for name in sorted(pending):
        parts = pending[name]
        if "down" not in parts or "up" not in parts:
            raise ValueError(f"LoRA for {name} needs both its down (A) and up (B) weights")
        down = parts["down"][1]
        up = parts["up"][1]
        layer = layers[name]
        r = int(down.shape[0])
        if down.dim() != 2 or up.dim() != 2 or int(up.shape[1]) != r:
            raise ValueError(f"LoRA for {name}: down {tuple(down.shape)} and up {tuple(up.shape)} do not pair")
        s = float(scale)
        if "alpha" in parts:
            s *= float(parts["alpha"][1].reshape(-1)[0]) / r
        dev = layer.weight.device
        a = down.to(device=dev, dtype=torch.bfloat16).T.contiguous()  # [in, r]
        b = up.to(device=dev, dtype=torch.bfloat16).T.contiguous()    # [r, out]
        layer.add_lora(a, b, s)
        applied += 1
        matched.update(k for k, _ in parts.values())
    return applied, matched


def iter_adapters(layer: object) -> Iterable[LoRAAdapter]:
    """The adapters attached to a layer: a ``loras`` list, or one
    ``lora_A``/``lora_B``/``scale`` triple (mflux-style LoRA linears)."""

    loras = getattr(layer, "loras", None)
    if loras:
        for ad in loras:
            yield ad if isinstance(ad, LoRAAdapter) else LoRAAdapter(ad.lora_A, ad.lora_B,
                                                                     float(getattr(ad, "scale", 1.0)))
    elif hasattr(layer, "lora_A") and hasattr(layer, "lora_B"):
        yield LoRAAdapter(layer.lora_A, layer.lora_B, float(getattr(layer, "scale", 1.0)))
