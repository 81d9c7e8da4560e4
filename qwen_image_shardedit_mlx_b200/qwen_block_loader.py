"""q6 Qwen transformer checkpoint loading: safetensors shards -> device-resident q6 layers.

Mirrors the reference's loader surface:

* ``plan_transformer_block_shards(weight_map, block_count=60)`` - which shard
  files hold each ``transformer_blocks.<i>.`` tensor (shardedit_mlx/sweep_profile.py:10-47);
* ``load_transformer_layout(model_dir)`` - reads
  ``transformer/model.safetensors.index.json`` and checks every shard exists
  (shardedit_mlx/qwen_block_loader.py:34-62);
* ``load_block_window(layout, block_indices)`` - consecutive blocks, each
  returned as ``LoadedBlock(block_index, module)`` (qwen_block_loader.py:105-157).

The block module here holds the q6 layers as ``QuantizedLinear`` (MLX tensor
names: ``<layer>.weight`` packed uint32, ``.scales``, ``.biases``, optional
``.bias``; benchmark_qwen_block.py:88-112) resident in device memory, plus the
block's other tensors (norms) by name, and exposes ``img_ff`` / ``txt_ff`` as
``QwenFeedForward`` when present.  Unlike the reference, which loads whole
shards and filters (qwen_block_loader.py:78-102), only the selected tensors'
bytes are read, straight from their file offsets.

The safetensors container (8-byte little-endian header length, JSON header of
``{name: {dtype, shape, data_offsets}}``, then the raw little-endian bytes) is
read and written here without third-party code.
"""

from __future__ import annotations

from collections.abc import Iterable, Mapping
from dataclasses import dataclass, field
import json
from pathlib import Path
import struct

import torch

from qwen_image_shardedit_mlx_b200.q6_metal_mlp import QuantizedLinear, QwenFeedForward

_DTYPES = {
    "BOOL": torch.bool, "U8": torch.uint8, "I8": torch.int8, "I16": torch.int16, "U16": torch.uint16,
    "F16": torch.float16, "BF16": torch.bfloat16, "I32": torch.int32, "U32": torch.uint32,
    "F32": torch.float32, "F64": torch.float64, "I64": torch.int64, "U64": torch.uint64,
}
_NAMES = {v: k for k, v in _DTYPES.items()}
_MAX_HEADER = 100 * 1024 * 1024


# --- safetensors container ---------------------------------------------------------------------

@dataclass(frozen=True)
class TensorEntry:
    dtype: str
    shape: tuple[int, ...]
    begin: int   # absolute file offset of the first byte
    nbytes: int


def read_safetensors_header(path: str | Path) -> tuple[dict[str, TensorEntry], dict[str, str]]:
    """Parse a safetensors header: (entries by name, metadata)."""

    path = Path(path)
    size = path.stat().st_size
    with path.open("rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise ValueError(f"{path}: not a safetensors file (short header)")
        (hlen,) = struct.unpack("<Q", raw)
        if hlen > _MAX_HEADER or 8 + hlen > size:
            raise ValueError(f"{path}: header length {hlen} is invalid")
        header = json.loads(f.read(hlen).decode("utf-8"))
    if not isinstance(header, dict):
        raise ValueError(f"{path}: header is not a JSON object")
    meta = header.pop("__metadata__", {}) or {}
    base = 8 + hlen
    entries: dict[str, TensorEntry] = {}
    for name, info in header.items():
        try:
            dtype, shape, (b, e) = info["dtype"], tuple(int(d) for d in info["shape"]), info["data_offsets"]
        except (KeyError, TypeError, ValueError) as exc:
            raise ValueError(f"{path}: malformed entry for {name!r}") from exc
        if dtype not in _DTYPES:
            raise ValueError(f"{path}: unsupported dtype {dtype} for {name!r}")
        count = 1
        for d in shape:
            count *= d
        nbytes = count * torch.empty((), dtype=_DTYPES[dtype]).element_size()
        if e - b != nbytes or b < 0 or base + e > size:
            raise ValueError(f"{path}: data_offsets of {name!r} do not match its shape and dtype")
        entries[name] = TensorEntry(dtype, shape, base + b, nbytes)
    return entries, dict(meta)


def load_safetensors(path: str | Path, names: Iterable[str] | None = None, *,
                     device: torch.device | str = "cpu") -> dict[str, torch.Tensor]:
    """Read the named tensors (all when ``names`` is None) from one file.

    For a CUDA ``device`` each tensor is read into pinned host memory and
    copied asynchronously; the function synchronises once before returning.
    """

    path = Path(path)
    entries, _ = read_safetensors_header(path)
    wanted = list(entries) if names is None else list(names)
    missing = [n for n in wanted if n not in entries]
    if missing:
        raise KeyError(f"{path}: missing tensors {missing[:5]}")
    dev = torch.device(device)
    pin = dev.type == "cuda"
    out: dict[str, torch.Tensor] = {}
    with path.open("rb", buffering=0) as f:
        for name in sorted(wanted, key=lambda n: entries[n].begin):
            e = entries[name]
            buf = torch.empty(e.nbytes, dtype=torch.uint8, pin_memory=pin)
            if e.nbytes:
                f.seek(e.begin)
                got = f.readinto(memoryview(buf.numpy()))
                if got != e.nbytes:
                    raise ValueError(f"{path}: short read for {name!r}")
            raw = buf.to(dev, non_blocking=True) if pin else buf  # bytes travel; the view is free
            out[name] = raw.view(_DTYPES[e.dtype]).reshape(e.shape)
    if pin:
        torch.cuda.synchronize(dev)
    return out


def save_safetensors(path: str | Path, tensors: Mapping[str, torch.Tensor],
                     metadata: Mapping[str, str] | None = None) -> None:
    """Write tensors (any device; copied to host) as one safetensors file."""

    header: dict[str, object] = {}
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    blobs = []
    offset = 0
    for name in sorted(tensors):
        t = tensors[name]
        if t.dtype not in _NAMES:
            raise ValueError(f"unsupported dtype {t.dtype} for {name!r}")
        host = t.detach().to("cpu").contiguous()
        raw = host.reshape(-1).view(torch.uint8).numpy().tobytes() if host.numel() else b""
        header[name] = {"dtype": _NAMES[t.dtype], "shape": list(host.shape),
                        "data_offsets": [offset, offset + len(raw)]}
        blobs.append(raw)
        offset += len(raw)
    text = json.dumps(header, separators=(",", ":")).encode("utf-8")
    text += b" " * (-len(text) % 8)
    with Path(path).open("wb") as f:
        f.write(struct.pack("<Q", len(text)))
        f.write(text)
        for raw in blobs:
            f.write(raw)


# --- shard plans (shardedit_mlx/sweep_profile.py) ----------------------------------------------

@dataclass(frozen=True)
class BlockShardPlan:
    block_index: int
    tensor_count: int
    shards: tuple[str, ...]


def plan_transformer_block_shards(weight_map: Mapping[str, str], *,
                                  block_count: int = 60) -> tuple[BlockShardPlan, ...]:
    """Describe which safetensors shards own every transformer block."""

    if block_count <= 0:
        raise ValueError("block_count must be positive")
    if not weight_map:
        raise ValueError("weight_map cannot be empty")
    by_block: dict[int, list[str]] = {}
    for name, shard in weight_map.items():
        for i in range(block_count):
            if name.startswith(f"transformer_blocks.{i}."):
                by_block.setdefault(i, []).append(shard)
                break
    missing = tuple(i for i in range(block_count) if i not in by_block)
    if missing:
        raise ValueError(f"weight_map is missing Transformer blocks: {missing}")
    return tuple(BlockShardPlan(block_index=i, tensor_count=len(by_block[i]), shards=tuple(sorted(set(by_block[i]))))
                 for i in range(block_count))


@dataclass(frozen=True)
class TransformerLayout:
    transformer_dir: Path
    plans: tuple[BlockShardPlan, ...]
    ordered_shards: tuple[str, ...]
    weight_map: Mapping[str, str] = field(default_factory=dict, compare=False, repr=False)


def load_transformer_layout(model_dir: str | Path, *, block_count: int = 60) -> TransformerLayout:
    transformer_dir = Path(model_dir) / "transformer"
    index_path = transformer_dir / "model.safetensors.index.json"
    if not index_path.exists():
        raise FileNotFoundError(f"missing Transformer index: {index_path}")
    payload = json.loads(index_path.read_text(encoding="utf-8"))
    weight_map = payload.get("weight_map") if isinstance(payload, dict) else None
    if not isinstance(weight_map, dict) or not all(
            isinstance(k, str) and isinstance(v, str) for k, v in weight_map.items()):
        raise ValueError(f"invalid weight_map in {index_path}")
    plans = plan_transformer_block_shards(weight_map, block_count=block_count)
    ordered = tuple(dict.fromkeys(s for plan in plans for s in plan.shards))
    missing = tuple(s for s in ordered if not (transformer_dir / s).is_file())
    if missing:
        raise FileNotFoundError(f"missing Transformer shards: {missing}")
    return TransformerLayout(transformer_dir=transformer_dir, plans=plans, ordered_shards=ordered,
                             weight_map=dict(weight_map))


# --- blocks ------------------------------------------------------------------------------------

class QwenBlockWeights:
    """One transformer block's weights, device resident.

    ``linears`` maps layer names (``attn.to_q``, ``img_ff.mlp_in``, ...) to
    ``QuantizedLinear``; ``tensors`` holds every other tensor by its name.
    ``img_ff`` / ``txt_ff`` are ``QwenFeedForward`` modules over the same
    layers when both their linears are present.
    """

    def __init__(self, linears: dict[str, QuantizedLinear], tensors: dict[str, torch.Tensor]) -> None:
        self.linears = linears
        self.tensors = tensors
        for ff in ("img_ff", "txt_ff"):
            if f"{ff}.mlp_in" in linears and f"{ff}.mlp_out" in linears:
                setattr(self, ff, QwenFeedForward(linears[f"{ff}.mlp_in"], linears[f"{ff}.mlp_out"]))

    def nbytes(self) -> int:
        total = 0
        for lin in self.linears.values():
            for t in (lin.weight, lin.scales, lin.biases, lin.bias):
                if t is not None:
                    total += t.numel() * t.element_size()
        return total + sum(t.numel() * t.element_size() for t in self.tensors.values())


@dataclass(frozen=True)
class LoadedBlock:
    block_index: int
    module: QwenBlockWeights


def build_block(flat: Mapping[str, torch.Tensor], *, bits: int = 6,
                group_size: int | None = None) -> QwenBlockWeights:
    """Group a block's flat tensors into q6 layers and plain tensors.

    A layer is every ``<name>.weight`` stored as uint32 with a ``.scales``
    sibling; its group size follows from the shapes (in_features =
    weight columns * 32 / bits, divided by the scale columns) and must be
    one of 32 / 64 / 128 (or equal ``group_size`` when given).
    """

    if bits != 6:
        raise ValueError(f"only bits=6 is supported, got {bits}")
    used: set[str] = set()
    linears: dict[str, QuantizedLinear] = {}
    for name, t in flat.items():
        if not name.endswith(".weight") or t.dtype not in (torch.uint32, torch.int32):
            continue
        base = name[: -len(".weight")]
        scales, biases = flat.get(f"{base}.scales"), flat.get(f"{base}.biases")
        if scales is None or biases is None:
            raise ValueError(f"quantized tensor has no scales/biases: {name}")
        if t.dim() != 2 or scales.shape != biases.shape or scales.dim() != 2 or scales.shape[0] != t.shape[0]:
            raise ValueError(f"{base}: weight {tuple(t.shape)} / scales {tuple(scales.shape)} / "
                             f"biases {tuple(biases.shape)} do not agree")
        k = int(t.shape[1]) * 32 // bits
        if int(scales.shape[1]) == 0 or k % int(scales.shape[1]):
            raise ValueError(f"{base}: {k} inputs do not split into {int(scales.shape[1])} groups")
        gs = k // int(scales.shape[1])
        if gs not in (32, 64, 128) or (group_size is not None and gs != group_size):
            raise ValueError(f"{base}: group size {gs} is not supported")
        bias = flat.get(f"{base}.bias")
        linears[base] = QuantizedLinear(t.view(torch.uint32) if t.dtype == torch.int32 else t,
                                        scales.to(torch.bfloat16), biases.to(torch.bfloat16),
                                        None if bias is None else bias.to(torch.bfloat16),
                                        group_size=gs, bits=bits)
        used.update({name, f"{base}.scales", f"{base}.biases", f"{base}.bias"})
    tensors = {n: t for n, t in flat.items() if n not in used}
    return QwenBlockWeights(linears, tensors)


def load_block_window(layout: TransformerLayout, block_indices: tuple[int, ...], *,
                      device: torch.device | str = "cuda", group_size: int | None = None) -> tuple[LoadedBlock, ...]:
    """Load the selected consecutive blocks' q6 layers into ``device`` memory."""

    if not block_indices:
        raise ValueError("block_indices cannot be empty")
    if tuple(block_indices) != tuple(range(block_indices[0], block_indices[-1] + 1)):
        raise ValueError("block_indices must be unique, consecutive, and ordered")
    plans = tuple(p for p in layout.plans if p.block_index in block_indices)
    if tuple(p.block_index for p in plans) != tuple(block_indices):
        raise ValueError(f"unknown Transformer block indices: {block_indices}")
    weight_map = layout.weight_map
    if not weight_map:
        raise ValueError("layout has no weight_map; build it with load_transformer_layout")
    per_shard: dict[str, list[str]] = {}
    for name, shard in weight_map.items():
        for i in block_indices:
            if name.startswith(f"transformer_blocks.{i}."):
                per_shard.setdefault(shard, []).append(name)
                break
    flat: dict[str, torch.Tensor] = {}
    for shard in layout.ordered_shards:
        if shard in per_shard:
            flat.update(load_safetensors(layout.transformer_dir / shard, per_shard[shard], device=device))
    loaded = []
    counts = {}
    for plan in plans:
        prefix = f"transformer_blocks.{plan.block_index}."
        part = {n[len(prefix):]: t for n, t in flat.items() if n.startswith(prefix)}
        counts[plan.block_index] = len(part)
        if len(part) != plan.tensor_count:
            raise RuntimeError("failed to load complete Transformer blocks: "
                               f"expected={tuple(block_indices)}, loaded_counts={counts}")
        loaded.append(LoadedBlock(block_index=plan.block_index, module=build_block(part, group_size=group_size)))
    return tuple(loaded)


def block_layers(blocks: Iterable[LoadedBlock]) -> dict[str, QuantizedLinear]:
    """Full layer names (``transformer_blocks.<i>.<layer>``) of loaded blocks,
    the namespace LoRA checkpoint keys resolve against."""

    return {f"transformer_blocks.{b.block_index}.{name}": lin
            for b in blocks for name, lin in b.module.linears.items()}
