"""CPU oracle (test infrastructure only) for the q6 affine linear / image FF MLP.

Everything here restates the reference's q6 path on the host:

* packing  - 6-bit codes as one continuous little-endian bit stream per row of
  uint32 words, the layout ``extract_q6`` reads
  (shardedit_mlx/q6_metal_mlp.py:28-40);
* dequant  - ``w = scale * q + bias`` in fp32 (q6_metal_mlp.py:42-54); the
  bf16 pre-dequantised form ``bf16_rn(fp32(s) * q + fp32(b))`` is what
  ``dequantize_linear`` / ``mx.dequantize(dtype=bf16)`` hands to the dense path
  (q6_metal_mlp.py:143-154);
* linear   - one output per (m, n), fp32 accumulation in k order, optional
  bias and GELU-tanh epilogue (q6_metal_mlp.py:58-83, GELU at :21-26);
* MLP      - fused order ``fc2(gelu(fc1(x)))`` with one rounding per linear
  (``fused_q6_mlp``, q6_metal_mlp.py:207-215) and eager order with one
  rounding per op (``eager_q6_mlp`` / ``dense_mlp``, q6_metal_mlp.py:218-253);
* LoRA     - additive ``out += scale * ((x @ A) @ B)``
  (shardedit_mlx/dense_img_ff_window.py:48-60).

The affine quantiser used to *generate* synthetic weights restates MLX's
published affine scheme (``mx.quantize``, mlx>=0.31 per pyproject.toml:27, not
vendored and not importable here): per group of ``group_size`` along K,
``scale = max((max - min) / 63, 1e-7)``, ``bias = min``, both stored in bf16,
``q = clip(round((w - bias) / scale), 0, 63)``.  Whether this matches
``mx.quantize`` bit for bit is parity unpinned (MLX is absent); the hot path
never depends on it because every kernel consumes whatever codes, scales and
biases it is given.

The compiled C restatement (q6_oracle.c -> libq6oracle.so) holds the
bit-exact loops; numpy versions here are used for sizes where the scalar loops
would be slow, and are checked against the C ones.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libq6oracle.so"
REF_LIB_PATH = HERE / "_ref" / "libq6ref.so"

GELU_K = np.float32(0.7978845608028654)
GELU_C = np.float32(0.044715)

__all__ = [
    "LIB_PATH",
    "REF_LIB_PATH",
    "Q6Weights",
    "affine_quantize",
    "bf16_bits_to_f32",
    "build_oracle",
    "c_dequant_bf16",
    "c_gelu",
    "c_pack",
    "c_qmm_t",
    "c_unpack",
    "dequantize",
    "eager_mlp",
    "f32_to_bf16_bits",
    "fused_mlp",
    "gelu",
    "linear",
    "load_ref",
    "pack_q6",
    "round_bf16",
    "unpack_q6",
]


# --------------------------------------------------------------------------
# build / load
# --------------------------------------------------------------------------


def build_oracle(force: bool = False) -> Path:
    """Compile q6_oracle.c into libq6oracle.so next to it (gcc, no fp contraction)."""

    src = HERE / "q6_oracle.c"
    if LIB_PATH.exists() and not force and LIB_PATH.stat().st_mtime >= src.stat().st_mtime:
        return LIB_PATH
    cc = os.environ.get("CC", "gcc")
    cmd = [cc, "-O2", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off", str(src), "-o", str(LIB_PATH), "-lm"]
    subprocess.run(cmd, check=True)
    return LIB_PATH


_LIB: ctypes.CDLL | None = None


def _lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            build_oracle()
        lib = ctypes.CDLL(str(LIB_PATH))
        p = ctypes.c_void_p
        i64 = ctypes.c_int64
        lib.q6o_extract.restype = ctypes.c_uint32
        lib.q6o_extract.argtypes = [p, ctypes.c_uint32]
        lib.q6o_pack.argtypes = [p, i64, i64, p]
        lib.q6o_unpack.argtypes = [p, i64, i64, p]
        lib.q6o_dequant_bf16.argtypes = [p, p, p, i64, i64, i64, p]
        lib.q6o_dequant_f32.argtypes = [p, p, p, i64, i64, i64, p]
        lib.q6o_qmm_t.argtypes = [p, p, p, p, p, ctypes.c_int, ctypes.c_int, i64, i64, i64, i64, p]
        lib.q6o_gelu.restype = ctypes.c_float
        lib.q6o_gelu.argtypes = [ctypes.c_float]
        _LIB = lib
    return _LIB


def load_ref() -> ctypes.CDLL | None:
    """The reference's own naive q6 kernel compiled for the CPU (oracle/_ref), if built."""

    if not REF_LIB_PATH.exists():
        return None
    lib = ctypes.CDLL(str(REF_LIB_PATH))
    p = ctypes.c_void_p
    u = ctypes.c_uint
    i = ctypes.c_int
    for name in ("q6ref_qmm_t_f32", "q6ref_qmm_t_bf16"):
        fn = getattr(lib, name)
        fn.restype = None
        fn.argtypes = [p, p, p, p, p, p, u, u, u, u, u, u, i, i]
    lib.q6ref_extract_q6.restype = u
    lib.q6ref_extract_q6.argtypes = [p, u]
    lib.q6ref_dequant_q6.restype = ctypes.c_float
    lib.q6ref_dequant_q6.argtypes = [p, p, p, u, u]
    lib.q6ref_gelu_approx.restype = ctypes.c_float
    lib.q6ref_gelu_approx.argtypes = [ctypes.c_float]
    return lib


def _ptr(a: np.ndarray | None) -> int | None:
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# --------------------------------------------------------------------------
# bf16 helpers (bf16 values carried as uint16 bit patterns)
# --------------------------------------------------------------------------


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (uint16)."""

    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    is_nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    r = np.where(is_nan, ((u >> 16) | 0x40) & 0xFFFF, r)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(a: np.ndarray) -> np.ndarray:
    """fp32 values rounded to the nearest bf16 (returned as fp32)."""

    return bf16_bits_to_f32(f32_to_bf16_bits(a))


# --------------------------------------------------------------------------
# packing (continuous LSB-first 6-bit stream over uint32 words)
# --------------------------------------------------------------------------


def pack_q6(codes: np.ndarray) -> np.ndarray:
    """codes uint8 [..., K] (values < 64, K % 16 == 0) -> uint32 [..., K*6/32].

    Sixteen codes fill three words: code j occupies stream bits [6j, 6j+6).
    """

    codes = np.asarray(codes)
    k = codes.shape[-1]
    if k % 16:
        raise ValueError(f"K={k} must be a multiple of 16 for 6-bit packing")
    c = codes.reshape(codes.shape[:-1] + (k // 16, 16)).astype(np.uint32) & 63
    w0 = c[..., 0] | c[..., 1] << 6 | c[..., 2] << 12 | c[..., 3] << 18 | c[..., 4] << 24 | (c[..., 5] & 3) << 30
    w1 = (c[..., 5] >> 2) | c[..., 6] << 4 | c[..., 7] << 10 | c[..., 8] << 16 | c[..., 9] << 22 | (c[..., 10] & 15) << 28
    w2 = (c[..., 10] >> 4) | c[..., 11] << 2 | c[..., 12] << 8 | c[..., 13] << 14 | c[..., 14] << 20 | c[..., 15] << 26
    out = np.stack([w0, w1, w2], axis=-1).astype(np.uint32)
    return out.reshape(codes.shape[:-1] + (k * 6 // 32,))


def unpack_q6(packed: np.ndarray, k: int) -> np.ndarray:
    """uint32 [..., K*6/32] -> codes uint8 [..., K]."""

    packed = np.asarray(packed, dtype=np.uint32)
    if packed.shape[-1] * 32 != k * 6:
        raise ValueError(f"packed width {packed.shape[-1]} does not hold K={k} 6-bit codes")
    t = packed.reshape(packed.shape[:-1] + (k // 16, 3))
    w0, w1, w2 = t[..., 0], t[..., 1], t[..., 2]
    cols = [
        w0, w0 >> 6, w0 >> 12, w0 >> 18, w0 >> 24, (w0 >> 30) | (w1 << 2),
        w1 >> 4, w1 >> 10, w1 >> 16, w1 >> 22, (w1 >> 28) | (w2 << 4),
        w2 >> 2, w2 >> 8, w2 >> 14, w2 >> 20, w2 >> 26,
    ]
    c = np.stack([col & 63 for col in cols], axis=-1).astype(np.uint8)
    return c.reshape(packed.shape[:-1] + (k,))


# --------------------------------------------------------------------------
# quantised weights
# --------------------------------------------------------------------------


@dataclass
class Q6Weights:
    """One q6 linear in MLX layout (host arrays)."""

    weight: np.ndarray  # uint32 [N, K*6/32]
    scales: np.ndarray  # uint16 bf16 bits [N, K/gs]
    biases: np.ndarray  # uint16 bf16 bits [N, K/gs]
    bias: np.ndarray | None  # uint16 bf16 bits [N] (output bias) or None
    group_size: int

    @property
    def out_features(self) -> int:
        return int(self.weight.shape[0])

    @property
    def in_features(self) -> int:
        return int(self.weight.shape[1] * 32 // 6)

    def scales_f32(self) -> np.ndarray:
        return bf16_bits_to_f32(self.scales)

    def biases_f32(self) -> np.ndarray:
        return bf16_bits_to_f32(self.biases)

    def bias_f32(self) -> np.ndarray | None:
        return None if self.bias is None else bf16_bits_to_f32(self.bias)


def affine_quantize(w: np.ndarray, group_size: int = 64, bits: int = 6) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """MLX-style affine min/max quantiser -> (packed uint32, scales bf16, biases bf16)."""

    if bits != 6:
        raise ValueError("only bits=6 is supported")
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    if k % group_size:
        raise ValueError(f"K={k} is not a multiple of group_size={group_size}")
    g = w.reshape(n, k // group_size, group_size)
    w_max = g.max(axis=-1)
    w_min = g.min(axis=-1)
    scale = np.maximum((w_max - w_min) / np.float32(63.0), np.float32(1e-7)).astype(np.float32)
    scale_bits = f32_to_bf16_bits(scale)
    bias_bits = f32_to_bf16_bits(w_min)
    s = bf16_bits_to_f32(scale_bits)[..., None]
    b = bf16_bits_to_f32(bias_bits)[..., None]
    q = np.clip(np.rint((g - b) / s), 0, 63).astype(np.uint8).reshape(n, k)
    return pack_q6(q), scale_bits, bias_bits


def dequantize(packed: np.ndarray, scales: np.ndarray, biases: np.ndarray, group_size: int, *, dtype: str = "bf16") -> np.ndarray:
    """Dense weights [N, K]: fp32 ``s*q + b``; ``dtype='bf16'`` returns the bf16 bit patterns.

    scales/biases are bf16 bit patterns (uint16) or fp32 values.
    """

    s = scales if scales.dtype == np.float32 else bf16_bits_to_f32(scales)
    b = biases if biases.dtype == np.float32 else bf16_bits_to_f32(biases)
    n = packed.shape[0]
    k = packed.shape[1] * 32 // 6
    q = unpack_q6(packed, k).astype(np.float32).reshape(n, k // group_size, group_size)
    w = (s[..., None] * q + b[..., None]).astype(np.float32).reshape(n, k)
    if dtype == "bf16":
        return f32_to_bf16_bits(w)
    if dtype == "f32":
        return w
    raise ValueError(dtype)


def gelu(v: np.ndarray) -> np.ndarray:
    v = np.asarray(v, dtype=np.float32)
    x3 = v * v * v
    return (np.float32(0.5) * v * (np.float32(1.0) + np.tanh(GELU_K * (v + GELU_C * x3)))).astype(np.float32)


def linear(
    x: np.ndarray,
    w: Q6Weights,
    *,
    apply_gelu: bool = False,
    weight_dtype: str = "bf16",
    residual: np.ndarray | None = None,
    gate: np.ndarray | None = None,
    lora: tuple[np.ndarray, np.ndarray, float] | list[tuple[np.ndarray, np.ndarray, float]] | None = None,
) -> np.ndarray:
    """fp32 result of one q6 linear (BLAS in float64, then fp32).

    ``weight_dtype='bf16'`` uses bf16-dequantised weights (the MLX qmm /
    dequantize_linear semantics the tensor-core kernels match); ``'f32'`` keeps
    fp32 weights like the reference's naive kernel.  ``x`` holds fp32 values
    (bf16 activations widened).  Epilogue: ``+bias``, GELU, then
    ``residual + gate * value`` (block residual gate, benchmarks/profile_qwen_block.py:294-301),
    LoRA added before the bias (dense_img_ff_window.py:54-59); a list of
    adapters adds sum_i s_i (x A_i) B_i, the delta the reference folds for
    several adapters (dense_img_ff_window.py:121-131).
    """

    wd = dequantize(w.weight, w.scales, w.biases, w.group_size, dtype=weight_dtype)
    wf = bf16_bits_to_f32(wd) if weight_dtype == "bf16" else wd
    acc = np.asarray(x, dtype=np.float64) @ wf.astype(np.float64).T
    for a, b, s in ([] if lora is None else [lora] if isinstance(lora, tuple) else lora):
        xa = np.asarray(x, dtype=np.float64) @ np.asarray(a, dtype=np.float64)
        acc = acc + float(s) * (xa @ np.asarray(b, dtype=np.float64))
    acc = acc.astype(np.float32)
    if w.bias is not None:
        acc = acc + w.bias_f32()
    if apply_gelu:
        acc = gelu(acc)
    if gate is not None:
        acc = np.asarray(gate, dtype=np.float32) * acc
    if residual is not None:
        acc = np.asarray(residual, dtype=np.float32) + acc
    return acc.astype(np.float32)


def fused_mlp(x: np.ndarray, fc1: Q6Weights, fc2: Q6Weights, *, weight_dtype: str = "bf16") -> np.ndarray:
    """fc2(gelu(fc1(x))) with the hidden rounded to bf16 once (fused_q6_mlp order); fp32 out."""

    h = round_bf16(linear(x, fc1, apply_gelu=True, weight_dtype=weight_dtype))
    return linear(h, fc2, weight_dtype=weight_dtype)


def eager_mlp(x: np.ndarray, fc1: Q6Weights, fc2: Q6Weights, *, weight_dtype: str = "bf16") -> np.ndarray:
    """Eager order (each op rounds to bf16): matmul, +bias, gelu, matmul, +bias."""

    def lin(v: np.ndarray, w: Q6Weights) -> np.ndarray:
        no_bias = Q6Weights(w.weight, w.scales, w.biases, None, w.group_size)
        out = round_bf16(linear(v, no_bias, weight_dtype=weight_dtype))
        if w.bias is not None:
            out = round_bf16(out + w.bias_f32())
        return out

    h = round_bf16(gelu(lin(x, fc1)))
    return lin(h, fc2)


# --------------------------------------------------------------------------
# compiled scalar loops (exact reference operation order)
# --------------------------------------------------------------------------


def c_gelu(v: float) -> float:
    return float(_lib().q6o_gelu(float(v)))


def c_pack(codes: np.ndarray) -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    n, k = codes.shape
    out = np.zeros((n, k * 6 // 32), dtype=np.uint32)
    _lib().q6o_pack(_ptr(codes), n, k, _ptr(out))
    return out


def c_unpack(packed: np.ndarray, k: int) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.uint32)
    n = packed.shape[0]
    out = np.zeros((n, k), dtype=np.uint8)
    _lib().q6o_unpack(_ptr(packed), n, k, _ptr(out))
    return out


def c_dequant_bf16(packed: np.ndarray, scales: np.ndarray, biases: np.ndarray, group_size: int) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.uint32)
    scales = np.ascontiguousarray(scales, dtype=np.uint16)
    biases = np.ascontiguousarray(biases, dtype=np.uint16)
    n = packed.shape[0]
    k = packed.shape[1] * 32 // 6
    out = np.zeros((n, k), dtype=np.uint16)
    _lib().q6o_dequant_bf16(_ptr(packed), _ptr(scales), _ptr(biases), n, k, group_size, _ptr(out))
    return out


def c_qmm_t(
    x: np.ndarray,
    packed: np.ndarray,
    scales: np.ndarray,
    biases: np.ndarray,
    bias: np.ndarray | None,
    group_size: int,
    *,
    apply_gelu: bool = False,
    round_w_bf16: bool = False,
) -> np.ndarray:
    """Scalar loop in the reference kernel's operation order; fp32 [M, N] before output rounding."""

    x = np.ascontiguousarray(x, dtype=np.float32)
    packed = np.ascontiguousarray(packed, dtype=np.uint32)
    scales = np.ascontiguousarray(scales, dtype=np.float32)
    biases = np.ascontiguousarray(biases, dtype=np.float32)
    bias_arr = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    m, k = x.shape
    n = packed.shape[0]
    out = np.zeros((m, n), dtype=np.float32)
    _lib().q6o_qmm_t(
        _ptr(x), _ptr(packed), _ptr(scales), _ptr(biases), _ptr(bias_arr),
        int(apply_gelu), int(round_w_bf16), m, n, k, group_size, _ptr(out),
    )
    return out
