"""Generate the golden vectors in tests/golden/q6_reference_golden.npz.

The outputs come from the reference's own q6 kernel source
(shardedit_mlx/q6_metal_mlp.py:17-83, SOURCE_QMM_T with HEADER's
`extract_q6`/`dequant_q6`/`gelu_approx_f`) compiled for the CPU by
oracle/build_ref.py.  The inputs are seeded synthetic tensors whose shapes
mirror the reference's own numeric tests:

* ``linear_bf16``   - x (2, 8, 64) bf16, 64 -> 128 with bias
  (tests/test_q6_metal_mlp.py:35-45);
* ``mlp_fc1/mlp_fc2`` - x (1, 12, 64) bf16, 64 -> 128 (+GELU) -> 64, the
  ``fused_q6_mlp`` composition (tests/test_q6_metal_mlp.py:48-64);
* ``linear_f32``    - x (16, 128) fp32, 128 -> 256 with bias
  (tests/test_q6_steel_mlp.py:13-33, tests/test_q6_simdgroup_mlp.py:56-76);
* ``gs32`` / ``gs128`` - group sizes 32 and 128, ragged N, GELU / no bias;
* ``extract``       - every code index of two packed rows through `extract_q6`.

Run once in a container that has the reference tree (the GPU box has none):

    python oracle/build_ref.py && python tests/golden/make_golden.py
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402

OUT = Path(__file__).resolve().parent / "q6_reference_golden.npz"


def _quantized(rng: np.random.Generator, n: int, k: int, gs: int, with_bias: bool) -> oracle.Q6Weights:
    # nn.Linear's default init scale, then the affine q6 quantiser.
    bound = 1.0 / np.sqrt(k)
    w = rng.uniform(-bound, bound, size=(n, k)).astype(np.float32)
    packed, scales, biases = oracle.affine_quantize(w, group_size=gs)
    bias = oracle.f32_to_bf16_bits(rng.uniform(-bound, bound, size=(n,)).astype(np.float32)) if with_bias else None
    return oracle.Q6Weights(packed, scales, biases, bias, gs)


def _run_ref(ref, x: np.ndarray, w: oracle.Q6Weights, *, gelu: bool, dtype: str) -> np.ndarray:
    m, k = x.shape
    n = w.out_features
    scales = np.ascontiguousarray(w.scales_f32())
    biases = np.ascontiguousarray(w.biases_f32())
    bias = np.ascontiguousarray(w.bias_f32() if w.bias is not None else np.zeros((n,), np.float32))
    if dtype == "bf16":
        xin = np.ascontiguousarray(x, dtype=np.uint16)
        out = np.zeros((m, n), dtype=np.uint16)
        fn = ref.q6ref_qmm_t_bf16
    else:
        xin = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros((m, n), dtype=np.float32)
        fn = ref.q6ref_qmm_t_f32
    fn(
        xin.ctypes.data, w.weight.ctypes.data, scales.ctypes.data, biases.ctypes.data,
        bias.ctypes.data, out.ctypes.data, m, n, k, w.group_size, w.weight.shape[1],
        scales.shape[1], int(w.bias is not None), int(gelu),
    )
    return out


def main() -> int:
    ref = oracle.load_ref()
    if ref is None:
        print("oracle/_ref/libq6ref.so is missing; run oracle/build_ref.py first", file=sys.stderr)
        return 1
    rng = np.random.default_rng(20251201)
    arrays: dict[str, np.ndarray] = {}

    def put(prefix: str, x: np.ndarray, w: oracle.Q6Weights, y: np.ndarray, gelu: bool) -> None:
        arrays[f"{prefix}.x"] = x
        arrays[f"{prefix}.weight"] = w.weight
        arrays[f"{prefix}.scales"] = w.scales
        arrays[f"{prefix}.biases"] = w.biases
        if w.bias is not None:
            arrays[f"{prefix}.bias"] = w.bias
        arrays[f"{prefix}.group_size"] = np.array(w.group_size, dtype=np.int32)
        arrays[f"{prefix}.gelu"] = np.array(int(gelu), dtype=np.int32)
        arrays[f"{prefix}.y"] = y

    # linear_bf16: x (2, 8, 64) -> (16, 64)
    x = oracle.f32_to_bf16_bits(rng.standard_normal((16, 64)).astype(np.float32))
    w = _quantized(rng, 128, 64, 64, True)
    put("linear_bf16", x, w, _run_ref(ref, x, w, gelu=False, dtype="bf16"), False)

    # fused MLP: fc1 with GELU epilogue, then fc2 on the bf16 hidden
    x = oracle.f32_to_bf16_bits(rng.standard_normal((12, 64)).astype(np.float32))
    w1 = _quantized(rng, 128, 64, 64, True)
    w2 = _quantized(rng, 64, 128, 64, True)
    h = _run_ref(ref, x, w1, gelu=True, dtype="bf16")
    y = _run_ref(ref, h, w2, gelu=False, dtype="bf16")
    put("mlp_fc1", x, w1, h, True)
    put("mlp_fc2", h, w2, y, False)

    # fp32 linear 128 -> 256
    x = rng.standard_normal((16, 128)).astype(np.float32)
    w = _quantized(rng, 256, 128, 64, True)
    put("linear_f32", x, w, _run_ref(ref, x, w, gelu=False, dtype="f32"), False)

    # group sizes 32 / 128, ragged N and M
    x = oracle.f32_to_bf16_bits(rng.standard_normal((7, 256)).astype(np.float32))
    w = _quantized(rng, 96, 256, 32, True)
    put("gs32", x, w, _run_ref(ref, x, w, gelu=True, dtype="bf16"), True)
    x = oracle.f32_to_bf16_bits(rng.standard_normal((5, 256)).astype(np.float32))
    w = _quantized(rng, 160, 256, 128, False)
    put("gs128", x, w, _run_ref(ref, x, w, gelu=False, dtype="bf16"), False)

    # extract_q6 over every index of two random rows
    packed = rng.integers(0, 2**32, size=(2, 24), dtype=np.uint64).astype(np.uint32)
    codes = np.zeros((2, 128), dtype=np.uint8)
    for r in range(2):
        row = np.ascontiguousarray(packed[r])
        for i in range(128):
            codes[r, i] = ref.q6ref_extract_q6(row.ctypes.data, i)
    arrays["extract.packed"] = packed
    arrays["extract.codes"] = codes

    # GELU at a spread of points
    pts = np.linspace(-8.0, 8.0, 257, dtype=np.float32)
    arrays["gelu.x"] = pts
    arrays["gelu.y"] = np.array([ref.q6ref_gelu_approx(float(v)) for v in pts], dtype=np.float32)

    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(arrays)} arrays)")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
