"""The CPU oracle pinned against the reference's own kernel source (golden vectors).

Every golden output was produced by the reference's SOURCE_QMM_T / extract_q6 /
gelu_approx_f (shardedit_mlx/q6_metal_mlp.py:17-83) compiled for the CPU; the
oracle's C restatement must reproduce them bit for bit.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.conftest import golden_case

LINEAR_CASES = ["linear_bf16", "mlp_fc1", "mlp_fc2", "linear_f32", "gs32", "gs128"]


def test_extract_matches_reference_golden(golden):
    packed = golden["extract.packed"]
    codes = golden["extract.codes"]
    assert (oracle.unpack_q6(packed, 128) == codes).all()
    assert (oracle.c_unpack(packed, 128) == codes).all()


def test_pack_roundtrip_all_code_values():
    rng = np.random.default_rng(3)
    for k in (16, 32, 64, 128, 3072):
        codes = rng.integers(0, 64, size=(9, k), dtype=np.uint8)
        codes[0, :64 if k >= 64 else k] = np.arange(min(64, k), dtype=np.uint8)
        packed = oracle.pack_q6(codes)
        assert packed.shape == (9, k * 6 // 32)
        assert (oracle.c_pack(codes) == packed).all()
        assert (oracle.unpack_q6(packed, k) == codes).all()


def test_pack_known_answer_ramp():
    # codes 0..15: stream bits 6j..6j+5 hold j.
    codes = np.arange(16, dtype=np.uint8)[None, :]
    words = oracle.pack_q6(codes)[0]
    stream = int(words[0]) | int(words[1]) << 32 | int(words[2]) << 64
    for j in range(16):
        assert (stream >> (6 * j)) & 63 == j


@pytest.mark.parametrize("case", LINEAR_CASES)
def test_c_oracle_bit_exact_vs_reference_golden(golden, case):
    x, w, y, gelu = golden_case(golden, case)
    is_f32 = y.dtype == np.float32
    xf = x if is_f32 else oracle.bf16_bits_to_f32(x)
    got = oracle.c_qmm_t(
        xf, w.weight, w.scales_f32(), w.biases_f32(), w.bias_f32(), w.group_size, apply_gelu=gelu
    )
    if is_f32:
        assert np.array_equal(got.view(np.uint32), y.view(np.uint32))
    else:
        assert np.array_equal(oracle.f32_to_bf16_bits(got), y)


@pytest.mark.parametrize("case", LINEAR_CASES)
def test_blas_oracle_close_to_reference_golden(golden, case):
    x, w, y, gelu = golden_case(golden, case)
    is_f32 = y.dtype == np.float32
    xf = x if is_f32 else oracle.bf16_bits_to_f32(x)
    got = oracle.linear(xf, w, apply_gelu=gelu, weight_dtype="f32")
    ref = y if is_f32 else oracle.bf16_bits_to_f32(y)
    tol = 1e-5 if is_f32 else 2e-2 * float(np.abs(ref).max())
    assert float(np.abs(got - ref).max()) <= tol


def test_gelu_matches_reference_golden(golden):
    xs = golden["gelu.x"]
    ys = golden["gelu.y"]
    got = np.array([oracle.c_gelu(v) for v in xs], dtype=np.float32)
    assert np.array_equal(got.view(np.uint32), ys.view(np.uint32))
    assert np.allclose(oracle.gelu(xs), ys, rtol=2e-6, atol=2e-6)


def test_dequant_bf16_c_and_numpy_agree():
    rng = np.random.default_rng(5)
    for gs in (32, 64, 128):
        w = rng.normal(0.0, 0.02, size=(33, 256)).astype(np.float32)
        packed, scales, biases = oracle.affine_quantize(w, group_size=gs)
        a = oracle.c_dequant_bf16(packed, scales, biases, gs)
        b = oracle.dequantize(packed, scales, biases, gs, dtype="bf16")
        assert np.array_equal(a, b)
        # quantisation error bounded by half a step (+ bf16 rounding of scale/bias)
        wf = oracle.dequantize(packed, scales, biases, gs, dtype="f32")
        step = oracle.bf16_bits_to_f32(scales).repeat(gs, axis=1)
        assert np.all(np.abs(wf - w) <= 0.51 * step + 2e-3 * np.abs(w) + 1e-6)


def test_fused_and_eager_mlp_orders_are_close():
    rng = np.random.default_rng(9)
    x = oracle.round_bf16(rng.standard_normal((24, 128)).astype(np.float32))
    fc1 = _rand_linear(rng, 256, 128, 64)
    fc2 = _rand_linear(rng, 128, 256, 64)
    fused = oracle.fused_mlp(x, fc1, fc2)
    eager = oracle.eager_mlp(x, fc1, fc2)
    assert float(np.abs(fused - eager).max()) < 0.05


def _rand_linear(rng, n, k, gs):
    w = rng.normal(0.0, 0.02, size=(n, k)).astype(np.float32)
    packed, scales, biases = oracle.affine_quantize(w, group_size=gs)
    bias = oracle.f32_to_bf16_bits(rng.normal(0.0, 0.01, size=(n,)).astype(np.float32))
    return oracle.Q6Weights(packed, scales, biases, bias, gs)


def test_reference_library_agrees_when_present(golden):
    """If oracle/_ref was built here, re-run one golden case through it directly."""

    ref = oracle.load_ref()
    if ref is None:
        pytest.skip("oracle/_ref/libq6ref.so not built")
    x, w, y, gelu = golden_case(golden, "gs32")
    n = w.out_features
    m, k = x.shape
    out = np.zeros((m, n), dtype=np.uint16)
    scales = np.ascontiguousarray(w.scales_f32())
    biases = np.ascontiguousarray(w.biases_f32())
    bias = np.ascontiguousarray(w.bias_f32())
    xin = np.ascontiguousarray(x)
    ref.q6ref_qmm_t_bf16(
        xin.ctypes.data, w.weight.ctypes.data, scales.ctypes.data, biases.ctypes.data,
        bias.ctypes.data, out.ctypes.data, m, n, k, w.group_size, w.weight.shape[1],
        scales.shape[1], 1, int(gelu),
    )
    assert np.array_equal(out, y)
