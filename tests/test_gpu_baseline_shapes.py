"""GPU parity at the exact shapes the benchmarks run, against the CPU oracle.

* Config 1: one q6 linear, x [1728, 3072] -> 12288 outputs, gs64, no bias.
* The block's projection shapes at production sizes on the tensor path:
  3072 -> 18432 (the adaLN modulation linear) at M in {16, 512, 3456},
  12288 -> 3072 (fc2) at M in {512, 1728, 8192}, and group sizes 32 / 128 at
  K = 3072 and K = 12288 with M >= 1728 (q6_linear_profile.py:144-159 lists
  the shapes; benchmarks/benchmark_qwen_gemm.py:119-200 sweeps them).
* The LoRA pre-pass kernel (x @ A) and the fused rank-64 delta at image-FF width.
* GELU with the accurate tanh (Q6_EPI_GELU_PRECISE) against the reference's
  own gelu_approx_f table (tests/golden, q6_metal_mlp.py:21-26).

Full-size outputs are too large for the float64 oracle, so each case runs
whole on the GPU and is checked on a sample of rows (an output row depends
only on its own input row).  Weights are generated on the GPU by the torch
quantiser, which is bit-identical to the oracle's (test_capi_cpu.py).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from qwen_image_shardedit_mlx_b200 import _lib, ops
from qwen_image_shardedit_mlx_b200.quantize import quantize_affine_q6
from tests.helpers import assert_close, f32, from_bits, random_bf16, to_bits

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert ops.device_error() == 0


def _gpu_weights(seed: int, n: int, k: int, gs: int, *, bias: bool):
    """q6 weights quantised on the GPU from N(0, 0.02), plus the oracle's view of them."""

    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randn((n, k), generator=g, device="cuda") * 0.02
    q, s, b = quantize_affine_q6(w, gs)
    del w
    bias_t = (torch.randn((n,), generator=g, device="cuda") * 0.01).to(torch.bfloat16) if bias else None
    ow = oracle.Q6Weights(q.view(torch.int32).cpu().numpy().view(np.uint32), to_bits(s), to_bits(b),
                          None if bias_t is None else to_bits(bias_t), gs)
    return (q, s, b, bias_t), ow


def _sample_rows(rng: np.random.Generator, m: int, count: int = 32) -> np.ndarray:
    rows = np.sort(rng.choice(m, size=min(count, m), replace=False))
    rows[0], rows[-1] = 0, m - 1
    return np.unique(rows)


def _check_rows(got: torch.Tensor, x_bits: np.ndarray, ow: oracle.Q6Weights, rows: np.ndarray, **kw) -> None:
    ref = oracle.linear(oracle.bf16_bits_to_f32(x_bits[rows]), ow, weight_dtype="bf16", **kw)
    assert_close(f32(got[torch.as_tensor(rows, device=got.device)]), ref, what=kw.get("what", ""))


CASES = [
    # (M, N, K, gs, epilogue) - config 1 first
    (1728, 12288, 3072, 64, "plain"),
    (16, 18432, 3072, 64, "bias"),
    (512, 18432, 3072, 64, "bias"),
    (3456, 18432, 3072, 64, "bias"),
    (512, 3072, 12288, 64, "bias"),
    (1728, 3072, 12288, 64, "residual_gate"),
    (8192, 3072, 12288, 64, "bias"),
    (1728, 12288, 3072, 32, "bias_gelu"),
    (1728, 12288, 3072, 128, "bias_gelu"),
    (2048, 3072, 12288, 32, "bias"),
    (1728, 3072, 12288, 128, "residual_gate"),
]


@pytest.mark.parametrize("m,n,k,gs,epi", CASES)
def test_tensor_path_production_shapes(m, n, k, gs, epi):
    rng = np.random.default_rng(m + n + k + gs)
    w, ow = _gpu_weights(m * 31 + n + k + gs, n, k, gs, bias=epi != "plain")
    x = random_bf16(rng, (m, k))
    kwargs, okw = {}, {}
    if epi == "residual_gate":
        residual = random_bf16(rng, (m, n))
        gate = random_bf16(rng, (n,), 0.5)
        kwargs = dict(residual=from_bits(residual), gate=from_bits(gate))
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    got = ops.q6_linear(from_bits(x), *w, group_size=gs, apply_gelu=epi == "bias_gelu", path="tensor", out=out,
                        **kwargs)
    torch.cuda.synchronize()
    assert ops.last_path() == "tensor"
    assert bool(torch.isfinite(got).all()), "some output element was not written"
    rows = _sample_rows(rng, m)
    if epi == "residual_gate":
        okw = dict(residual=oracle.bf16_bits_to_f32(residual[rows]), gate=oracle.bf16_bits_to_f32(gate))
    _check_rows(got, x, ow, rows, apply_gelu=epi == "bias_gelu", **okw)


def test_config1_gemv_rows_and_tensor_rows_agree():
    """The few-row paths (fp32 weights) and the tensor path (bf16 weights) on
    the config-1 weight, as the auto path picks them: the streaming GEMV for
    one row, the warp-MMA kernel for 2-16 rows, the tensor core past that;
    each within tolerance of its oracle."""

    from oracle.block import kernel_weight_dtype

    rng = np.random.default_rng(17)
    w, ow = _gpu_weights(1717, 12288, 3072, 64, bias=False)
    for m, path in ((1, "simt"), (2, "skinny"), (4, "skinny"), (16, "skinny"), (17, "tensor")):
        x = random_bf16(rng, (m, 3072))
        got = ops.q6_linear(from_bits(x), *w, group_size=64)
        torch.cuda.synchronize()
        assert ops.last_path() == path
        dtype = kernel_weight_dtype(m, 12288, 3072, 64)
        assert dtype == ("bf16" if path == "tensor" else "f32")
        ref = oracle.linear(oracle.bf16_bits_to_f32(x), ow, weight_dtype=dtype)
        assert_close(f32(got), ref, what=f"config-1 weight, {m} rows")


@pytest.mark.parametrize("m,k,r", [(3456, 3072, 64), (37, 256, 32), (130, 12288, 256), (1000, 1040, 96),
                                   (5, 192, 128), (16, 64, 160), (20, 512, 64)])
def test_lora_prepass_kernel(m, k, r):
    """xa = x @ A by the library's pre-pass kernel against float64, rounded to
    bf16 once (fp32 accumulation: a few bf16 units at most)."""

    rng = np.random.default_rng(m + k + r)
    x = random_bf16(rng, (m, k))
    a = random_bf16(rng, (k, r), 0.01)
    got = ops.lora_xa(from_bits(x), from_bits(a))
    torch.cuda.synchronize()
    ref = oracle.bf16_bits_to_f32(x).astype(np.float64) @ oracle.bf16_bits_to_f32(a).astype(np.float64)
    assert_close(f32(got), ref.astype(np.float32), max_abs_rel=1e-2, mean_abs_rel=2e-3, what=f"lora xa {m}x{k}x{r}")


def test_lora_rank64_image_ff_width():
    """Config 4's rank-64 LoRA delta fused into the q6 tile at 3456 x 3072 -> 12288."""

    rng = np.random.default_rng(64)
    m, n, k, r = 3456, 12288, 3072, 64
    w, ow = _gpu_weights(6464, n, k, 64, bias=True)
    x = random_bf16(rng, (m, k))
    a_bits = random_bf16(rng, (k, r), 0.01)
    b_bits = random_bf16(rng, (r, n), 0.01)
    got = ops.q6_linear(from_bits(x), *w, group_size=64, apply_gelu=True,
                        lora=(from_bits(a_bits), from_bits(b_bits), 1.0))
    # B also given transposed ([N, r]: the fused stages' 16-byte row loads): the same bits
    got_t = ops.q6_linear(from_bits(x), *w, group_size=64, apply_gelu=True,
                          lora=(from_bits(a_bits), from_bits(b_bits), 1.0),
                          lora_b_nmajor=from_bits(b_bits).t().contiguous())
    torch.cuda.synchronize()
    assert torch.equal(got, got_t)
    rows = _sample_rows(rng, m, 24)
    lora = (oracle.bf16_bits_to_f32(a_bits), oracle.bf16_bits_to_f32(b_bits), 1.0)
    _check_rows(got, x, ow, rows, apply_gelu=True, lora=lora)


@pytest.mark.parametrize("r,scale", [(32, 0.5), (96, 2.0), (256, 1.0)])
def test_lora_nmajor_b_matches_row_major(r, scale):
    """The [N, r] LoRA B layout (Q6_LORA_B_NMAJOR) against the [r, N] one: same
    bits, including ranks whose second LoRA stage is partly padding."""

    rng = np.random.default_rng(r)
    m, n, k = 300, 1000, 512
    w, _ = _gpu_weights(r + 1, n, k, 64, bias=True)
    x = from_bits(random_bf16(rng, (m, k)))
    a = from_bits(random_bf16(rng, (k, r), 0.05))
    b = from_bits(random_bf16(rng, (r, n), 0.05))
    want = ops.q6_linear(x, *w, group_size=64, lora=(a, b, scale))
    got = ops.q6_linear(x, *w, group_size=64, lora=(a, b, scale), lora_b_nmajor=b.t().contiguous())
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.parametrize("path,m", [("tensor", 16), ("tensor", 64), ("simt", 1), ("simt", 3)])
def test_precise_gelu_matches_reference_table(golden, path, m):
    """Zero weights (codes, scales and biases all 0) make the pre-activation
    equal the output bias exactly, so the epilogue evaluates GELU at the
    reference table's inputs.  With the accurate tanh the bf16 outputs equal
    the reference's fp32 GELU rounded to bf16 but for rare one-unit
    rounding-boundary cases; with the hardware tanh.approx they differ more."""

    gx, gy = golden["gelu.x"], golden["gelu.y"]
    n, k, gs = gx.size, 64, 64
    w = torch.zeros((n, k * 6 // 32), dtype=torch.int32, device="cuda").view(torch.uint32)
    z = torch.zeros((n, k // gs), dtype=torch.bfloat16, device="cuda")
    bias = torch.from_numpy(gx).to(torch.bfloat16).cuda()
    x = torch.ones((m, k), dtype=torch.bfloat16, device="cuda")
    want = oracle.round_bf16(gy)
    got = f32(ops.q6_linear(x, w, z, z, bias, group_size=gs, apply_gelu=True, precise_gelu=True, path=path))
    torch.cuda.synchronize()
    assert ops.last_path() == path
    ulp = np.maximum(np.abs(want), 2.0 ** -126) * 2.0 ** -7
    for row in got:
        assert np.all(np.abs(row - want) <= ulp + 1e-30)
        assert np.mean(row == want) >= 0.98
    if path == "tensor":
        fast = f32(ops.q6_linear(x, w, z, z, bias, group_size=gs, apply_gelu=True, path=path))
        torch.cuda.synchronize()
        # the hardware tanh (about 2^-11 relative) stays within a few thousandths of the table
        assert np.all(np.abs(fast - want) <= 4 * ulp + 4e-3)


def test_precise_gelu_through_split_k(monkeypatch, golden):
    """The split-K reduce applies the precise GELU too."""

    monkeypatch.setenv("Q6_TC_KSPLIT", "2")
    rng = np.random.default_rng(3)
    m, n, k, gs = 24, 256, 2048, 64
    w, ow = _gpu_weights(303, n, k, gs, bias=True)
    x = random_bf16(rng, (m, k))
    got = ops.q6_linear(from_bits(x), *w, group_size=gs, apply_gelu=True, precise_gelu=True, path="tensor")
    torch.cuda.synchronize()
    ref = oracle.linear(oracle.bf16_bits_to_f32(x), ow, apply_gelu=True, weight_dtype="bf16")
    assert_close(f32(got), ref)


def test_pair_launch_not_refused():
    """The CTA-pair GEMM runs as pairs on B200 (no fallback recorded)."""

    rng = np.random.default_rng(8)
    before = ops.pair_fallback_count()
    w, _ = _gpu_weights(808, 12288, 3072, 64, bias=True)
    x = from_bits(random_bf16(rng, (3456, 3072)))
    ops.q6_linear(x, *w, group_size=64, apply_gelu=True)
    torch.cuda.synchronize()
    assert _lib.lib().q6_tensor_token_tile(3456, 12288) >= 128
    assert ops.pair_fallback_count() == before
