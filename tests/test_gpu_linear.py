"""GPU parity of the q6 kernels against the CPU oracle, through the C ABI.

Bars:
* dequantised weights: bit-exact vs bf16_rn(fp32(s)*q + fp32(b));
* bf16 matmul outputs: max|err| <= 2e-2 * max|ref| and mean|err| <= 1e-3 * rms(ref)
  against the oracle with the same weight precision (bf16 weights for the
  tensor-core path, fp32 weights for the CUDA-core path);
* against the reference kernel's own golden outputs (fp32 weights), the
  tensor-core path meets max-abs-rel 2e-2 and the reference tests' own bar
  of max|err| < 0.05 (tests/test_q6_metal_mlp.py:35-45);
* fp32 path vs the fp32 golden: max|err| < 1e-5 (tests/test_q6_steel_mlp.py:13-33).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from qwen_image_shardedit_mlx_b200 import _lib, ops
from tests.conftest import golden_case
from tests.helpers import (
    assert_close,
    f32,
    from_bits,
    random_bf16,
    random_weights,
    to_bits,
    u32_to_torch,
    weights_to_torch,
)

pytestmark = pytest.mark.gpu

BF16_GOLDEN = ["linear_bf16", "mlp_fc1", "mlp_fc2", "gs32", "gs128"]


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert ops.device_error() == 0


@pytest.mark.parametrize("gs", [32, 64, 128])
def test_dequantize_bit_exact(gs):
    rng = np.random.default_rng(100 + gs)
    w = random_weights(rng, 300, 3072, gs, bias=False)
    wt, st, bt, _ = weights_to_torch(w)
    dense = ops.q6_dequantize(wt, st, bt, gs)
    torch.cuda.synchronize()
    assert np.array_equal(to_bits(dense), oracle.dequantize(w.weight, w.scales, w.biases, gs, dtype="bf16"))


def test_dequantize_bit_exact_extreme_scales():
    # scales / biases spanning many binades, including values whose fp32 sum rounds
    rng = np.random.default_rng(7)
    n, k, gs = 64, 256, 64
    codes = rng.integers(0, 64, size=(n, k), dtype=np.uint8)
    packed = oracle.pack_q6(codes)
    exps = rng.integers(-40, 20, size=(n, k // gs)).astype(np.float32)
    scales = oracle.f32_to_bf16_bits((rng.uniform(1, 2, size=(n, k // gs)) * 2.0 ** exps).astype(np.float32))
    biases = oracle.f32_to_bf16_bits((rng.uniform(-2, 2, size=(n, k // gs)) * 2.0 ** (exps + rng.integers(-10, 10, size=exps.shape))).astype(np.float32))
    dense = ops.q6_dequantize(u32_to_torch(packed), from_bits(scales), from_bits(biases), gs)
    torch.cuda.synchronize()
    assert np.array_equal(to_bits(dense), oracle.c_dequant_bf16(packed, scales, biases, gs))


@pytest.mark.parametrize("case", BF16_GOLDEN)
@pytest.mark.parametrize("path", ["tensor", "simt"])
def test_reference_golden_bf16(golden, case, path):
    x, w, y, gelu = golden_case(golden, case)
    wt, st, bt, bias = weights_to_torch(w)
    got = ops.q6_linear(from_bits(x), wt, st, bt, bias, group_size=w.group_size, apply_gelu=gelu, path=path)
    torch.cuda.synchronize()
    assert ops.last_path() == path
    ref = oracle.bf16_bits_to_f32(y)
    assert float(np.abs(f32(got) - ref).max()) < 0.05
    if path == "simt":
        # same weight precision as the reference kernel: only summation order differs
        assert_close(f32(got), ref, what=case)
    else:
        # bf16-dequantised weights: compare with the oracle of the same precision
        xf = oracle.bf16_bits_to_f32(x)
        assert_close(f32(got), oracle.linear(xf, w, apply_gelu=gelu, weight_dtype="bf16"), what=case)
        assert_close(f32(got), ref, mean_abs_rel=4e-3, what=case + " vs fp32-weight golden")


def test_reference_golden_f32(golden):
    x, w, y, gelu = golden_case(golden, "linear_f32")
    wt, st, bt, bias = weights_to_torch(w)
    got = ops.q6_linear(torch.from_numpy(x).cuda(), wt, st, bt, bias, group_size=w.group_size)
    torch.cuda.synchronize()
    assert got.dtype == torch.float32
    assert float(np.abs(f32(got) - y).max()) < 1e-5


SHAPES = [
    # (M, N, K, gs)
    (5, 128, 64, 64),
    (16, 384, 192, 32),
    (17, 300, 256, 128),
    (130, 640, 1024, 64),
    (256, 3072, 3072, 64),
    (333, 256, 12288, 64),
    (1000, 96, 512, 32),
]


@pytest.mark.parametrize("m,n,k,gs", SHAPES)
@pytest.mark.parametrize("epi", ["plain", "bias_gelu", "residual_gate"])
def test_tensor_path_vs_oracle(m, n, k, gs, epi):
    rng = np.random.default_rng(m * 7 + n * 3 + k)
    w = random_weights(rng, n, k, gs, bias=epi != "plain")
    x = random_bf16(rng, (m, k))
    wt, st, bt, bias = weights_to_torch(w)
    kwargs = {}
    residual = gate = None
    if epi == "residual_gate":
        residual = random_bf16(rng, (m, n))
        gate = random_bf16(rng, (n,), 0.5)
        kwargs = dict(residual=from_bits(residual), gate=from_bits(gate))
    got = ops.q6_linear(from_bits(x), wt, st, bt, bias, group_size=gs, apply_gelu=epi == "bias_gelu",
                        path="tensor", **kwargs)
    torch.cuda.synchronize()
    ref = oracle.linear(
        oracle.bf16_bits_to_f32(x), w, apply_gelu=epi == "bias_gelu", weight_dtype="bf16",
        residual=None if residual is None else oracle.bf16_bits_to_f32(residual),
        gate=None if gate is None else oracle.bf16_bits_to_f32(gate),
    )
    assert_close(f32(got), ref, what=f"{m}x{n}x{k} gs{gs} {epi}")


@pytest.mark.parametrize("m,n,k", [(16, 128, 64), (5, 96, 256), (40, 200, 128), (200, 130, 192), (700, 256, 64)])
@pytest.mark.parametrize("path", ["tensor", "simt"])
def test_every_output_written(m, n, k, path):
    """The output buffer starts as NaN; every element must be overwritten."""

    rng = np.random.default_rng(m + n + k)
    w = random_weights(rng, n, k, 64)
    x = random_bf16(rng, (m, k))
    wt, st, bt, bias = weights_to_torch(w)
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    got = ops.q6_linear(from_bits(x), wt, st, bt, bias, group_size=64, path=path, out=out)
    torch.cuda.synchronize()
    assert got.data_ptr() == out.data_ptr()
    assert bool(torch.isfinite(got).all())
    ref = oracle.linear(oracle.bf16_bits_to_f32(x), w, weight_dtype="bf16" if path == "tensor" else "f32")
    assert_close(f32(got), ref)


@pytest.mark.parametrize("m", [1, 2, 3, 4, 7])
def test_simt_path_small_m(m):
    rng = np.random.default_rng(40 + m)
    w = random_weights(rng, 1000, 3072, 64)
    x = random_bf16(rng, (m, 3072))
    wt, st, bt, bias = weights_to_torch(w)
    got = ops.q6_linear(from_bits(x), wt, st, bt, bias, group_size=64, path="simt")
    torch.cuda.synchronize()
    ref = oracle.linear(oracle.bf16_bits_to_f32(x), w, weight_dtype="f32")
    assert_close(f32(got), ref)


GEMV_SHAPES = [
    (1001, 3072, 64),   # odd row count: the last row pair has one row
    (257, 12288, 64),   # fc2-shaped K: three 4096-code chunks per row
    (130, 1024, 32),    # one group per 32-code half unit
    (64, 2048, 128),    # one group per two units
    (3, 64, 64),        # one scale group per row: the CUDA-core fallback
]


@pytest.mark.parametrize("m", [1, 2, 3, 4])
@pytest.mark.parametrize("n,k,gs", GEMV_SHAPES)
@pytest.mark.parametrize("epi", ["plain", "bias_gelu", "residual_gate"])
def test_gemv_path_vs_oracle(m, n, k, gs, epi):
    """The streaming GEMV (M <= 4) against the fp32-weight oracle; the output
    starts as NaN so every element must be written."""

    rng = np.random.default_rng(m * 11 + n + k + gs)
    w = random_weights(rng, n, k, gs, bias=epi != "plain")
    x = random_bf16(rng, (m, k))
    wt, st, bt, bias = weights_to_torch(w)
    kwargs = {}
    residual = gate = None
    if epi == "residual_gate":
        residual = random_bf16(rng, (m, n))
        gate = random_bf16(rng, (n,), 0.5)
        kwargs = dict(residual=from_bits(residual), gate=from_bits(gate))
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    got = ops.q6_linear(from_bits(x), wt, st, bt, bias, group_size=gs, apply_gelu=epi == "bias_gelu",
                        path="simt", out=out, **kwargs)
    torch.cuda.synchronize()
    assert ops.last_path() == "simt"
    assert bool(torch.isfinite(got).all())
    ref = oracle.linear(
        oracle.bf16_bits_to_f32(x), w, apply_gelu=epi == "bias_gelu", weight_dtype="f32",
        residual=None if residual is None else oracle.bf16_bits_to_f32(residual),
        gate=None if gate is None else oracle.bf16_bits_to_f32(gate),
    )
    assert_close(f32(got), ref, what=f"gemv {m}x{n}x{k} gs{gs} {epi}")


SKINNY_SHAPES = [
    (12288, 3072, 64),   # the image FF's fc1 shape
    (3072, 12288, 64),   # fc2 shape: 24 stages of 512 codes
    (18432, 3072, 128),  # modulation-linear shape at group size 128
    (1001, 1024, 64),    # ragged N: the last row block is partly out of range
    (2048, 1536, 32),    # group size 32: two scale groups per 64-code block, an odd stage count
]


@pytest.mark.parametrize("m", [1, 2, 3, 8, 13, 16])
@pytest.mark.parametrize("n,k,gs", SKINNY_SHAPES)
@pytest.mark.parametrize("epi", ["plain", "bias_gelu", "residual_gate"])
def test_skinny_path_vs_oracle(m, n, k, gs, epi):
    """The warp-MMA kernel for 1..16 token rows on the raw codes against the
    fp32-weight oracle (the reference kernel's weight precision); the output
    starts as NaN so every element must be written."""

    rng = np.random.default_rng(m * 13 + n + k + gs)
    w = random_weights(rng, n, k, gs, bias=epi != "plain")
    x = random_bf16(rng, (m, k))
    wt, st, bt, bias = weights_to_torch(w)
    kwargs = {}
    residual = gate = None
    if epi == "residual_gate":
        residual = random_bf16(rng, (m, n))
        gate = random_bf16(rng, (n,), 0.5)
        kwargs = dict(residual=from_bits(residual), gate=from_bits(gate))
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    got = ops.q6_linear(from_bits(x), wt, st, bt, bias, group_size=gs, apply_gelu=epi == "bias_gelu",
                        path="skinny", out=out, **kwargs)
    torch.cuda.synchronize()
    assert ops.last_path() == "skinny"
    assert bool(torch.isfinite(got).all())
    ref = oracle.linear(
        oracle.bf16_bits_to_f32(x), w, apply_gelu=epi == "bias_gelu", weight_dtype="f32",
        residual=None if residual is None else oracle.bf16_bits_to_f32(residual),
        gate=None if gate is None else oracle.bf16_bits_to_f32(gate),
    )
    assert_close(f32(got), ref, what=f"skinny {m}x{n}x{k} gs{gs} {epi}")


@pytest.mark.parametrize("m", [5, 16])
def test_skinny_plans_are_reproducible(monkeypatch, m):
    """For a given K split, each output is summed in the same order (the
    CTA's stages in K order within a block warp, the eight block warps in
    order, the cluster's CTAs in rank order) whatever the row-block size and
    the number of clusters, so the results are bitwise equal across those,
    including clusters that walk several row blocks; other splits agree with
    the oracle."""

    rng = np.random.default_rng(6 + m)
    w = random_weights(rng, 4096, 2048, 64)  # four 512-code stages
    wt, st, bt, bias = weights_to_torch(w)
    x = from_bits(random_bf16(rng, (m, 2048)))
    ref = oracle.linear(f32(x), w, weight_dtype="f32")
    by_split = {}
    # tpw 1: 128 row blocks of 32 rows, more than one per cluster at splits 2-4
    for plan in ("1,1", "1,1", "4,1", "2,1", "1,2", "4,2", "2,2", "1,3", "4,3", "4,4", "1,4"):
        monkeypatch.setenv("Q6_SKINNY_PLAN", plan)
        out = ops.q6_linear(x, wt, st, bt, bias, group_size=64, path="skinny")
        by_split.setdefault(plan.split(",")[1], []).append(out)
    torch.cuda.synchronize()
    for split, outs in by_split.items():
        for o in outs[1:]:
            assert torch.equal(outs[0], o), f"split {split}"
        assert_close(f32(outs[0]), ref, what=f"skinny split {split}")


def test_skinny_plan_query(monkeypatch):
    """q6_skinny_plan reports the plan the path launches: the override when
    Q6_SKINNY_PLAN is set, otherwise row blocks that spread the weights over
    the SMs (at least 96 clusters x split CTAs for the image FF's shapes)."""

    monkeypatch.setenv("Q6_SKINNY_PLAN", "3,2")
    plan = ops.skinny_plan(4, 12288, 3072)
    assert (plan["tpw"], plan["rows"], plan["split"]) == (3, 96, 2) and plan["clusters"] >= 1
    monkeypatch.delenv("Q6_SKINNY_PLAN")
    for m in (1, 16):
        for n, k in ((12288, 3072), (3072, 12288)):
            plan = ops.skinny_plan(m, n, k)
            assert 1 <= plan["tpw"] <= 4 and 1 <= plan["split"] <= 4
            assert plan["clusters"] * plan["split"] >= 96, (m, n, k, plan)
    with pytest.raises(_lib.Q6Error):
        ops.skinny_plan(17, 12288, 3072)


def test_skinny_refuses_more_than_16_rows():
    rng = np.random.default_rng(7)
    w = random_weights(rng, 256, 1024, 64)
    wt, st, bt, bias = weights_to_torch(w)
    x = from_bits(random_bf16(rng, (17, 1024)))
    with pytest.raises(_lib.Q6Error):
        ops.q6_linear(x, wt, st, bt, bias, group_size=64, path="skinny")


LORA_CASES = [
    (200, 384, 512, 64, 64, "bias_gelu"),
    (17, 256, 192, 32, 32, "plain"),          # K % 128 == 64 tail before the LoRA stages
    (130, 640, 1024, 128, 64, "residual_gate"),
    (3, 512, 256, 96, 64, "bias_gelu"),       # a few rows: the auto path still takes the fused kernel
    (1000, 3072, 3072, 64, 64, "plain"),      # image-FF width
    (64, 256, 320, 8, 64, "bias_gelu"),       # rank 8: zero-padded to 32 on the host
    (150, 384, 448, 160, 64, "plain"),        # r > 128: each LoRA stage spans both activation boxes
    (40, 512, 1024, 256, 128, "residual_gate"),  # the fused maximum
    (129, 320, 192, 224, 32, "bias_gelu"),    # r > 128 after a K % 128 == 64 tail
]


@pytest.mark.parametrize("m,n,k,r,gs,epi", LORA_CASES)
def test_lora_fused_vs_oracle(m, n, k, r, gs, epi):
    """q6(x) + s * ((x @ A) @ B) with the LoRA product accumulated in the q6
    tile (dense_img_ff_window.py:48-60), against the float64 oracle."""

    rng = np.random.default_rng(m + n + k + r)
    w = random_weights(rng, n, k, gs, bias=epi != "plain")
    x = random_bf16(rng, (m, k))
    a_bits = random_bf16(rng, (k, r), 0.01)
    b_bits = random_bf16(rng, (r, n), 0.01)
    s = 0.75
    wt, st, bt, bias = weights_to_torch(w)
    kwargs = {}
    residual = gate = None
    if epi == "residual_gate":
        residual = random_bf16(rng, (m, n))
        gate = random_bf16(rng, (n,), 0.5)
        kwargs = dict(residual=from_bits(residual), gate=from_bits(gate))
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    got = ops.q6_linear(from_bits(x), wt, st, bt, bias, group_size=gs, apply_gelu=epi == "bias_gelu",
                        lora=(from_bits(a_bits), from_bits(b_bits), s), out=out, **kwargs)
    torch.cuda.synchronize()
    assert ops.last_path() == "tensor"
    assert bool(torch.isfinite(got).all())
    xf = oracle.bf16_bits_to_f32(x)
    res_f = None if residual is None else oracle.bf16_bits_to_f32(residual)
    gate_f = None if gate is None else oracle.bf16_bits_to_f32(gate)
    ref = oracle.linear(xf, w, apply_gelu=epi == "bias_gelu", weight_dtype="bf16", residual=res_f, gate=gate_f,
                        lora=(oracle.bf16_bits_to_f32(a_bits), oracle.bf16_bits_to_f32(b_bits), s))
    assert_close(f32(got), ref, what=f"lora {m}x{n}x{k} r{r} gs{gs} {epi}")
    # the delta is really in the output: without it the oracle moves by more than the tolerance allows
    plain = oracle.linear(xf, w, apply_gelu=epi == "bias_gelu", weight_dtype="bf16", residual=res_f, gate=gate_f)
    assert float(np.abs(ref - plain).max()) > 5e-3 * float(np.abs(ref).max())


def test_lora_rejected_off_the_tensor_path():
    rng = np.random.default_rng(9)
    w = random_weights(rng, 128, 256, 64)
    wt, st, bt, bias = weights_to_torch(w)
    x = from_bits(random_bf16(rng, (8, 256)))
    a = torch.zeros((256, 64), dtype=torch.bfloat16, device="cuda")
    b = torch.zeros((64, 128), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.Q6Error):
        ops.q6_linear(x, wt, st, bt, bias, lora=(a, b, 1.0), path="simt")
    big_a = torch.zeros((256, 288), dtype=torch.bfloat16, device="cuda")
    big_b = torch.zeros((288, 128), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="exceeds"):  # past the two fused LoRA stages
        ops.q6_linear(x, wt, st, bt, bias, lora=(big_a, big_b, 1.0))


def test_auto_path_choice():
    rng = np.random.default_rng(1)
    w = random_weights(rng, 256, 128, 64)
    wt, st, bt, bias = weights_to_torch(w)
    ops.q6_linear(from_bits(random_bf16(rng, (2, 128))), wt, st, bt, bias)
    assert ops.last_path() == "simt"  # small weights, 1-2 rows: the streaming GEMV
    ops.q6_linear(from_bits(random_bf16(rng, (3, 128))), wt, st, bt, bias)
    assert ops.last_path() == "tensor"  # small weights from 3 rows: the tensor-core path
    ops.q6_linear(from_bits(random_bf16(rng, (64, 128))), wt, st, bt, bias)
    assert ops.last_path() == "tensor"
    # weights of 2^24 codes and more: the warp-MMA kernel for 2-16 rows (8 at group size 32)
    for gs, cases in ((64, ((1, "simt"), (2, "skinny"), (16, "skinny"), (17, "tensor"))),
                      (32, ((8, "skinny"), (9, "tensor")))):
        wb = [torch.zeros((4096, 4096 * 6 // 32), dtype=torch.int32, device="cuda"),
              torch.ones((4096, 4096 // gs), dtype=torch.bfloat16, device="cuda"),
              torch.zeros((4096, 4096 // gs), dtype=torch.bfloat16, device="cuda")]
        for m, path in cases:
            ops.q6_linear(torch.ones((m, 4096), dtype=torch.bfloat16, device="cuda"), *wb, group_size=gs)
            assert ops.last_path() == path, (gs, m)
    torch.cuda.synchronize()


def test_mlp_vs_oracle_fused_order():
    rng = np.random.default_rng(21)
    m, d, h = 300, 512, 2048
    fc1 = random_weights(rng, h, d, 64)
    fc2 = random_weights(rng, d, h, 64)
    x = random_bf16(rng, (m, d))
    y = ops.q6_mlp(from_bits(x), weights_to_torch(fc1), weights_to_torch(fc2), group_size=64)
    torch.cuda.synchronize()
    ref = oracle.fused_mlp(oracle.bf16_bits_to_f32(x), fc1, fc2)
    assert_close(f32(y), ref)
    eager = oracle.eager_mlp(oracle.bf16_bits_to_f32(x), fc1, fc2)
    assert float(np.abs(f32(y) - eager).max()) < 0.05


def test_mlp_split_k_workspace():
    """A text-stream-sized MLP (few hundred tokens, fc2 with K = H): the fused
    MLP's workspace past the hidden activations lets both linears split K;
    with the hidden activations only, they do not.  Both agree with the oracle."""

    rng = np.random.default_rng(22)
    m, d, h = 256, 512, 4096
    assert ops.mlp_workspace_bytes(m, h, d) > ops.mlp_workspace_bytes(m, h)  # split-K space planned
    fc1 = random_weights(rng, h, d, 64)
    fc2 = random_weights(rng, d, h, 64)
    x = random_bf16(rng, (m, d))
    residual = random_bf16(rng, (m, d))
    gate = random_bf16(rng, (d,), 0.5)
    args = (from_bits(x), weights_to_torch(fc1), weights_to_torch(fc2))
    kw = dict(group_size=64, residual=from_bits(residual), gate=from_bits(gate))
    y_split = ops.q6_mlp(*args, **kw)
    base_ws = torch.empty(ops.mlp_workspace_bytes(m, h), dtype=torch.uint8, device="cuda")
    y_plain = ops.q6_mlp(*args, workspace=base_ws, **kw)
    torch.cuda.synchronize()
    hid = oracle.round_bf16(oracle.linear(oracle.bf16_bits_to_f32(x), fc1, apply_gelu=True))
    ref = oracle.linear(hid, fc2, residual=oracle.bf16_bits_to_f32(residual), gate=oracle.bf16_bits_to_f32(gate))
    assert_close(f32(y_split), ref, what="mlp split-K workspace")
    assert_close(f32(y_plain), ref, what="mlp hidden-only workspace")


def test_mlp_image_ff_full_size_rows_sample():
    """Config-2 shapes (3456 tokens, 3072 -> 12288 -> 3072): full run on the GPU,
    oracle on a sample of rows (each output row depends only on its input row)."""

    rng = np.random.default_rng(2)
    m, d, h = 3456, 3072, 12288
    fc1 = random_weights(rng, h, d, 64)
    fc2 = random_weights(rng, d, h, 64)
    x = random_bf16(rng, (m, d))
    y = ops.q6_mlp(from_bits(x), weights_to_torch(fc1), weights_to_torch(fc2), group_size=64)
    torch.cuda.synchronize()
    rows = np.sort(rng.choice(m, size=48, replace=False))
    rows[0], rows[-1] = 0, m - 1
    ref = oracle.fused_mlp(oracle.bf16_bits_to_f32(x[rows]), fc1, fc2)
    assert_close(f32(y)[rows], ref)


def test_dropin_feed_forward_module():
    from qwen_image_shardedit_mlx_b200 import QwenFeedForward, make_feed_forward_callables

    g = torch.Generator(device="cuda").manual_seed(0)
    ff = QwenFeedForward.random(256, 1024, generator=g)
    x = torch.randn((1, 12, 256), generator=g, device="cuda").to(torch.bfloat16)
    eager, fused, dense = make_feed_forward_callables(ff)
    ye, yf, yd = eager(x), fused(x), dense(x)
    assert yf.shape == (1, 12, 256) and yf.dtype == torch.bfloat16
    assert float((ye.float() - yf.float()).abs().max()) < 0.05
    assert float((yd.float() - yf.float()).abs().max()) < 0.05
    assert torch.equal(ff(x), yf)


SPLITK_CASES = [
    # (M, N, K, gs, epi, forced splits or None for the planner's choice)
    (16, 3072, 12288, 64, "plain", None),         # 24 weight tiles: the planner splits K
    (16, 12288, 3072, 64, "bias_gelu", 3),
    (200, 640, 3072, 64, "residual_gate", 3),
    (37, 256, 1536, 32, "bias_gelu", 2),          # scale chunks of 2 stages
    (40, 384, 2048, 128, "plain", 2),             # scale chunks of 8 stages
    (24, 256, 1088, 64, "plain", 2),              # K % 128 == 64: the tail stage in the last split
    (24, 256, 1216, 64, "bias_gelu", 2),          # K / gs % 8 != 0: per-lane scale loads
]


@pytest.mark.parametrize("m,n,k,gs,epi,splits", SPLITK_CASES)
def test_split_k_vs_oracle(m, n, k, gs, epi, splits, monkeypatch):
    """Split-K on the tensor-core path: fp32 partials per K split, summed in
    split order by the reduce kernel, which applies the epilogue."""

    if splits is not None:
        monkeypatch.setenv("Q6_TC_KSPLIT", str(splits))
    lib = _lib.lib()
    assert lib.q6_linear_tc_workspace_bytes(m, n, k) > 0
    rng = np.random.default_rng(m + n + k + gs)
    w = random_weights(rng, n, k, gs, bias=epi != "plain")
    x = random_bf16(rng, (m, k))
    wt, st, bt, bias = weights_to_torch(w)
    kwargs = {}
    residual = gate = None
    if epi == "residual_gate":
        residual = random_bf16(rng, (m, n))
        gate = random_bf16(rng, (n,), 0.5)
        kwargs = dict(residual=from_bits(residual), gate=from_bits(gate))
    outs = []
    for _ in range(2):
        out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        outs.append(ops.q6_linear(from_bits(x), wt, st, bt, bias, group_size=gs, apply_gelu=epi == "bias_gelu",
                                  path="tensor", out=out, **kwargs))
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])  # the split order is fixed: bitwise reproducible
    assert bool(torch.isfinite(outs[0]).all())
    ref = oracle.linear(
        oracle.bf16_bits_to_f32(x), w, apply_gelu=epi == "bias_gelu", weight_dtype="bf16",
        residual=None if residual is None else oracle.bf16_bits_to_f32(residual),
        gate=None if gate is None else oracle.bf16_bits_to_f32(gate),
    )
    assert_close(f32(outs[0]), ref, what=f"splitk {m}x{n}x{k} gs{gs} {epi} s{splits}")


@pytest.mark.parametrize("r", [64, 256])
def test_split_k_with_lora(monkeypatch, r):
    monkeypatch.setenv("Q6_TC_KSPLIT", "2")
    rng = np.random.default_rng(77 + r)
    m, n, k, gs = 64, 512, 2048, 64
    w = random_weights(rng, n, k, gs)
    x = random_bf16(rng, (m, k))
    a_bits = random_bf16(rng, (k, r), 0.01)
    b_bits = random_bf16(rng, (r, n), 0.01)
    wt, st, bt, bias = weights_to_torch(w)
    got = ops.q6_linear(from_bits(x), wt, st, bt, bias, group_size=gs,
                        lora=(from_bits(a_bits), from_bits(b_bits), 0.5))
    torch.cuda.synchronize()
    ref = oracle.linear(oracle.bf16_bits_to_f32(x), w, weight_dtype="bf16",
                        lora=(oracle.bf16_bits_to_f32(a_bits), oracle.bf16_bits_to_f32(b_bits), 0.5))
    assert_close(f32(got), ref, what=f"splitk lora r{r}")


PAIR_CASES = [
    # (m, n, k, gs, epi, token tile, lora rank)
    (3456, 1536, 1024, 128, "bias_gelu", 192, 0),  # the image-FF token count
    (700, 640, 512, 32, "residual_gate", 128, 0),  # N % 256 != 0: the second CTA of the last pair is idle
    (513, 384, 1088, 64, "plain", 256, 0),         # ragged M, K % 128 == 64, scales not staged (17 groups)
    (300, 512, 768, 64, "plain", 128, 64),         # LoRA stages: each CTA stages half of x @ A
]


@pytest.mark.parametrize("m,n,k,gs,epi,tile,r", PAIR_CASES)
def test_cta_pair_mode(m, n, k, gs, epi, tile, r, monkeypatch):
    """CTA pairs (Q6_TC_PAIR=1): one cta_group::2 MMA per 256 weight rows,
    each CTA staging half of the token rows.  The accumulation order per
    output is the single-CTA one (split-K off, which pairs never use), so
    the outputs are bitwise equal."""

    monkeypatch.setenv("Q6_TC_TOKEN_TILE", str(tile))
    monkeypatch.setenv("Q6_TC_KSPLIT", "1")
    rng = np.random.default_rng(m + n + k + r)
    w = random_weights(rng, n, k, gs, bias=epi != "plain")
    x = random_bf16(rng, (m, k))
    wt, st, bt, bias = weights_to_torch(w)
    kwargs = {}
    residual = gate = lora_ref = None
    if epi == "residual_gate":
        residual = random_bf16(rng, (m, n))
        gate = random_bf16(rng, (n,), 0.5)
        kwargs = dict(residual=from_bits(residual), gate=from_bits(gate))
    if r:
        a_bits, b_bits = random_bf16(rng, (k, r), 0.02), random_bf16(rng, (r, n), 0.02)
        kwargs["lora"] = (from_bits(a_bits), from_bits(b_bits), 0.75)
        lora_ref = (oracle.bf16_bits_to_f32(a_bits), oracle.bf16_bits_to_f32(b_bits), 0.75)
    outs = {}
    for pair in ("0", "1"):
        monkeypatch.setenv("Q6_TC_PAIR", pair)
        out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        outs[pair] = ops.q6_linear(from_bits(x), wt, st, bt, bias, group_size=gs, apply_gelu=epi == "bias_gelu",
                                   path="tensor", out=out, **kwargs)
    torch.cuda.synchronize()
    assert torch.equal(outs["0"], outs["1"])
    ref = oracle.linear(
        oracle.bf16_bits_to_f32(x), w, apply_gelu=epi == "bias_gelu", weight_dtype="bf16",
        residual=None if residual is None else oracle.bf16_bits_to_f32(residual),
        gate=None if gate is None else oracle.bf16_bits_to_f32(gate), lora=lora_ref,
    )
    assert_close(f32(outs["1"]), ref, what=f"pair {m}x{n}x{k} gs{gs} {epi} nt{tile} r{r}")


def test_split_k_reduce_vector_matches_scalar(monkeypatch):
    """The split-K reduce takes 16-byte loads and stores when N % 8 == 0 and
    every operand is 16-byte aligned; an output two bytes off that alignment
    takes the one-element-per-thread kernel.  Same sums in the same order:
    bitwise equal outputs."""

    monkeypatch.setenv("Q6_TC_KSPLIT", "3")
    rng = np.random.default_rng(31)
    m, n, k = 200, 512, 3072
    w = random_weights(rng, n, k, 64)
    wt, st, bt, bias = weights_to_torch(w)
    x = from_bits(random_bf16(rng, (m, k)))
    residual = from_bits(random_bf16(rng, (m, n)))
    gate = from_bits(random_bf16(rng, (n,), 0.5))
    outs = []
    for off in (0, 1):
        buf = torch.full((m * n + 8,), float("nan"), dtype=torch.bfloat16, device="cuda")
        out = buf[off:off + m * n].view(m, n)
        outs.append(ops.q6_linear(x, wt, st, bt, bias, group_size=64, apply_gelu=True, residual=residual,
                                  gate=gate, path="tensor", out=out))
    torch.cuda.synchronize()
    assert bool(torch.isfinite(outs[0]).all())
    assert torch.equal(outs[0], outs[1])
