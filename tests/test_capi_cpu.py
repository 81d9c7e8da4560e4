"""C-ABI boundary checks that need no GPU: the library loads, exports every
symbol include/q6_b200.h declares, and rejects bad arguments with the right
status codes before touching the device."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from qwen_image_shardedit_mlx_b200 import _lib
from qwen_image_shardedit_mlx_b200.quantize import pack_codes, quantize_affine_q6, unpack_codes

HEADER = Path(__file__).resolve().parents[1] / "include" / "q6_b200.h"


def _declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"Q6_API\s+[a-z0-9_ ]+\*?\s*(q6_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_expected_entry_points():
    names = _declared_symbols()
    for required in ("q6_linear_bf16", "q6_mlp_bf16", "q6_dequantize_bf16", "q6_linear_f32"):
        assert required in names
    assert set(names) == set(_lib.SIGNATURES), "ctypes table and header disagree"


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in _declared_symbols():
        assert hasattr(lib, name), name
    assert lib.q6_abi_version() == 2


def test_status_strings():
    for code in range(0, 9):
        assert _lib.status_string(code)
    assert "group_size" in _lib.status_string(_lib.Q6_ERR_GROUP_SIZE)


def test_workspace_sizes():
    lib = _lib.lib()
    assert lib.q6_mlp_workspace_bytes(3456, 12288) == 3456 * 12288 * 2
    assert lib.q6_mlp_workspace_bytes(0, 12288) == 0


def _linear(lib, **kw):
    args = dict(x=256, w=256, scales=256, qbiases=256, bias=None, residual=None, gate=None, lora_xa=None,
                lora_b=None, lora_scale=0.0, rank=0, y=256, M=4, N=128, K=64, gs=64, flags=0, path=0, ws=None, ws_bytes=0,
                stream=None)
    args.update(kw)
    return lib.q6_linear_bf16(*args.values())


def test_argument_validation_without_gpu():
    lib = _lib.lib()
    assert _linear(lib, x=None) == _lib.Q6_ERR_INVALID_ARGUMENT
    assert _linear(lib, w=None) == _lib.Q6_ERR_INVALID_ARGUMENT
    assert _linear(lib, M=0) == _lib.Q6_ERR_INVALID_ARGUMENT
    assert _linear(lib, gs=16) == _lib.Q6_ERR_GROUP_SIZE
    assert _linear(lib, K=96, gs=64) == _lib.Q6_ERR_SHAPE
    assert _linear(lib, flags=8) == _lib.Q6_ERR_INVALID_ARGUMENT
    assert _linear(lib, flags=4) == _lib.Q6_ERR_INVALID_ARGUMENT  # transposed LoRA B without a LoRA
    assert _linear(lib, flags=16) == _lib.Q6_ERR_INVALID_ARGUMENT
    assert _linear(lib, flags=4, lora_xa=256, lora_b=264, rank=64) == _lib.Q6_ERR_INVALID_ARGUMENT  # B not 16-aligned
    assert _linear(lib, w=258) == _lib.Q6_ERR_ALIGNMENT
    # LoRA: x @ A and B come together, with a positive rank
    assert _linear(lib, lora_xa=256) == _lib.Q6_ERR_INVALID_ARGUMENT
    assert _linear(lib, lora_b=256, rank=64) == _lib.Q6_ERR_INVALID_ARGUMENT
    assert _linear(lib, lora_xa=256, lora_b=256, rank=0) == _lib.Q6_ERR_INVALID_ARGUMENT
    assert lib.q6_dequantize_bf16(None, 1, 1, 1, 4, 64, 64, None) == _lib.Q6_ERR_INVALID_ARGUMENT
    # q6_mlp needs a workspace large enough for the hidden activations
    st = lib.q6_mlp_bf16(16, 16, 16, 16, None, 16, 16, 16, None, None, None, 16, 8, 64, 256, 64, None, 0, None)
    assert st == _lib.Q6_ERR_WORKSPACE
    err = ctypes.c_int(0)
    assert lib.q6_get_device_error(None) == _lib.Q6_ERR_INVALID_ARGUMENT
    del err
    # LoRA pre-pass: rank a multiple of 32 in [32, 256], K a multiple of 16, 16-byte alignment
    assert lib.q6_lora_xa_bf16(None, 16, 16, 4, 64, 64, None) == _lib.Q6_ERR_INVALID_ARGUMENT
    assert lib.q6_lora_xa_bf16(16, 16, 16, 4, 64, 48, None) == _lib.Q6_ERR_SHAPE
    assert lib.q6_lora_xa_bf16(16, 16, 16, 4, 64, 288, None) == _lib.Q6_ERR_SHAPE
    assert lib.q6_lora_xa_bf16(16, 16, 16, 4, 72, 64, None) == _lib.Q6_ERR_SHAPE
    assert lib.q6_lora_xa_bf16(18, 16, 16, 4, 64, 64, None) == _lib.Q6_ERR_ALIGNMENT
    # joint-row add + adaLN modulate
    add_ln = lib.q6_add_layernorm_modulate_bf16
    inval, shape, align = _lib.Q6_ERR_INVALID_ARGUMENT, _lib.Q6_ERR_SHAPE, _lib.Q6_ERR_ALIGNMENT
    assert add_ln(16, None, 16, 16, 16, 0, 16, 4, 256, 0, 0, 0, 1e-6, None) == inval  # h_out without add
    assert add_ln(16, 16, None, 16, 16, 0, 16, 4, 256, 0, 10, 20, 1e-6, None) == inval  # text_len > seq_len
    assert add_ln(16, 16, None, 16, 16, 0, 16, 4, 320, 0, 0, 0, 1e-6, None) == shape
    assert add_ln(16, 24, None, 16, 16, 0, 16, 4, 256, 0, 0, 0, 1e-6, None) == align
    assert add_ln(16, 16, None, 16, 16, 128, 16, 4, 256, 0, 0, 0, 1e-6, None) == inval  # vector stride < D
    assert add_ln(16, 16, None, 16, 16, 260, 16, 4, 256, 0, 0, 0, 1e-6, None) == align  # stride not 8-aligned
    # sequence-parallel modulate + gather: the same vector-stride rules
    sp = lib.q6_sp_add_layernorm_gather_bf16
    one = (ctypes.c_void_p * 1)(16)
    assert sp(16, None, None, 16, 16, 128, one, 1, 0, 4, 256, 0, 0, 1e-6, None) == inval
    assert sp(16, None, None, 16, 16, 260, one, 1, 0, 4, 256, 0, 0, 1e-6, None) == align
    assert sp(16, None, None, 16, 16, 0, one, 2, 2, 4, 256, 0, 0, 1e-6, None) == inval  # rank >= world
    # self-test limits: 1 us .. 1 s
    assert lib.q6_selftest_bounded_wait(10, None) == _lib.Q6_ERR_INVALID_ARGUMENT
    assert lib.q6_selftest_bounded_wait(2_000_000_000, None) == _lib.Q6_ERR_INVALID_ARGUMENT
    assert lib.q6_pair_fallback_count() == 0


def test_torch_quantizer_matches_oracle_bit_for_bit():
    rng = np.random.default_rng(11)
    for gs in (32, 64, 128):
        w = rng.normal(0.0, 0.02, size=(40, 384)).astype(np.float32)
        packed, scales, biases = oracle.affine_quantize(w, group_size=gs)
        tq, ts, tb = quantize_affine_q6(torch.from_numpy(w), gs)
        assert np.array_equal(tq.view(torch.int32).numpy().view(np.uint32), packed)
        assert np.array_equal(ts.view(torch.int16).numpy().view(np.uint16), scales)
        assert np.array_equal(tb.view(torch.int16).numpy().view(np.uint16), biases)


def test_torch_pack_unpack_roundtrip():
    g = torch.Generator().manual_seed(1)
    codes = torch.randint(0, 64, (7, 256), generator=g)
    packed = pack_codes(codes)
    assert packed.dtype == torch.uint32 and packed.shape == (7, 48)
    assert torch.equal(unpack_codes(packed, 256), codes)
    ref = oracle.pack_q6(codes.numpy().astype(np.uint8))
    assert np.array_equal(packed.view(torch.int32).numpy().view(np.uint32), ref)


def test_ops_refuse_cpu_tensors():
    from qwen_image_shardedit_mlx_b200 import ops

    w, s, b = quantize_affine_q6(torch.randn(128, 64) * 0.02, 64)
    x = torch.randn(4, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.q6_linear(x, w, s, b)


def test_python_surface_validation_errors():
    from qwen_image_shardedit_mlx_b200 import Q6LinearSpec, affine_q6_qmm_t, quantized_linear_spec

    w, s, b = quantize_affine_q6(torch.randn(128, 64) * 0.02, 64)
    spec = Q6LinearSpec(w, s, b, None, 64, 6)
    assert spec.in_features == 64 and spec.out_features == 128
    with pytest.raises(ValueError, match="rank 2 or 3"):
        affine_q6_qmm_t(torch.zeros(2, 2, 2, 64), spec)
    with pytest.raises(ValueError, match="in_features"):
        affine_q6_qmm_t(torch.zeros(2, 32), spec)

    class Layer:
        weight = w
        scales = s
        biases = b
        bits = 4
        group_size = 64

    with pytest.raises(ValueError, match="bits=6"):
        quantized_linear_spec(Layer())
