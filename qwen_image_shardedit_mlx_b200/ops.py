"""Torch-facing q6 ops; every call goes through the C ABI of libq6b200.so.

Tensors must live on a CUDA device.  Launches are ordered on the current torch
stream of that device; nothing here synchronises.  Output buffers are
allocated with torch (the library itself never allocates).
"""

from __future__ import annotations

import ctypes

import torch

from qwen_image_shardedit_mlx_b200 import _lib
from qwen_image_shardedit_mlx_b200.lora import MAX_FUSED_RANK, pad_lora_rank

GROUP_SIZES = (32, 64, 128)


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _as_u32(weight: torch.Tensor) -> torch.Tensor:
    if weight.dtype not in (torch.uint32, torch.int32):
        raise ValueError(f"expected packed uint32 weight, got {weight.dtype}")
    return weight


def _require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("q6 ops run on CUDA tensors only (the library has no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all tensors must be on the same device")
    assert dev is not None
    return dev


def _bf16_vec(t: torch.Tensor | None, n: int, name: str) -> torch.Tensor | None:
    if t is None:
        return None
    t = t.reshape(-1)
    if t.numel() != n:
        raise ValueError(f"{name} must hold {n} values, got {t.numel()}")
    return t.to(torch.bfloat16).contiguous()


def check_q6_weights(weight: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group_size: int) -> tuple[int, int]:
    """Validate the MLX q6 triplet; returns (N, K)."""

    _as_u32(weight)
    if group_size not in GROUP_SIZES:
        raise ValueError(f"group_size must be one of {GROUP_SIZES}, got {group_size}")
    if weight.dim() != 2:
        raise ValueError(f"packed weight must be 2-D, got shape {tuple(weight.shape)}")
    n = int(weight.shape[0])
    if (int(weight.shape[1]) * 32) % 6:
        raise ValueError(f"packed width {weight.shape[1]} is not a whole number of 6-bit codes")
    k = int(weight.shape[1]) * 32 // 6
    if k % group_size:
        raise ValueError(f"in_features {k} is not a multiple of group_size {group_size}")
    expect = (n, k // group_size)
    if tuple(scales.shape) != expect or tuple(biases.shape) != expect:
        raise ValueError(f"scales/biases must be {expect}, got {tuple(scales.shape)} / {tuple(biases.shape)}")
    return n, k


def q6_dequantize(weight: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group_size: int = 64) -> torch.Tensor:
    """Dense bf16 [N, K] = bf16_rn(scale * q + bias) (MLX affine dequantisation)."""

    n, k = check_q6_weights(weight, scales, biases, group_size)
    dev = _require_cuda(weight, scales, biases)
    out = torch.empty((n, k), dtype=torch.bfloat16, device=dev)
    st = _lib.lib().q6_dequantize_bf16(
        weight.contiguous().data_ptr(),
        scales.to(torch.bfloat16).contiguous().data_ptr(),
        biases.to(torch.bfloat16).contiguous().data_ptr(),
        out.data_ptr(), n, k, group_size, _stream(dev),
    )
    _lib.check(st, "q6_dequantize_bf16")
    return out


def q6_linear(
    x: torch.Tensor,
    weight: torch.Tensor,
    scales: torch.Tensor,
    biases: torch.Tensor,
    bias: torch.Tensor | None = None,
    *,
    group_size: int = 64,
    apply_gelu: bool = False,
    residual: torch.Tensor | None = None,
    gate: torch.Tensor | None = None,
    lora: tuple[torch.Tensor, torch.Tensor, float] | None = None,
    path: str = "auto",
    out: torch.Tensor | None = None,
    precise_gelu: bool = False,
    lora_b_nmajor: torch.Tensor | None = None,
) -> torch.Tensor:
    """y = epilogue(x @ dequant(W)^T) for x [..., K]; returns [..., N].

    bf16 x runs the tensor-core path (bf16-dequantised weights, fp32
    accumulation) or, for a handful of rows, the CUDA-core path; fp32 x runs
    the CUDA-core path with fp32 weights and returns fp32.
    Epilogue order: + bias, GELU, then residual + gate * value.  The tensor
    path's GELU takes the hardware tanh approximation unless ``precise_gelu``
    asks for the accurate tanh the reference kernel uses.  ``lora_b_nmajor``
    (optional) is the LoRA B transposed to [N, r_padded] (``lora_b_nmajor``
    of a ``QuantizedLinear``), which the fused LoRA stages read with 16-byte
    loads.
    """

    n, k = check_q6_weights(weight, scales, biases, group_size)
    if x.shape[-1] != k:
        raise ValueError(f"x in_features {x.shape[-1]} != weight in_features {k}")
    dev = _require_cuda(x, weight, scales, biases, bias, residual, gate)
    leading = tuple(x.shape[:-1])
    flat = x.reshape(-1, k)
    m = int(flat.shape[0])
    if m == 0:
        return torch.empty(leading + (n,), dtype=x.dtype, device=dev)
    flags = _lib.Q6_EPI_NONE
    if apply_gelu:
        flags = _lib.Q6_EPI_GELU | (_lib.Q6_EPI_GELU_PRECISE if precise_gelu else 0)
    sc = scales.to(torch.bfloat16).contiguous()
    qb = biases.to(torch.bfloat16).contiguous()
    bias_t = _bf16_vec(bias, n, "bias")
    gate_t = _bf16_vec(gate, n, "gate")
    w = weight.contiguous()
    stream = _stream(dev)
    if flat.dtype == torch.float32:
        if residual is not None or gate is not None or lora is not None:
            raise ValueError("the fp32 path supports bias and GELU only")
        xf = flat.contiguous()
        y = out if out is not None else torch.empty((m, n), dtype=torch.float32, device=dev)
        st = _lib.lib().q6_linear_f32(
            xf.data_ptr(), w.data_ptr(), sc.data_ptr(), qb.data_ptr(), _ptr(bias_t), y.data_ptr(),
            m, n, k, group_size, flags, stream,
        )
        _lib.check(st, "q6_linear_f32")
        return y.reshape(leading + (n,))
    if flat.dtype != torch.bfloat16:
        flat = flat.to(torch.bfloat16)
    xb = flat.contiguous()
    res_t = None
    if residual is not None:
        res_t = residual.reshape(m, n).to(torch.bfloat16).contiguous()
    xa = lb = None
    lscale, rank = 0.0, 0
    if lora is not None:
        a, b, lscale = lora
        rank = int(a.shape[-1])
        la = a.to(device=dev, dtype=torch.bfloat16)
        lb = b.to(device=dev, dtype=torch.bfloat16).contiguous()
        if tuple(la.shape) != (k, rank) or tuple(lb.shape) != (rank, n) or rank == 0:
            raise ValueError(f"LoRA A must be ({k}, r) and B (r, {n}); got {tuple(la.shape)}, {tuple(lb.shape)}")
        if rank > MAX_FUSED_RANK:
            raise ValueError(f"LoRA rank {rank} exceeds the fused maximum {MAX_FUSED_RANK}")
        la, lb = pad_lora_rank(la, lb)  # the kernel takes ranks in steps of 32
        rank = int(la.shape[1])
        if (lora_b_nmajor is not None and tuple(lora_b_nmajor.shape) == (n, rank)
                and lora_b_nmajor.dtype == torch.bfloat16 and lora_b_nmajor.is_contiguous()
                and lora_b_nmajor.device == lb.device and lora_b_nmajor.data_ptr() % 16 == 0):
            lb = lora_b_nmajor
            flags |= _lib.Q6_LORA_B_NMAJOR
        # x @ A (fp32 accumulation, bf16 result, as the reference's LoRA
        # linear computes it) by the library's pre-pass kernel; the q6 kernel
        # then fuses s * (xa @ B) into its own accumulator.
        xa = lora_xa(xb, la.contiguous())
    y = out if out is not None else torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    # split-K workspace for the tensor-core path when its tiles alone leave SMs idle
    ws_bytes = int(_lib.lib().q6_linear_tc_workspace_bytes(m, n, k)) if path != "simt" else 0
    workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
    st = _lib.lib().q6_linear_bf16(
        xb.data_ptr(), w.data_ptr(), sc.data_ptr(), qb.data_ptr(), _ptr(bias_t), _ptr(res_t), _ptr(gate_t),
        _ptr(xa), _ptr(lb), float(lscale), rank, y.data_ptr(), m, n, k, group_size, flags,
        _lib.PATHS[path], _ptr(workspace), ws_bytes, stream,
    )
    _lib.check(st, "q6_linear_bf16")
    return y.reshape(leading + (n,))


def lora_xa(x: torch.Tensor, a: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """xa = x @ A for x bf16 [M, K] and A bf16 [K, r] (r a multiple of 32 up
    to 256): the LoRA pre-pass kernel, fp32 accumulation, bf16 result."""

    dev = _require_cuda(x, a)
    m, k = int(x.shape[0]), int(x.shape[1])
    r = int(a.shape[1])
    if tuple(a.shape) != (k, r):
        raise ValueError(f"A must be ({k}, r), got {tuple(a.shape)}")
    xb = x.to(torch.bfloat16).contiguous()
    ab = a.to(torch.bfloat16).contiguous()
    y = out if out is not None else torch.empty((m, r), dtype=torch.bfloat16, device=dev)
    _lib.check(_lib.lib().q6_lora_xa_bf16(xb.data_ptr(), ab.data_ptr(), y.data_ptr(), m, k, r, _stream(dev)),
               "q6_lora_xa_bf16")
    return y


def selftest_bounded_wait(limit_ns: int = 1_000_000, device: torch.device | str | None = None) -> int:
    """Run the library's bounded-wait self-test on ``device`` and return the
    device error word afterwards (Q6_SITE_SELFTEST when the wait gave up as
    designed).  Clears nothing: call clear_device_error() after reading it."""

    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().q6_selftest_bounded_wait(int(limit_ns), _stream(dev)), "q6_selftest_bounded_wait")
        return device_error()


def pair_fallback_count() -> int:
    """Tensor-path launches whose CTA-pair cluster the device refused (they ran one CTA per tile)."""

    return int(_lib.lib().q6_pair_fallback_count())


def mlp_workspace_bytes(m: int, h: int, d: int | None = None) -> int:
    """Bytes of device workspace q6_mlp needs for m tokens and hidden width h
    (the bf16 hidden activations).  With the model width d it also counts the
    split-K space of the two linears, placed from the next 256-byte boundary,
    which lets a few-hundred-token MLP spread its K loop over idle SMs."""

    base = int(_lib.lib().q6_mlp_workspace_bytes(int(m), int(h)))
    if d is None:
        return base
    lib = _lib.lib()
    split = max(int(lib.q6_linear_tc_workspace_bytes(int(m), int(h), int(d))),
                int(lib.q6_linear_tc_workspace_bytes(int(m), int(d), int(h))))
    return (base + 255) // 256 * 256 + split if split else base


def q6_mlp(
    x: torch.Tensor,
    w1: tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor | None],
    w2: tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor | None],
    *,
    group_size: int = 64,
    residual: torch.Tensor | None = None,
    gate: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """fc2(gelu(fc1(x))) [+ residual + gate * .]; w1/w2 = (weight, scales, biases, bias)."""

    h, d = check_q6_weights(w1[0], w1[1], w1[2], group_size)
    d2, h2 = check_q6_weights(w2[0], w2[1], w2[2], group_size)
    if (d2, h2) != (d, h):
        raise ValueError(f"fc2 must map {h} -> {d}, got {h2} -> {d2}")
    if x.shape[-1] != d:
        raise ValueError(f"x features {x.shape[-1]} != {d}")
    dev = _require_cuda(x, *w1[:3], *w2[:3])
    leading = tuple(x.shape[:-1])
    xb = x.reshape(-1, d).to(torch.bfloat16).contiguous()
    m = int(xb.shape[0])
    # a caller's workspace needs the hidden activations at least; one made here
    # also holds the linears' split-K space
    if workspace is None or workspace.numel() * workspace.element_size() < mlp_workspace_bytes(m, h):
        workspace = torch.empty(mlp_workspace_bytes(m, h, d), dtype=torch.uint8, device=dev)
    y = out if out is not None else torch.empty((m, d), dtype=torch.bfloat16, device=dev)
    res_t = None if residual is None else residual.reshape(m, d).to(torch.bfloat16).contiguous()
    gate_t = _bf16_vec(gate, d, "gate")
    b1 = _bf16_vec(w1[3], h, "fc1 bias")
    b2 = _bf16_vec(w2[3], d, "fc2 bias")
    st = _lib.lib().q6_mlp_bf16(
        xb.data_ptr(),
        w1[0].contiguous().data_ptr(), w1[1].to(torch.bfloat16).contiguous().data_ptr(),
        w1[2].to(torch.bfloat16).contiguous().data_ptr(), _ptr(b1),
        w2[0].contiguous().data_ptr(), w2[1].to(torch.bfloat16).contiguous().data_ptr(),
        w2[2].to(torch.bfloat16).contiguous().data_ptr(), _ptr(b2),
        _ptr(res_t), _ptr(gate_t), y.data_ptr(), m, d, h, group_size,
        workspace.data_ptr(), workspace.numel() * workspace.element_size(), _stream(dev),
    )
    _lib.check(st, "q6_mlp_bf16")
    return y.reshape(leading + (d,))


class MlpCall:
    """A prepared ``q6_mlp`` for fixed weights, row count and workspace: the
    checks, dtype views and pointer lookups run once, and each call passes
    only the activation and output pointers and the stream to the C ABI.  For
    loops that launch the same MLP on rotating device buffers (the streamed
    host-batch path), where the per-call Python work of ``q6_mlp`` would
    otherwise pace the GPU.  The weight and workspace tensors are kept alive
    by the object; they must not be reallocated while it is in use."""

    def __init__(self, w1, w2, m: int, group_size: int, workspace: torch.Tensor):
        h, d = check_q6_weights(w1[0], w1[1], w1[2], group_size)
        d2, h2 = check_q6_weights(w2[0], w2[1], w2[2], group_size)
        if (d2, h2) != (d, h):
            raise ValueError(f"fc2 must map {h} -> {d}, got {h2} -> {d2}")
        dev = _require_cuda(*w1[:3], *w2[:3], workspace)
        if workspace.numel() * workspace.element_size() < mlp_workspace_bytes(m, h):
            raise ValueError("workspace smaller than mlp_workspace_bytes(m, h)")
        self.m, self.d, self.h, self.group_size, self.device = int(m), d, h, group_size, dev
        self._keep = [w1[0].contiguous(), w1[1].to(torch.bfloat16).contiguous(), w1[2].to(torch.bfloat16).contiguous(),
                      _bf16_vec(w1[3], h, "fc1 bias"),
                      w2[0].contiguous(), w2[1].to(torch.bfloat16).contiguous(), w2[2].to(torch.bfloat16).contiguous(),
                      _bf16_vec(w2[3], d, "fc2 bias"), workspace]
        k = self._keep
        self._w = (k[0].data_ptr(), k[1].data_ptr(), k[2].data_ptr(), _ptr(k[3]),
                   k[4].data_ptr(), k[5].data_ptr(), k[6].data_ptr(), _ptr(k[7]))
        self._tail = (self.m, d, h, group_size, workspace.data_ptr(), workspace.numel() * workspace.element_size())
        self._fn = _lib.lib().q6_mlp_bf16

    def __call__(self, x_ptr: int, y_ptr: int, stream: int) -> None:
        """y = fc2(gelu(fc1(x))) for bf16 [m, d] device buffers given by pointer, on ``stream`` (a raw handle)."""
        _lib.check(self._fn(x_ptr, *self._w, None, None, y_ptr, *self._tail, stream), "q6_mlp_bf16")


def skinny_plan(m: int, n: int, k: int, group_size: int = 64) -> dict:
    """The plan the few-row path would launch for an m x n x k linear on the
    current device: 16-row weight tiles per warp, CTAs per cluster sharing K,
    clusters."""
    tpw, split, clusters = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
    _lib.check(_lib.lib().q6_skinny_plan(m, n, k, group_size, ctypes.byref(tpw), ctypes.byref(split),
                                         ctypes.byref(clusters)), "q6_skinny_plan")
    return {"tpw": tpw.value, "rows": 32 * tpw.value, "split": split.value, "clusters": clusters.value}


def last_path() -> str:
    code = _lib.lib().q6_last_path()
    return {v: k for k, v in _lib.PATHS.items()}.get(code, "none")


def device_error() -> int:
    code = ctypes.c_int(0)
    _lib.check(_lib.lib().q6_get_device_error(ctypes.byref(code)), "q6_get_device_error")
    return int(code.value)


def clear_device_error() -> None:
    _lib.check(_lib.lib().q6_clear_device_error(), "q6_clear_device_error")
