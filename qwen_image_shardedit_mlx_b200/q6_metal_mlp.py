"""Reference-compatible q6 linear / image-MLP surface, backed by the B200 kernels.

Mirrors the names, argument meanings and errors of the reference module
shardedit_mlx/q6_metal_mlp.py so callers can switch by import:

=========================  =====================================================
reference (file:line)      here
=========================  =====================================================
Q6LinearSpec :96-111       Q6LinearSpec (weight uint32 [N, K*6/32], scales and
                           qbiases [N, K/gs], optional bias, group_size, bits)
quantized_linear_spec      quantized_linear_spec(layer): bits must be 6 and the
:114-134                   weight uint32, else ValueError
DenseLinearWeights :137    DenseLinearWeights(weight [N, K], bias)
dequantize_linear :143     dequantize_linear(spec, dtype=...) on the GPU kernel
affine_q6_qmm_t :157-204   affine_q6_qmm_t(x, spec, apply_gelu=, dtype=): rank 2/3
                           input, K check, leading dims kept, returns dtype
fused_q6_mlp :207-215      fused_q6_mlp(hidden, mlp_in, mlp_out)
dense_mlp :218-232         dense_mlp(hidden, mlp_in, mlp_out) on dense weights
eager_q6_mlp :249-253      eager_q6_mlp(ff, hidden): mlp_in -> gelu -> mlp_out
make_feed_forward_callables make_feed_forward_callables(ff, dtype=) ->
:256-280                   (eager_q6, fused, dense_predequant)
=========================  =====================================================

One deliberate difference: the reference's spec widens scales/biases to fp32
for its Metal kernel (:129-131).  Here they stay bf16 - the checkpoint dtype
the C ABI reads - which carries exactly the same values.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from qwen_image_shardedit_mlx_b200 import ops
from qwen_image_shardedit_mlx_b200.lora import LoRAAdapter, fold_lora_adapters, pad_lora_rank
from qwen_image_shardedit_mlx_b200.quantize import quantize_affine_q6


@dataclass(frozen=True)
class Q6LinearSpec:
    weight: torch.Tensor  # uint32 [N, K*bits/32]
    scales: torch.Tensor  # bf16 [N, K/group_size]
    qbiases: torch.Tensor  # bf16 [N, K/group_size]
    bias: torch.Tensor | None  # [N]
    group_size: int
    bits: int

    @property
    def out_features(self) -> int:
        return int(self.weight.shape[0])

    @property
    def in_features(self) -> int:
        return int(self.weight.shape[1] * 32 // self.bits)


class QuantizedLinear(torch.nn.Module):
    """q6 linear layer holding MLX-layout tensors (weight, scales, biases, bias).

    Same attribute names as mlx ``nn.QuantizedLinear``; calling it runs the
    q6 kernel with the output bias fused into the epilogue.
    """

    def __init__(self, weight: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                 bias: torch.Tensor | None = None, *, group_size: int = 64, bits: int = 6) -> None:
        super().__init__()
        self.register_buffer("weight", weight)
        self.register_buffer("scales", scales)
        self.register_buffer("biases", biases)
        self.register_buffer("bias", bias)
        self.group_size = int(group_size)
        self.bits = int(bits)
        self.mode = "affine"
        self.loras: list[LoRAAdapter] = []
        self.lora: tuple[torch.Tensor, torch.Tensor, float] | None = None  # the fused delta of ``loras``
        self.lora_b_nmajor: torch.Tensor | None = None  # its B transposed, [N, r padded to 32]

    @classmethod
    def from_linear(cls, linear: torch.nn.Linear, *, bits: int = 6, group_size: int = 64) -> "QuantizedLinear":
        if bits != 6:
            raise ValueError(f"only bits=6 is supported, got {bits}")
        w, s, b = quantize_affine_q6(linear.weight.detach(), group_size)
        bias = None if linear.bias is None else linear.bias.detach().to(torch.bfloat16)
        return cls(w, s, b, bias, group_size=group_size, bits=bits)

    @property
    def in_features(self) -> int:
        return int(self.weight.shape[1] * 32 // self.bits)

    @property
    def out_features(self) -> int:
        return int(self.weight.shape[0])

    def set_lora(self, a: torch.Tensor | None, b: torch.Tensor | None = None, scale: float = 1.0) -> None:
        """Attach (or with ``a=None`` remove) a LoRA delta, replacing any
        adapters: the layer then computes ``q6(x) + scale * ((x @ a) @ b)``
        before its bias, as the reference's LoRA-additive linear does
        (dense_img_ff_window.py:48-60).  ``a`` is [in_features, r], ``b`` is
        [r, out_features]; the ``(x @ a) @ b`` product is fused into the q6
        kernel's accumulator."""

        if a is None:
            self.loras = []
            self.lora = None
            self.lora_b_nmajor = None
            return
        if b is None:
            raise ValueError("LoRA needs both A and B")
        self.loras = []
        self.add_lora(a, b, scale)

    def add_lora(self, a: torch.Tensor, b: torch.Tensor, scale: float = 1.0) -> None:
        """Add one more adapter.  Several adapters are stacked into one fused
        delta of rank sum(r_i) <= 256 (``lora.fold_lora_adapters``); each adds
        exactly what it would add alone."""

        ad = LoRAAdapter(a.to(torch.bfloat16).contiguous(), b.to(torch.bfloat16).contiguous(), float(scale))
        adapters = [*self.loras, ad]
        self.lora = fold_lora_adapters(adapters, in_features=self.in_features, out_features=self.out_features)
        self.loras = adapters
        # the fused kernel reads B one output row at a time: keep it transposed too
        _, b_pad = pad_lora_rank(self.lora[0], self.lora[1])
        self.lora_b_nmajor = b_pad.t().contiguous()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.q6_linear(x, self.weight, self.scales, self.biases, self.bias, group_size=self.group_size,
                             lora=self.lora, lora_b_nmajor=self.lora_b_nmajor)


def quantized_linear_spec(layer: torch.nn.Module) -> Q6LinearSpec:
    """Extract packed affine q6 tensors from a QuantizedLinear-like module."""

    weight = layer.weight
    bits = int(layer.bits)
    group_size = int(layer.group_size)
    if bits != 6:
        raise ValueError(f"only bits=6 is supported, got {bits}")
    if weight.dtype not in (torch.uint32, torch.int32):
        raise ValueError(f"expected packed uint32 weight, got {weight.dtype}")
    bias = getattr(layer, "bias", None)
    return Q6LinearSpec(
        weight=weight,
        scales=layer.scales.to(torch.bfloat16),
        qbiases=layer.biases.to(torch.bfloat16),
        bias=None if bias is None else bias.to(torch.bfloat16),
        group_size=group_size,
        bits=bits,
    )


@dataclass(frozen=True)
class DenseLinearWeights:
    weight: torch.Tensor  # [N, K]
    bias: torch.Tensor | None


def dequantize_linear(spec: Q6LinearSpec, *, dtype: torch.dtype = torch.bfloat16) -> DenseLinearWeights:
    weight = ops.q6_dequantize(spec.weight, spec.scales, spec.qbiases, spec.group_size).to(dtype)
    bias = None if spec.bias is None else spec.bias.to(dtype)
    return DenseLinearWeights(weight=weight, bias=bias)


def affine_q6_qmm_t(
    x: torch.Tensor,
    spec: Q6LinearSpec,
    *,
    apply_gelu: bool = False,
    dtype: torch.dtype | None = None,
) -> torch.Tensor:
    """Affine q6 matmul, weight in Linear layout: act(x @ W.T + b)."""

    if x.dim() not in (2, 3):
        raise ValueError(f"expected x with rank 2 or 3, got shape {tuple(x.shape)}")
    out_dtype = x.dtype if dtype is None else dtype
    if x.shape[-1] != spec.in_features:
        raise ValueError(f"x in_features {x.shape[-1]} != weight in_features {spec.in_features}")
    xin = x.to(torch.float32) if out_dtype == torch.float32 else x.to(torch.bfloat16)
    y = ops.q6_linear(xin, spec.weight, spec.scales, spec.qbiases, spec.bias,
                      group_size=spec.group_size, apply_gelu=apply_gelu)
    return y.to(out_dtype)


def fused_q6_mlp(hidden: torch.Tensor, mlp_in: Q6LinearSpec, mlp_out: Q6LinearSpec) -> torch.Tensor:
    """Image/text MLP: q6 mlp_in + GELU epilogue, then q6 mlp_out."""

    if hidden.dtype == torch.float32:
        mid = affine_q6_qmm_t(hidden, mlp_in, apply_gelu=True)
        return affine_q6_qmm_t(mid, mlp_out, apply_gelu=False)
    return ops.q6_mlp(
        hidden,
        (mlp_in.weight, mlp_in.scales, mlp_in.qbiases, mlp_in.bias),
        (mlp_out.weight, mlp_out.scales, mlp_out.qbiases, mlp_out.bias),
        group_size=mlp_in.group_size,
    ).to(hidden.dtype)


def dense_mlp(hidden: torch.Tensor, mlp_in: DenseLinearWeights, mlp_out: DenseLinearWeights) -> torch.Tensor:
    """Dense Linear math with already-dequantised weights (library GEMM; an upper bound)."""

    mid = hidden @ mlp_in.weight.T
    if mlp_in.bias is not None:
        mid = mid + mlp_in.bias
    mid = F.gelu(mid, approximate="tanh")
    out = mid @ mlp_out.weight.T
    if mlp_out.bias is not None:
        out = out + mlp_out.bias
    return out


def dense_mlp_from_q6(hidden: torch.Tensor, mlp_in: Q6LinearSpec, mlp_out: Q6LinearSpec) -> torch.Tensor:
    """Dequantise each call, then dense math (diagnostic; includes the unpack cost)."""

    return dense_mlp(hidden, dequantize_linear(mlp_in, dtype=hidden.dtype), dequantize_linear(mlp_out, dtype=hidden.dtype))


def eager_q6_mlp(ff: torch.nn.Module, hidden: torch.Tensor) -> torch.Tensor:
    hidden = ff.mlp_in(hidden)
    hidden = F.gelu(hidden, approximate="tanh")
    hidden = ff.mlp_out(hidden)
    return hidden


def make_feed_forward_callables(
    ff: torch.nn.Module, *, dtype: torch.dtype = torch.bfloat16
) -> tuple[Callable[[torch.Tensor], torch.Tensor], Callable[[torch.Tensor], torch.Tensor], Callable[[torch.Tensor], torch.Tensor]]:
    """Return (eager_q6, fused_q6, dense_predequant) callables for one FF module."""

    mlp_in = quantized_linear_spec(ff.mlp_in)
    mlp_out = quantized_linear_spec(ff.mlp_out)
    dense_in = dequantize_linear(mlp_in, dtype=dtype)
    dense_out = dequantize_linear(mlp_out, dtype=dtype)
    return (
        lambda x, module=ff: eager_q6_mlp(module, x),
        lambda x, a=mlp_in, b=mlp_out: fused_q6_mlp(x, a, b),
        lambda x, a=dense_in, b=dense_out: dense_mlp(x, a, b),
    )


class QwenFeedForward(torch.nn.Module):
    """``img_ff`` / ``txt_ff`` shaped module: mlp_in (D -> H), GELU-tanh, mlp_out (H -> D)."""

    def __init__(self, mlp_in: QuantizedLinear, mlp_out: QuantizedLinear) -> None:
        super().__init__()
        self.mlp_in = mlp_in
        self.mlp_out = mlp_out

    @classmethod
    def random(cls, dim: int = 3072, hidden: int = 12288, *, group_size: int = 64, std: float = 0.02,
               bias_std: float = 0.01, generator: torch.Generator | None = None,
               device: torch.device | str = "cuda") -> "QwenFeedForward":
        def make(n: int, k: int) -> QuantizedLinear:
            w = torch.randn((n, k), generator=generator, device=device) * std
            q, s, b = quantize_affine_q6(w, group_size)
            bias = (torch.randn((n,), generator=generator, device=device) * bias_std).to(torch.bfloat16)
            return QuantizedLinear(q, s, b, bias, group_size=group_size)

        return cls(make(hidden, dim), make(dim, hidden))

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        if hidden.device.type == "cpu" and self.mlp_in.weight.is_cuda:
            return self.forward_host(hidden)
        if self.mlp_in.lora is not None or self.mlp_out.lora is not None:
            # LoRA-carrying layers: each linear fuses its own delta
            mid = ops.q6_linear(hidden, self.mlp_in.weight, self.mlp_in.scales, self.mlp_in.biases, self.mlp_in.bias,
                                group_size=self.mlp_in.group_size, apply_gelu=True, lora=self.mlp_in.lora,
                                lora_b_nmajor=self.mlp_in.lora_b_nmajor)
            return self.mlp_out(mid)
        return fused_q6_mlp(hidden, quantized_linear_spec(self.mlp_in), quantized_linear_spec(self.mlp_out))

    def forward_host(self, hidden: torch.Tensor, out: torch.Tensor | None = None,
                     chunks: int | None = None) -> torch.Tensor:
        """``ff(hidden)`` for activations in host memory, result in host memory
        (``out``, or a new pinned tensor): the rows are cut into ``chunks``
        equal batches (default: as many as 4 of at least 512 rows that divide
        the rows) that run through ``forward_host_stream``, so the upload of
        one chunk and the download of the previous overlap the kernels of the
        current one.  Returns once the result is on the host.  Each chunk's
        rows equal ``ff(chunk.cuda())`` exactly; pinned inputs copy fastest."""

        d = self.mlp_in.in_features
        x2 = hidden.reshape(-1, d)
        if x2.dtype != torch.bfloat16:
            x2 = x2.to(torch.bfloat16)
        m = int(x2.shape[0])
        if chunks is None:
            chunks = max(1, min(4, m // 512))
            while m % chunks:
                chunks -= 1
        if chunks < 1 or m % chunks:
            raise ValueError(f"{m} rows do not split into {chunks} equal chunks")
        if out is None:
            y2 = torch.empty((m, d), dtype=torch.bfloat16, pin_memory=True)
        else:
            if out.device.type != "cpu" or out.dtype != torch.bfloat16 or out.numel() != m * d or \
                    not out.is_contiguous():
                raise ValueError("out must be a contiguous bf16 host tensor of the input's size")
            y2 = out.view(m, d)
        step = m // chunks
        self.forward_host_stream([x2[i * step:(i + 1) * step] for i in range(chunks)],
                                 [y2[i * step:(i + 1) * step] for i in range(chunks)])
        torch.cuda.current_stream(self.mlp_in.weight.device).synchronize()
        if out is not None:
            return out
        y = y2.reshape(*hidden.shape[:-1], d)
        return y if hidden.dtype == torch.bfloat16 else y.to(hidden.dtype)

    def forward_host_stream(self, xs: Sequence[torch.Tensor], ys: Sequence[torch.Tensor]) -> None:
        """Run the MLP over a sequence of batches that live in (pinned) host
        memory: ``ys[i] = ff(xs[i])``.

        The upload of batch i + 1 and the download of batch i - 1 overlap
        the kernels of batch i (one stream per direction plus the compute
        stream, two device buffers each way), so a serving loop that holds
        its activations on the host pays max(copy, compute) per batch instead
        of their sum.  Returns once all work is queued; the current stream
        waits for the last download, so synchronising it (or an event
        recorded on it) marks the end.  Batches must share one shape.
        """

        if len(xs) != len(ys):
            raise ValueError("xs and ys must pair up")
        if not xs:
            return
        dev = self.mlp_in.weight.device
        d, h = self.mlp_in.in_features, self.mlp_in.out_features
        m = int(xs[0].reshape(-1, d).shape[0])
        lora = self.mlp_in.lora is not None or self.mlp_out.lora is not None
        w1 = (self.mlp_in.weight, self.mlp_in.scales, self.mlp_in.biases, self.mlp_in.bias)
        w2 = (self.mlp_out.weight, self.mlp_out.scales, self.mlp_out.biases, self.mlp_out.bias)
        key = (m, d, h, str(dev), lora, tuple(0 if t is None else t.data_ptr() for t in (*w1, *w2)))
        if getattr(self, "_stream_key", None) != key:
            x_dev = [torch.empty((m, d), dtype=torch.bfloat16, device=dev) for _ in range(2)]
            y_dev = [torch.empty((m, d), dtype=torch.bfloat16, device=dev) for _ in range(2)]
            workspace = torch.empty(int(ops.mlp_workspace_bytes(m, h, d)), dtype=torch.uint8, device=dev)
            # One prepared MLP call per slot (fixed pointers): the loop's host work
            # per batch stays far below the kernels' time.
            call = None if lora else ops.MlpCall(w1, w2, m, self.mlp_in.group_size, workspace)
            events = [[torch.cuda.Event() for _ in range(2)] for _ in range(3)]  # loaded, computed, done
            self._stream_bufs = (x_dev, y_dev, workspace, [torch.cuda.Stream(dev) for _ in range(3)], call, events)
            self._stream_key = key
        x_dev, y_dev, workspace, (s_in, s_comp, s_out), call, (loaded, computed, done) = self._stream_bufs
        caller = torch.cuda.current_stream(dev)
        for s in (s_in, s_comp, s_out):
            s.wait_stream(caller)
        comp_handle = s_comp.cuda_stream
        # A wait on an event takes its latest record at the time of the wait, so
        # the per-slot events recorded again two batches later stay correct.
        for i, (xh, yh) in enumerate(zip(xs, ys)):
            slot = i % 2
            if xh.reshape(-1, d).shape[0] != m or yh.numel() != m * d:
                raise ValueError("all batches must have the first batch's shape")
            if i >= 2:
                s_in.wait_event(computed[slot])  # the compute of batch i - 2 has read x_dev[slot]
            with torch.cuda.stream(s_in):
                x_dev[slot].copy_(xh.reshape(m, d), non_blocking=True)
            loaded[slot].record(s_in)
            s_comp.wait_event(loaded[slot])
            if i >= 2:
                s_comp.wait_event(done[slot])  # the download of batch i - 2 has read y_dev[slot]
            if call is not None:
                call(x_dev[slot].data_ptr(), y_dev[slot].data_ptr(), comp_handle)
            else:
                with torch.cuda.stream(s_comp):
                    y_dev[slot].copy_(self.forward(x_dev[slot]))  # each linear fuses its own delta
            computed[slot].record(s_comp)
            s_out.wait_event(computed[slot])
            with torch.cuda.stream(s_out):
                yh.reshape(m, d).copy_(y_dev[slot], non_blocking=True)
            done[slot].record(s_out)
        caller.wait_stream(s_out)
