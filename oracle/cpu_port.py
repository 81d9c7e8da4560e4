"""Host-core baselines for bench.py (test infrastructure; never on the product path).

* ``time_mlp_port``: the oracle's torch-CPU restatement of the image MLP with
  pre-dequantised bf16 weights (dequantised once, outside the timed region -
  the reference's ``dense_mlp`` upper-bound path, shardedit_mlx/q6_metal_mlp.py:218-232),
  timed on a token sample with every host thread.
* ``time_reference_kernel_mlp``: the reference's own q6 kernel source
  (SOURCE_QMM_T, shardedit_mlx/q6_metal_mlp.py:58-83, compiled for the host by
  oracle/build_ref.py into oracle/_ref/libq6ref.so) running the
  ``fused_q6_mlp`` composition (fc1 with GELU epilogue, then fc2;
  q6_metal_mlp.py:207-215) on a token sample.  Falls back to the port when the
  compiled reference is absent.
"""

from __future__ import annotations

import os
import time

import numpy as np

from oracle import oracle as _o


def mlp_port_flops(tokens: int, dim: int, hidden: int) -> float:
    return 4.0 * tokens * dim * hidden


def _weights(rng: np.random.Generator, n: int, k: int, gs: int) -> _o.Q6Weights:
    w = rng.normal(0.0, 0.02, size=(n, k)).astype(np.float32)
    packed, scales, biases = _o.affine_quantize(w, group_size=gs)
    bias = _o.f32_to_bf16_bits(rng.normal(0.0, 0.01, size=(n,)).astype(np.float32))
    return _o.Q6Weights(packed, scales, biases, bias, gs)


def time_mlp_port(max_tokens: int, dim: int, hidden: int, gs: int, *, budget_s: float = 12.0) -> tuple[int, float, int]:
    """Returns (tokens per step, timed seconds, steps)."""

    import torch

    rng = np.random.default_rng(99)
    fc1 = _weights(rng, hidden, dim, gs)
    fc2 = _weights(rng, dim, hidden, gs)

    def dense(w: _o.Q6Weights):
        bits = _o.dequantize(w.weight, w.scales, w.biases, gs, dtype="bf16")
        wt = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16)
        bt = torch.from_numpy(w.bias.view(np.int16)).view(torch.bfloat16)
        return wt, bt

    w1, b1 = dense(fc1)
    w2, b2 = dense(fc2)

    def step(x):
        h = torch.nn.functional.gelu(x @ w1.T + b1, approximate="tanh")
        return h @ w2.T + b2

    tokens = 32
    x = torch.randn((tokens, dim)).to(torch.bfloat16)
    t0 = time.perf_counter()
    step(x)
    per_token = max((time.perf_counter() - t0) / tokens, 1e-6)
    tokens = int(max(1, min(max_tokens, (budget_s / 4) / per_token)))
    x = torch.randn((tokens, dim)).to(torch.bfloat16)
    steps, elapsed = 0, 0.0
    while elapsed < budget_s and steps < 64:
        t0 = time.perf_counter()
        step(x)
        elapsed += time.perf_counter() - t0
        steps += 1
    return tokens, elapsed, steps


def time_reference_kernel_mlp(dim: int, hidden: int, gs: int, *, tokens: int, steps: int,
                              total_budget_s: float = 110.0) -> dict:
    """The reference kernel's fused_q6_mlp composition on full ``tokens``-row
    steps: a 16-token warm-up (which also estimates the step time), then as
    many full steps as fit ``total_budget_s`` (at least one, at most ``steps``)."""

    ref = _o.load_ref()
    cores = int(os.environ.get("Q6REF_THREADS", "0")) or (os.cpu_count() or 1)
    if ref is None:
        import torch

        torch.set_num_threads(cores)
        ntok, seconds, nsteps = time_mlp_port(tokens, dim, hidden, gs, budget_s=min(total_budget_s, 30.0))
        return {"tflops": mlp_port_flops(ntok, dim, hidden) * nsteps / seconds / 1e12, "steps": nsteps,
                "tokens": ntok, "cores": torch.get_num_threads(), "kind": "port",
                "sample": f"oracle/_ref not built; torch-CPU port, {nsteps} x {ntok} tokens"}

    rng = np.random.default_rng(98)
    fc1 = _weights(rng, hidden, dim, gs)
    fc2 = _weights(rng, dim, hidden, gs)
    prepared = []
    for w in (fc1, fc2):
        prepared.append((np.ascontiguousarray(w.weight), np.ascontiguousarray(w.scales_f32()),
                         np.ascontiguousarray(w.biases_f32()), np.ascontiguousarray(w.bias_f32())))

    def run(ntok: int) -> float:
        x = _o.f32_to_bf16_bits(rng.standard_normal((ntok, dim)).astype(np.float32))
        h = np.zeros((ntok, hidden), dtype=np.uint16)
        y = np.zeros((ntok, dim), dtype=np.uint16)
        (w1, s1, q1, b1), (w2, s2, q2, b2) = prepared
        t0 = time.perf_counter()
        ref.q6ref_qmm_t_bf16(x.ctypes.data, w1.ctypes.data, s1.ctypes.data, q1.ctypes.data, b1.ctypes.data,
                             h.ctypes.data, ntok, hidden, dim, gs, w1.shape[1], s1.shape[1], 1, 1)
        ref.q6ref_qmm_t_bf16(h.ctypes.data, w2.ctypes.data, s2.ctypes.data, q2.ctypes.data, b2.ctypes.data,
                             y.ctypes.data, ntok, dim, hidden, gs, w2.shape[1], s2.shape[1], 1, 0)
        return time.perf_counter() - t0

    probe_tokens = 16
    per_token = run(probe_tokens) / probe_tokens
    nsteps = int(max(1, min(steps, total_budget_s // max(per_token * tokens, 1e-6))))
    elapsed = sum(run(tokens) for _ in range(nsteps))
    return {"tflops": mlp_port_flops(tokens, dim, hidden) * nsteps / elapsed / 1e12, "steps": nsteps,
            "tokens": tokens, "cores": cores, "kind": "reference",
            "sample": (f"{nsteps} full step(s) of {tokens} tokens (after a {probe_tokens}-token warm-up) through "
                       f"the reference's SOURCE_QMM_T compiled for the host (fc1+GELU, then fc2), {cores} threads")}
