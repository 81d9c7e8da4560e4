"""bench.py on the CPU: it imports, every leg it runs exists, and both arms
describe the same workload (the reference arm's config is ours at one GPU)."""

from __future__ import annotations

import importlib
import sys

from tests.conftest import ROOT


def _bench():
    if str(ROOT) not in sys.path:
        sys.path.insert(0, str(ROOT))
    return importlib.import_module("bench")


def test_bench_legs_exist():
    b = _bench()
    for name in ("run_ours", "run_reference", "measure_block", "measure_stack", "measure_gemv", "measure_sweep",
                 "measure_kernels", "_time_launches", "_graph_ms", "cpu_baseline_port", "workload_config"):
        assert callable(getattr(b, name)), name
    assert b.FLOP_PER_STEP == 4 * 3456 * 3072 * 12288


def test_reference_arm_config_is_ours():
    b = _bench()
    assert b.workload_config(1) == b.workload_config(1)
    assert b.workload_config(1)["tokens_per_gpu"] == 3456


def test_block_form_auto_policy():
    """--block-form auto: the CFG pair on an even GPU count runs context-parallel
    in sample groups; one sample runs tensor-parallel over peer memory at 2 GPUs
    and context-parallel from 4; an explicit form is kept."""

    b = _bench()
    expect = {(2, 1): "tp-peer", (2, 2): "cp", (4, 1): "cp", (4, 2): "cp", (8, 1): "cp", (8, 2): "cp",
              (3, 2): "cp"}
    for (world, batch), form in expect.items():
        got = b.block_form("auto", world, batch)
        assert got == form, (world, batch, got)
        assert got in b.BLOCK_FORMS
    for form in b.BLOCK_FORMS:
        if form != "auto":
            assert b.block_form(form, 8, 2) == form
