"""Compile the reference's own q6 kernel source for the CPU (test infrastructure).

The reference keeps its q6 device code as Metal Shading Language text inside
Python string constants (shardedit_mlx/q6_metal_mlp.py:17-83: HEADER with
`extract_q6`, `dequant_q6`, `gelu_approx_f`, and SOURCE_QMM_T, the
one-output-per-thread affine q6 matmul).  That text is a C-like subset, so this
recipe reads it from the reference tree where it lies, wraps it in a CPU
driver loop (one iteration per Metal thread), and compiles it with g++ against
the small stand-in header oracle/ref_shim/metal_stdlib.

Outputs go to oracle/_ref/ only (git-ignored; the built .so travels to the GPU
box so tests can use it there).  Nothing from the reference is committed.

Usage:  python oracle/build_ref.py --reference <reference checkout>
        (or set Q6_REFERENCE_ROOT to the checkout)
"""

from __future__ import annotations

import argparse
import ast
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
LIB = OUT_DIR / "libq6ref.so"
REF_FILE = Path("shardedit_mlx") / "q6_metal_mlp.py"

_DRIVER = r"""
// ---- CPU driver around the reference's SOURCE_QMM_T (generated; do not commit) ----
#include <thread>
#include <vector>
#include <cstdlib>

static int q6ref_threads() {
    const char* env = std::getenv("Q6REF_THREADS");
    int n = env ? std::atoi(env) : 0;
    if (n <= 0) n = (int)std::thread::hardware_concurrency();
    return n > 0 ? n : 1;
}

// One loop iteration per Metal thread of the dispatch grid (M, N); the
// iterations are split over host threads by output row n.
template <typename T>
static void q6ref_qmm_t_impl(const T* x, const uint* weight, const float* scales,
                             const float* qbiases, const float* bias, T* out,
                             uint M, uint N, uint K, uint group_size,
                             uint weight_stride, uint scale_stride,
                             int has_bias, int apply_gelu) {
    auto run = [&](long n_begin, long n_end) {
        for (long mm = 0; mm < (long)M; ++mm) {
            for (long nn = n_begin; nn < n_end; ++nn) {
                const uint3 thread_position_in_grid = {(uint)mm, (uint)nn, 0u};
                [&]() {
@@SOURCE@@
                }();
            }
        }
    };
    int workers = q6ref_threads();
    if ((long)workers > (long)N) workers = (int)N;
    if (workers <= 1) { run(0, (long)N); return; }
    std::vector<std::thread> pool;
    long chunk = ((long)N + workers - 1) / workers;
    for (int t = 0; t < workers; ++t) {
        long b = t * chunk, e = b + chunk < (long)N ? b + chunk : (long)N;
        if (b < e) pool.emplace_back(run, b, e);
    }
    for (auto& th : pool) th.join();
}

extern "C" {
void q6ref_qmm_t_f32(const float* x, const uint* weight, const float* scales,
                     const float* qbiases, const float* bias, float* out,
                     uint M, uint N, uint K, uint group_size, uint weight_stride,
                     uint scale_stride, int has_bias, int apply_gelu) {
    q6ref_qmm_t_impl<float>(x, weight, scales, qbiases, bias, out, M, N, K, group_size,
                            weight_stride, scale_stride, has_bias, apply_gelu);
}
void q6ref_qmm_t_bf16(const bfloat16_t* x, const uint* weight, const float* scales,
                      const float* qbiases, const float* bias, bfloat16_t* out,
                      uint M, uint N, uint K, uint group_size, uint weight_stride,
                      uint scale_stride, int has_bias, int apply_gelu) {
    q6ref_qmm_t_impl<bfloat16_t>(x, weight, scales, qbiases, bias, out, M, N, K, group_size,
                                 weight_stride, scale_stride, has_bias, apply_gelu);
}
uint q6ref_extract_q6(const uint* packed, uint index) { return extract_q6(packed, index); }
float q6ref_dequant_q6(const uint* packed, const float* scales, const float* qbiases,
                       uint k, uint group_size) {
    return dequant_q6(packed, scales, qbiases, k, group_size);
}
float q6ref_gelu_approx(float v) { return gelu_approx_f(v); }
}
"""


def _string_constants(path: Path) -> dict[str, str]:
    tree = ast.parse(path.read_text(encoding="utf-8"))
    found: dict[str, str] = {}
    for node in tree.body:
        if isinstance(node, ast.Assign) and len(node.targets) == 1:
            target = node.targets[0]
            if isinstance(target, ast.Name) and isinstance(node.value, ast.Constant):
                if isinstance(node.value.value, str):
                    found[target.id] = node.value.value
    return found


def build(reference: Path, *, verbose: bool = False) -> Path:
    src_file = reference / REF_FILE
    consts = _string_constants(src_file)
    missing = [name for name in ("HEADER", "SOURCE_QMM_T") if name not in consts]
    if missing:
        raise RuntimeError(f"{src_file}: string constants not found: {missing}")
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    generated = OUT_DIR / "q6_ref_naive.cpp"
    text = (
        f"// Generated from {src_file} by oracle/build_ref.py.\n"
        + consts["HEADER"]
        + _DRIVER.replace("@@SOURCE@@", consts["SOURCE_QMM_T"])
    )
    generated.write_text(text, encoding="utf-8")
    cmd = [
        os.environ.get("CXX", "g++"),
        "-O2",
        "-std=c++17",
        "-fPIC",
        "-shared",
        "-pthread",
        "-ffp-contract=off",
        "-I",
        str(HERE / "ref_shim"),
        str(generated),
        "-o",
        str(LIB),
    ]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return LIB


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", type=Path, default=None,
                        help="checkout of the reference project (default: $Q6_REFERENCE_ROOT)")
    parser.add_argument("-v", "--verbose", action="store_true")
    args = parser.parse_args()
    if args.reference is None:
        env = os.environ.get("Q6_REFERENCE_ROOT")
        if not env:
            print("give --reference or set Q6_REFERENCE_ROOT; nothing built", file=sys.stderr)
            return 1
        args.reference = Path(env)
    if not (args.reference / REF_FILE).exists():
        print(f"reference source not found under {args.reference}; nothing built", file=sys.stderr)
        return 1
    print(build(args.reference, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
