"""ctypes binding of libq6b200.so (the C ABI declared in include/q6_b200.h).

The library is the only compute path: if it is missing or fails to load,
every op raises instead of falling back to anything else.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libq6b200.so")

Q6_OK = 0
Q6_ERR_INVALID_ARGUMENT = 1
Q6_ERR_SHAPE = 2
Q6_ERR_GROUP_SIZE = 3
Q6_ERR_ALIGNMENT = 4
Q6_ERR_UNSUPPORTED = 5
Q6_ERR_CUDA = 6
Q6_ERR_DEVICE = 7
Q6_ERR_WORKSPACE = 8

Q6_EPI_NONE = 0
Q6_EPI_GELU = 1
Q6_EPI_GELU_PRECISE = 2
Q6_LORA_B_NMAJOR = 4

Q6_SITE_PEER_BARRIER = 13
Q6_SITE_SELFTEST = 64

Q6_PATH_AUTO = 0
Q6_PATH_SIMT = 1
Q6_PATH_TENSOR = 2
Q6_PATH_SKINNY = 3

PATHS = {"auto": Q6_PATH_AUTO, "simt": Q6_PATH_SIMT, "tensor": Q6_PATH_TENSOR, "skinny": Q6_PATH_SKINNY}

# Every symbol include/q6_b200.h declares, with its ctypes signature.
_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t
_F = ctypes.c_float
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "q6_dequantize_bf16": (_I, [_P, _P, _P, _P, _I64, _I64, _I, _P]),
    "q6_linear_bf16": (
        _I,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _F, _I, _P, _I64, _I64, _I64, _I, _I, _I, _P, _SZ, _P],
    ),
    "q6_lora_xa_bf16": (_I, [_P, _P, _P, _I64, _I64, _I, _P]),
    "q6_linear_tc_workspace_bytes": (_SZ, [_I64, _I64, _I64]),
    "q6_linear_f32": (_I, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I, _I, _P]),
    "q6_mlp_bf16": (
        _I,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I, _P, _SZ, _P],
    ),
    "q6_mlp_workspace_bytes": (_SZ, [_I64, _I64]),
    "q6_mlp_bf16_noalloc": (
        _I,
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I, _P],
    ),
    "q6_layernorm_modulate_bf16": (_I, [_P, _P, _P, _P, _I64, _I64, _F, _P]),
    "q6_add_layernorm_modulate_bf16": (_I, [_P, _P, _P, _P, _P, _I64, _P, _I64, _I64, _I64, _I64, _I64, _F, _P]),
    "q6_qk_rmsnorm_rope_bf16": (_I, [_P, _I64, _I64, _I, _I, _P, _P, _P, _F, _P]),
    "q6_qk_rmsnorm_rope_joint_bf16": (_I, [_P, _I64, _I64, _I, _I, _P, _P, _P, _P, _I64, _I64, _I64, _F, _P]),
    "q6_get_device_error": (_I, [ctypes.POINTER(ctypes.c_int)]),
    "q6_clear_device_error": (_I, []),
    "q6_last_path": (_I, []),
    "q6_tensor_token_tile": (_I, [_I64, _I64]),
    "q6_skinny_plan": (_I, [_I64, _I64, _I64, _I, _P, _P, _P]),
    "q6_pair_fallback_count": (_I64, []),
    "q6_sp_add_layernorm_gather_bf16": (_I, [_P, _P, _P, _P, _P, _I64, _P, _I, _I, _I64, _I64, _I64, _I64, _F,
                                             _P]),
    "q6_sp_barrier": (_I, [_P, _P, _I, _I, _I64, _P]),
    "q6_selftest_bounded_wait": (_I, [_I64, _P]),
    "q6_status_string": (ctypes.c_char_p, [_I]),
    "q6_abi_version": (_I, []),
}


class Q6Error(RuntimeError):
    """A non-zero q6_status from the library."""

    def __init__(self, status: int, where: str) -> None:
        self.status = int(status)
        super().__init__(f"{where}: q6 status {status} ({status_string(status)})")


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"{LIB_PATH} is not built; run `python -m qwen_image_shardedit_mlx_b200.build`"
                    )
                handle = ctypes.CDLL(str(LIB_PATH))
                for name, (restype, argtypes) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = restype
                    fn.argtypes = argtypes
                _lib = handle
    return _lib


def status_string(status: int) -> str:
    try:
        raw = lib().q6_status_string(int(status))
    except Exception:  # pragma: no cover - library missing
        return "unknown"
    return raw.decode() if raw else "unknown"


def check(status: int, where: str) -> None:
    if status != Q6_OK:
        raise Q6Error(status, where)
