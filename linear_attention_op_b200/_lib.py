"""ctypes binding of the C-ABI in ``include/gdn_b200.h`` (libgdn_b200.so, built in-tree).

There is no fallback: if the library is missing or cannot be loaded, every entry point raises
``GDNLibraryError``.  Build it with ``python -m linear_attention_op_b200.build``.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libgdn_b200.so"

GDN_OK = 0
STATUS_NAMES = {
    0: "GDN_OK", 1: "GDN_ERR_INVALID_ARGUMENT", 2: "GDN_ERR_NULL_POINTER", 3: "GDN_ERR_UNSUPPORTED",
    4: "GDN_ERR_CUDA", 5: "GDN_ERR_NCCL", 6: "GDN_ERR_TIMEOUT", 7: "GDN_ERR_OUT_OF_MEMORY",
}

# Every symbol the header declares (checked by tests/test_abi_exports.py).
EXPORTED = (
    "gdn_layer_create", "gdn_layer_destroy", "gdn_layer_get_info", "gdn_layer_reserve", "gdn_layer_forward",
    "gdn_recurrence_forward", "gdn_comm_get_unique_id", "gdn_comm_create", "gdn_comm_destroy", "gdn_comm_allgather",
    "gdn_device_error", "gdn_last_error_string", "gdn_kernel_launch_count", "gdn_abi_version", "gdn_gemm_bf16",
    "gdn_layer_set_stage_events", "gdn_layer_decode_static", "gdn_layer_share_workspace",
    "gdn_layer_set_weight_format", "gdn_selftest_peer_wait", "gdn_layer_reserve_batch", "gdn_layer_set_max_rows",
    "gdn_decoder_create", "gdn_decoder_destroy", "gdn_decoder_reserve", "gdn_decoder_forward",
)


class GDNLibraryError(RuntimeError):
    """The CUDA library is missing or failed to load."""


class GDNError(RuntimeError):
    """A C-ABI call returned a non-OK status."""

    def __init__(self, status: int, func: str, message: str):
        self.status = status
        super().__init__(f"{func} -> {STATUS_NAMES.get(status, status)}: {message}")


class Dims(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int32), ("num_k_heads", ctypes.c_int32), ("num_v_heads", ctypes.c_int32),
                ("head_k_dim", ctypes.c_int32), ("head_v_dim", ctypes.c_int32), ("conv_kernel", ctypes.c_int32),
                ("eps", ctypes.c_float), ("chunk", ctypes.c_int32)]


class Weights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in
                ("w_qkv", "w_z", "w_a", "w_b", "conv_w", "a_log", "dt_bias", "norm_w", "w_out")]


class MlpWeights(ctypes.Structure):
    _fields_ = [("input_norm_w", ctypes.c_void_p), ("post_norm_w", ctypes.c_void_p), ("w_gate", ctypes.c_void_p),
                ("w_up", ctypes.c_void_p), ("w_down", ctypes.c_void_p), ("intermediate", ctypes.c_int32),
                ("eps", ctypes.c_float)]


class LayerInfo(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int32), ("num_k_heads_local", ctypes.c_int32),
                ("num_v_heads_local", ctypes.c_int32), ("conv_dim_local", ctypes.c_int32),
                ("tp_rank", ctypes.c_int32), ("tp_size", ctypes.c_int32),
                ("rec_state_floats_per_seq", ctypes.c_int64), ("conv_state_floats_per_seq", ctypes.c_int64),
                ("workspace_bytes", ctypes.c_int64)]


_lib = None


def _declare(lib: ctypes.CDLL) -> None:
    P = ctypes.c_void_p
    I32, I64, F = ctypes.c_int32, ctypes.c_int64, ctypes.c_float
    sigs = {
        "gdn_layer_create": [ctypes.POINTER(Dims), ctypes.POINTER(Weights), I32, I32, ctypes.POINTER(P)],
        "gdn_layer_destroy": [P],
        "gdn_layer_get_info": [P, ctypes.POINTER(LayerInfo)],
        "gdn_layer_reserve": [P, I64],
        "gdn_layer_forward": [P, P, I32, I32, P, P, P, P, P],
        "gdn_recurrence_forward": [P, P, P, P, P, I32, I32, I32, I32, I32, F, P, P, P],
        "gdn_comm_get_unique_id": [P, ctypes.c_size_t],
        "gdn_comm_create": [P, ctypes.c_size_t, I32, I32, ctypes.POINTER(P)],
        "gdn_comm_destroy": [P],
        "gdn_comm_allgather": [P, P, ctypes.c_size_t, P],
        "gdn_device_error": [ctypes.POINTER(I32)],
        "gdn_gemm_bf16": [P, I64, P, I64, I32, I32, I32, I32, P, I64, I32, P],
        "gdn_layer_set_stage_events": [P, ctypes.POINTER(P), I32],
        "gdn_layer_decode_static": [P, P, I32, P, P, P, P],
        "gdn_layer_share_workspace": [P, P],
        "gdn_layer_set_weight_format": [P, I32],
        "gdn_selftest_peer_wait": [P, ctypes.c_uint64, P],
        "gdn_layer_reserve_batch": [P, I64, I32],
        "gdn_decoder_create": [P, ctypes.POINTER(MlpWeights), ctypes.POINTER(P)],
        "gdn_decoder_destroy": [P],
        "gdn_decoder_reserve": [P, I64],
        "gdn_decoder_forward": [P, P, I32, I32, P, P, P, P, P],
        "gdn_layer_set_max_rows": [P, I64],
    }
    for name, args in sigs.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    lib.gdn_last_error_string.argtypes = []
    lib.gdn_last_error_string.restype = ctypes.c_char_p
    lib.gdn_kernel_launch_count.argtypes = []
    lib.gdn_kernel_launch_count.restype = ctypes.c_uint64
    lib.gdn_abi_version.argtypes = []
    lib.gdn_abi_version.restype = ctypes.c_int32


def lib() -> ctypes.CDLL:
    """Load libgdn_b200.so once (raises GDNLibraryError if it is not built)."""
    global _lib
    if _lib is None:
        path = Path(os.environ.get("GDN_B200_LIB", LIB_PATH))
        if not path.exists():
            raise GDNLibraryError(
                f"{path} not found: build it with `python -m linear_attention_op_b200.build` (no CPU fallback)")
        try:
            handle = ctypes.CDLL(str(path), mode=ctypes.RTLD_GLOBAL)
        except OSError as e:
            raise GDNLibraryError(f"cannot load {path}: {e}") from e
        _declare(handle)
        _lib = handle
    return _lib


def check(status: int, func: str) -> None:
    if status != GDN_OK:
        msg = lib().gdn_last_error_string().decode(errors="replace")
        raise GDNError(status, func, msg)


def call(func: str, *args) -> None:
    check(getattr(lib(), func)(*args), func)


def device_error() -> int:
    """Synchronise and return (and clear) the device error word; raises on a recorded error."""
    code = ctypes.c_int32(0)
    st = lib().gdn_device_error(ctypes.byref(code))
    if st != GDN_OK and code.value == 0:
        check(st, "gdn_device_error")
    return code.value


def launch_count() -> int:
    return int(lib().gdn_kernel_launch_count())
