"""The C-ABI library loads, exports every symbol the header declares, and validates arguments before
touching the GPU (CPU only: no compute call is made)."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from linear_attention_op_b200 import _lib
from linear_attention_op_b200._lib import Dims, Weights

HEADER = Path(__file__).resolve().parents[1] / "include" / "gdn_b200.h"


def declared_symbols():
    return sorted(set(re.findall(r"^GDN_API\s+[\w\s\*]+?\b(gdn_\w+)\(", HEADER.read_text(), flags=re.M)))


def test_every_declared_symbol_is_exported():
    lib = _lib.lib()
    syms = declared_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in gdn_b200.h but not exported"
    assert set(syms) == set(_lib.EXPORTED)


def test_abi_version():
    assert _lib.lib().gdn_abi_version() == 1


def _dims(**kw):
    d = dict(hidden=256, num_k_heads=2, num_v_heads=4, head_k_dim=128, head_v_dim=128, conv_kernel=4, eps=1e-6, chunk=64)
    d.update(kw)
    return Dims(**d)


def _fake_weights():
    # Non-null pointers that are never dereferenced: validation fails first.
    buf = (ctypes.c_uint8 * 64)()
    p = ctypes.cast(buf, ctypes.c_void_p)
    return Weights(*([p] * 9)), buf


@pytest.mark.parametrize("kw, status", [
    (dict(head_k_dim=64), 3), (dict(head_v_dim=256), 3), (dict(conv_kernel=3), 3), (dict(chunk=32), 3),
    (dict(hidden=100), 1), (dict(num_v_heads=3), 1), (dict(num_k_heads=0), 1), (dict(eps=0.0), 1),
    (dict(num_k_heads=1, num_v_heads=16), 3),
])
def test_layer_create_rejects_bad_geometry(kw, status):
    w, _keep = _fake_weights()
    h = ctypes.c_void_p()
    st = _lib.lib().gdn_layer_create(ctypes.byref(_dims(**kw)), ctypes.byref(w), 0, 1, ctypes.byref(h))
    assert st == status
    assert not h.value
    assert _lib.lib().gdn_last_error_string()


def test_layer_create_rejects_bad_tp():
    w, _keep = _fake_weights()
    h = ctypes.c_void_p()
    lib = _lib.lib()
    assert lib.gdn_layer_create(ctypes.byref(_dims()), ctypes.byref(w), 0, 3, ctypes.byref(h)) == 1  # 3 !| 2, 4
    assert lib.gdn_layer_create(ctypes.byref(_dims()), ctypes.byref(w), 2, 2, ctypes.byref(h)) == 1
    assert lib.gdn_layer_create(ctypes.byref(_dims()), ctypes.byref(w), 0, 0, ctypes.byref(h)) == 1


def test_null_pointers_are_reported():
    lib = _lib.lib()
    h = ctypes.c_void_p()
    assert lib.gdn_layer_create(None, None, 0, 1, ctypes.byref(h)) == 2
    w = Weights()
    assert lib.gdn_layer_create(ctypes.byref(_dims()), ctypes.byref(w), 0, 1, ctypes.byref(h)) == 2
    assert lib.gdn_layer_forward(None, None, 1, 1, None, None, None, None, None) == 2
    assert lib.gdn_layer_destroy(None) == 2
    assert lib.gdn_comm_destroy(None) == 2
    assert lib.gdn_recurrence_forward(None, None, None, None, None, 1, 1, 1, 1, 1, 0.0, None, None, None) == 2


def test_recurrence_rejects_bad_shapes():
    lib = _lib.lib()
    buf = torch.zeros(64)
    p = ctypes.c_void_p(buf.data_ptr())
    assert lib.gdn_recurrence_forward(p, p, p, p, p, 1, 1, 2, 3, 1, 0.0, p, p, None) == 1  # Hv % Hk
    assert lib.gdn_recurrence_forward(p, p, p, p, p, 0, 1, 1, 1, 1, 0.0, p, p, None) == 1


def test_gemm_rejects_bad_shapes():
    lib = _lib.lib()
    buf = torch.zeros(64)
    p = ctypes.c_void_p(buf.data_ptr())
    assert lib.gdn_gemm_bf16(p, 12, p, 12, 4, 4, 12, 0, p, 4, 0, None) == 1  # k % 8
    assert lib.gdn_gemm_bf16(p, 16, p, 16, 4, 4, 16, 7, p, 4, 0, None) == 1  # out kind
    assert lib.gdn_gemm_bf16(p, 16, p, 16, 4, 4, 16, 0, p, 4, 9, None) == 1  # ksplit


def test_python_errors_raise():
    from linear_attention_op_b200._lib import GDNError, call

    w, _keep = _fake_weights()
    h = ctypes.c_void_p()
    with pytest.raises(GDNError, match="UNSUPPORTED"):
        call("gdn_layer_create", ctypes.byref(_dims(head_k_dim=64)), ctypes.byref(w), 0, 1, ctypes.byref(h))


def test_workspace_format_and_selftest_entry_points_check_pointers():
    """The workspace, weight-format and self-test entry points reject null handles before any CUDA call."""
    lib = _lib.lib()
    assert lib.gdn_layer_share_workspace(None, None) == 2
    assert lib.gdn_layer_set_weight_format(None, 1) == 2
    assert lib.gdn_layer_reserve(None, 64) == 2
    assert lib.gdn_selftest_peer_wait(None, 1, None) == 2
    assert lib.gdn_layer_decode_static(None, None, 1, None, None, None, None) == 2
    assert lib.gdn_layer_reserve_batch(None, 64, 1) == 2
    assert lib.gdn_layer_set_max_rows(None, 128) == 2
    assert lib.gdn_comm_allgather(None, None, 16, None) == 2
    assert lib.gdn_last_error_string()
