"""The allocation-free decode entry point (gdn_layer_decode_static) against gdn_layer_forward and the oracle.

Some callers cannot allocate device memory while they call the layer: a serving runtime that owns the
GPU's memory budget, or code that issues the call while a stream is being captured (a cudaMalloc there
breaks the capture).  gdn_layer_decode_static runs the same decode step with its intermediates in a
static device array instead of the layer's workspace.  This file is collected last on purpose."""
import ctypes

import pytest
import torch

from linear_attention_op_b200 import Qwen35GatedDeltaNet, _lib, device_error
from oracle import gdn_oracle as O
from tests._util import STATE_TOL, check, requires_b200

pytestmark = [pytest.mark.gpu, requires_b200]


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("hidden, hk, hv, B", [(1024, 16, 16, 3), (4096, 16, 32, 64)])
def test_static_decode_matches_forward_two_calls(hidden, hk, hv, B):
    w = O.make_weights(hidden, hk, hv, seed=21)
    layer = Qwen35GatedDeltaNet(weights=w, batch=B)
    s0 = torch.randn(B, hv, 128, 128, generator=torch.Generator().manual_seed(22)) * 0.1
    c0 = torch.randn(B, 3, layer.conv_dim_local, generator=torch.Generator().manual_seed(23))
    xs = O.make_hidden(B, 2, hidden, seed=24).to("cuda", torch.bfloat16)
    # reference: the existing entry point
    layer.set_state(s0, c0)
    want = [layer.forward_into(xs[:, t:t + 1].contiguous(), torch.empty_like(xs[:, :1])).clone() for t in range(2)]
    want_s, want_c = layer.rec_state.clone(), layer.conv_state.clone()
    # the allocation-free entry point, two calls in a row on the same state buffers
    layer.set_state(s0, c0)
    got = []
    for t in range(2):
        x = xs[:, t:t + 1].contiguous()
        out = torch.full_like(x, float("nan"))
        _lib.call("gdn_layer_decode_static", layer._h.handle, _p(x), B, _p(layer.rec_state), _p(layer.conv_state),
                  _p(out), _stream())
        got.append(out)
    assert device_error() == 0
    for t in range(2):
        check(f"static decode call {t}", got[t], want[t])
    check("static decode state", layer.rec_state, want_s, max_rel=STATE_TOL)
    check("static decode conv state", layer.conv_state, want_c, max_rel=1e-4)
    # and against the CPU oracle on the same inputs and starting state
    with torch.no_grad():
        o_want, o_s, o_c = O.layer_forward(w, xs.float().cpu(), rec_state=s0, conv_state=c0, mode="recurrent")
    check("static decode vs oracle", torch.cat(got, 1), o_want)
    check("static decode state vs oracle", layer.rec_state, o_s, max_rel=STATE_TOL)
    check("static decode conv state vs oracle", layer.conv_state, o_c, max_rel=1e-4)


def test_static_decode_rejects_batch_beyond_scratch():
    w = O.make_weights(4096, 16, 32, seed=25)
    B = 200  # 200 * (4 * 12352 + 2 * 4096) bytes > 8 MiB
    layer = Qwen35GatedDeltaNet(weights=w, batch=1)
    x = torch.zeros(B, 1, 4096, dtype=torch.bfloat16, device="cuda")
    s = torch.zeros(B, 32, 128, 128, device="cuda")
    c = torch.zeros(B, 3, layer.conv_dim_local, device="cuda")
    out = torch.empty_like(x)
    st = _lib.lib().gdn_layer_decode_static(layer._h.handle, _p(x), B, _p(s), _p(c), _p(out), _stream())
    assert st == 1
    assert b"static array" in _lib.lib().gdn_last_error_string()
