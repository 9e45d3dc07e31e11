"""Row-limited prefill (gdn_layer_set_max_rows, the reference's max_rows: 9B/gdn_layer.py:55-66, 282-292),
workspace reservation for many sequences (gdn_layer_reserve_batch), the pipelined host entry point
(forward_host_async) and the device check of the C-ABI."""
import ctypes

import pytest
import torch

from linear_attention_op_b200 import GDNError, Qwen35GatedDeltaNet, device_error
from linear_attention_op_b200._lib import call
from oracle import gdn_oracle as O
from tests._util import STATE_TOL, check, requires_b200

pytestmark = [pytest.mark.gpu, requires_b200]


@pytest.mark.parametrize("B, T_, max_rows", [(3, 300, 192), (3, 300, 100), (3, 298, 99), (1, 300, 128), (2, 130, 130)])
def test_row_limited_prefill_matches_one_call(B, T_, max_rows):
    """Pieces of max_rows // B tokens of every sequence (64-aligned when >= 64) carry the state and give the
    one-call result."""
    w = O.make_weights(1024, 16, 32, seed=50)
    x = O.make_hidden(B, T_, 1024, seed=51)
    want, s, c = O.layer_forward(w, x, mode="chunk")
    layer = Qwen35GatedDeltaNet(weights=w, batch=B, max_rows=max_rows)
    ws = layer.workspace_bytes()
    got = layer(x)
    assert device_error() == 0
    assert layer.workspace_bytes() == ws, "the reservation covers calls of any length"
    check(f"row limit {max_rows} out", got, want)
    check("row limit state", layer.get_recurrent_state(), s, max_rel=STATE_TOL)
    check("row limit conv", layer.get_conv_state(), c, max_rel=1e-4)


def test_row_limit_below_batch_is_rejected():
    w = O.make_weights(1024, 16, 16, seed=52)
    with pytest.raises(ValueError):
        Qwen35GatedDeltaNet(weights=w, batch=4, max_rows=2)
    layer = Qwen35GatedDeltaNet(weights=w, batch=4)
    call("gdn_layer_set_max_rows", layer._h.handle, 2)
    with pytest.raises(GDNError, match="below the batch"):
        layer(O.make_hidden(4, 10, 1024, seed=53))


def test_reserve_batch_covers_many_short_sequences():
    """128 prompts of 16 tokens need 128 chunks: gdn_layer_reserve_batch(2048, 128) reserves them, so the
    call allocates nothing (it runs under stream capture, where an allocation is refused)."""
    w = O.make_weights(1024, 16, 16, seed=54)
    B, T_ = 128, 16
    x = O.make_hidden(B, T_, 1024, seed=55)
    want = O.layer_forward(w, x, mode="chunk")[0]
    layer = Qwen35GatedDeltaNet(weights=w, batch=B)
    layer.reserve(B * T_, B)
    xd = x.to("cuda", torch.bfloat16)
    out = torch.empty_like(xd)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        layer.forward_into(xd, out, stream=s)
    layer.reset_state()
    g.replay()
    torch.cuda.synchronize()
    assert device_error() == 0
    check("reserved 128 x 16 prefill (graph)", out, want)


def test_forward_host_async_matches_forward_into():
    w = O.make_weights(2048, 16, 32, seed=56)
    B, steps = 8, 6
    x = O.make_hidden(B, steps, 2048, seed=57).to(torch.bfloat16)
    a = Qwen35GatedDeltaNet(weights=w, batch=B)
    b = Qwen35GatedDeltaNet(weights=w, batch=B)
    want = [a.forward_into(x[:, t:t + 1].cuda().contiguous(), torch.empty(B, 1, 2048, dtype=torch.bfloat16,
                                                                         device="cuda")).cpu() for t in range(steps)]
    xh = [x[:, t:t + 1].contiguous().pin_memory() for t in range(steps)]
    yh = [torch.empty(B, 1, 2048, dtype=torch.bfloat16).pin_memory() for _ in range(steps)]
    evs = [b.forward_host_async(xh[t], yh[t]) for t in range(steps)]
    evs[-1].synchronize()
    torch.cuda.synchronize()
    assert device_error() == 0
    for t in range(steps):
        assert torch.equal(yh[t], want[t]), f"step {t}"
    assert torch.equal(a.rec_state, b.rec_state)


def test_call_on_another_device_is_rejected():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    w = O.make_weights(1024, 16, 16, seed=58)
    layer = Qwen35GatedDeltaNet(weights=w, batch=1, device="cuda:0")
    x = torch.zeros(1, 1, 1024, dtype=torch.bfloat16, device="cuda:0")
    out = torch.empty_like(x)
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    with torch.cuda.device(1):
        with pytest.raises(GDNError, match="lives on device 0"):
            call("gdn_layer_forward", layer._h.handle, p(x), 1, 1, p(layer.rec_state), p(layer.conv_state), p(out),
                 None, ctypes.c_void_p(0))
        with pytest.raises(GDNError, match="lives on device 0"):
            call("gdn_layer_decode_static", layer._h.handle, p(x), 1, p(layer.rec_state), p(layer.conv_state),
                 p(out), ctypes.c_void_p(0))
