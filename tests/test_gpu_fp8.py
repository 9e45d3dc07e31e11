"""fp8 mode (gdn_layer_set_weight_format(GDN_WEIGHTS_FP8_E4M3); the reference's weight_dtype=bfloat8_b
counterpart) against the oracle run with the same quantisation (fp8_weights, act_fp8): decode steps are
e4m3 x e4m3 GEMMs with per-row / per-token power-of-two scales, prefill uses the dequantised weights."""
import ctypes

import pytest
import torch

from linear_attention_op_b200 import GDNError, Qwen35GatedDeltaNet, device_error
from linear_attention_op_b200._lib import call
from oracle import gdn_oracle as O
from tests._util import STATE_TOL, check, requires_b200

pytestmark = [pytest.mark.gpu, requires_b200]


def test_fp8_decode_9b_batch64_random_state():
    w = O.make_weights(4096, 16, 32, seed=60)
    B = 64
    x = O.make_hidden(B, 3, 4096, seed=61)
    s0 = torch.randn(B, 32, 128, 128, generator=torch.Generator().manual_seed(62)) * 0.1
    want, s, c = O.layer_forward(O.fp8_weights(w), x, rec_state=s0, mode="recurrent", act_fp8=True)
    layer = Qwen35GatedDeltaNet(weights=w, batch=B, weight_dtype="fp8")
    layer.set_state(rec_state=s0)
    got = torch.cat([layer(x[:, t:t + 1]) for t in range(3)], 1)
    assert device_error() == 0
    check("fp8 decode out", got, want)
    check("fp8 decode state", layer.get_recurrent_state(), s, max_rel=STATE_TOL)
    check("fp8 decode conv", layer.get_conv_state(), c, max_rel=1e-4)
    bf16_ref = O.layer_forward(w, x, rec_state=s0, mode="recurrent")[0]
    print(f"fp8 vs bf16 oracle: max_abs_rel={O.max_abs_rel(got.float(), bf16_ref):.3e}")


@pytest.mark.parametrize("hidden, hk, hv, B", [(1024, 16, 16, 2), (2048, 16, 32, 3)])
def test_fp8_prefill_then_decode(hidden, hk, hv, B):
    w = O.make_weights(hidden, hk, hv, seed=63)
    wq = O.fp8_weights(w)
    x = O.make_hidden(B, 70, hidden, seed=64)
    want_pre, s, c = O.layer_forward(wq, x[:, :66], mode="chunk")
    want_dec, s, c = O.layer_forward(wq, x[:, 66:], s, c, mode="recurrent", act_fp8=True)
    layer = Qwen35GatedDeltaNet(weights=w, batch=B, weight_dtype="fp8")
    got_pre = layer(x[:, :66])
    got_dec = torch.cat([layer(x[:, t:t + 1]) for t in range(66, 70)], 1)
    assert device_error() == 0
    check("fp8 prefill out", got_pre, want_pre)
    check("fp8 decode out", got_dec, want_dec)
    check("fp8 state", layer.get_recurrent_state(), s, max_rel=STATE_TOL)


def test_fp8_unsupported_cases_fail_loudly():
    w = O.make_weights(1024, 16, 16, seed=65)
    with pytest.raises(GDNError):  # tensor parallel: out_proj row scales would differ per shard
        Qwen35GatedDeltaNet(weights=w, batch=1, tp_rank=0, tp_size=2, weight_dtype="fp8")
    layer = Qwen35GatedDeltaNet(weights=w, batch=1, weight_dtype="fp8")
    x = torch.zeros(1, 1, 1024, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(GDNError):  # the static-scratch decode has no fp8 variant
        p = lambda t: ctypes.c_void_p(t.data_ptr())
        call("gdn_layer_decode_static", layer._h.handle, p(x), 1, p(layer.rec_state), p(layer.conv_state),
             p(torch.empty_like(x)), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    with pytest.raises(GDNError):  # one way: the bf16 originals are gone
        call("gdn_layer_set_weight_format", layer._h.handle, 0)
