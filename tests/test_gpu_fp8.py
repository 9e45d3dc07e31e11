"""fp8 modes against the oracle run with the same quantisation.

* weight-only (gdn_layer_set_weight_format(GDN_WEIGHTS_FP8_WEIGHT_ONLY), weight_dtype="fp8"): the reference's
  bfloat8_b semantics -- weights quantised, activations not -- checked as the reference checks its
  low-precision modes, against the layer run with the same quantised weights (0.8B/test_gdn_l1.py:24-52,
  59-63: rel-Frobenius < 1.5e-2, PCC > 0.9999), plus the spec's max-abs-rel 2e-2 and state 1e-3; single GPU
  and two head-parallel shards;
* W8A8 (GDN_WEIGHTS_FP8_E4M3, weight_dtype="fp8_w8a8"): decode activations quantised per token too (e4m3 x
  e4m3 GEMMs), against the oracle with act_fp8."""
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
    layer = Qwen35GatedDeltaNet(weights=w, batch=B, weight_dtype="fp8_w8a8")
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
    layer = Qwen35GatedDeltaNet(weights=w, batch=B, weight_dtype="fp8_w8a8")
    got_pre = layer(x[:, :66])
    got_dec = torch.cat([layer(x[:, t:t + 1]) for t in range(66, 70)], 1)
    assert device_error() == 0
    check("fp8 prefill out", got_pre, want_pre)
    check("fp8 decode out", got_dec, want_dec)
    check("fp8 state", layer.get_recurrent_state(), s, max_rel=STATE_TOL)


def test_weight_only_fp8_decode_9b_batch64():
    w = O.make_weights(4096, 16, 32, seed=66)
    B = 64
    x = O.make_hidden(B, 3, 4096, seed=67)
    s0 = torch.randn(B, 32, 128, 128, generator=torch.Generator().manual_seed(68)) * 0.1
    with torch.no_grad():
        want, s, c = O.layer_forward(O.fp8_weights(w), x, rec_state=s0, mode="recurrent")
    layer = Qwen35GatedDeltaNet(weights=w, batch=B, weight_dtype="fp8")
    layer.set_state(rec_state=s0)
    got = torch.cat([layer(x[:, t:t + 1]) for t in range(3)], 1)
    assert device_error() == 0
    check("fp8 weight-only decode out", got, want)
    check("fp8 weight-only decode state", layer.get_recurrent_state(), s, max_rel=STATE_TOL)
    bf16_ref = O.layer_forward(w, x, rec_state=s0, mode="recurrent")[0]
    print(f"fp8 weight-only vs bf16 weights: max_abs_rel={O.max_abs_rel(got.float(), bf16_ref):.3e} "
          f"rel_fro={O.rel_fro(got.float(), bf16_ref):.3e} pcc={O.pcc(got.float(), bf16_ref):.6f}")


@pytest.mark.parametrize("hidden, hk, hv, B", [(1024, 16, 16, 2), (4096, 16, 32, 3)])
def test_weight_only_fp8_prefill_then_decode(hidden, hk, hv, B):
    w = O.make_weights(hidden, hk, hv, seed=69)
    wq = O.fp8_weights(w)
    x = O.make_hidden(B, 70, hidden, seed=70)
    with torch.no_grad():
        want_pre, s, c = O.layer_forward(wq, x[:, :66], mode="chunk")
        want_dec, s, c = O.layer_forward(wq, x[:, 66:], s, c, mode="recurrent")
    layer = Qwen35GatedDeltaNet(weights=w, batch=B, weight_dtype="fp8")
    got_pre = layer(x[:, :66])
    got_dec = torch.cat([layer(x[:, t:t + 1]) for t in range(66, 70)], 1)
    assert device_error() == 0
    check("fp8 weight-only prefill out", got_pre, want_pre)
    check("fp8 weight-only decode out", got_dec, want_dec)
    check("fp8 weight-only state", layer.get_recurrent_state(), s, max_rel=STATE_TOL)


def test_weight_only_fp8_head_parallel_shards_sum_to_one_gpu():
    """Two head-parallel shards quantise out_proj with the scales of the whole rows, so their partial
    outputs sum to the single-GPU fp8 layer's (decode steps on the one GPU, all-reduce skipped)."""
    w = O.make_weights(2048, 16, 32, seed=71)
    B = 4
    x = O.make_hidden(B, 3, 2048, seed=72)
    with torch.no_grad():
        want, s, _ = O.layer_forward(O.fp8_weights(w), x, mode="recurrent")
    parts, states = [], []
    for r in range(2):
        L = Qwen35GatedDeltaNet(weights=w, batch=B, tp_rank=r, tp_size=2, weight_dtype="fp8")
        parts.append(torch.cat([L(x[:, t:t + 1]).float() for t in range(3)], 1))
        states.append(L.get_recurrent_state())
    one = Qwen35GatedDeltaNet(weights=w, batch=B, weight_dtype="fp8")
    whole = torch.cat([one(x[:, t:t + 1]).float() for t in range(3)], 1)
    assert device_error() == 0
    check("fp8 weight-only tp2 partial sum vs oracle", parts[0] + parts[1], want)
    check("fp8 weight-only tp2 partial sum vs one GPU", parts[0] + parts[1], whole)
    check("fp8 weight-only tp2 states", torch.cat(states, 1), s, max_rel=STATE_TOL)


def test_fp8_unsupported_cases_fail_loudly():
    w = O.make_weights(1024, 16, 16, seed=65)
    with pytest.raises(GDNError):  # W8A8 with tensor parallel: per-token activation scales differ per shard
        Qwen35GatedDeltaNet(weights=w, batch=1, tp_rank=0, tp_size=2, weight_dtype="fp8_w8a8")
    layer = Qwen35GatedDeltaNet(weights=w, batch=1, weight_dtype="fp8_w8a8")
    x = torch.zeros(1, 1, 1024, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(GDNError):  # the static-scratch decode has no fp8 variant
        p = lambda t: ctypes.c_void_p(t.data_ptr())
        call("gdn_layer_decode_static", layer._h.handle, p(x), 1, p(layer.rec_state), p(layer.conv_state),
             p(torch.empty_like(x)), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    with pytest.raises(GDNError):  # one way: the bf16 originals are gone
        call("gdn_layer_set_weight_format", layer._h.handle, 0)
