"""The headline configurations at their full length against the CPU oracle (the long-sequence state check of
9B/test_gated_delta_l1.py:69-78, at the benchmark's sizes):

* config 3's geometry over one whole sequence: 9B layer, T = 8192 tokens (128 chunks) of chunked prefill --
  the chunk scan's fp32 state, carried through 128 chunk products of bf16 hi/lo operands, stays within the
  1e-3 state bar and the output within 2e-2;
* config 2 for all of its 256 decode steps: 9B layer, batch 64, from the N(0, 0.1) state.
"""
import pytest
import torch

from linear_attention_op_b200 import Qwen35GatedDeltaNet, device_error
from oracle import gdn_oracle as O
from tests._util import STATE_TOL, check, requires_b200

pytestmark = [pytest.mark.gpu, requires_b200]


def test_config3_full_sequence_8192_tokens():
    w = O.make_weights(4096, 16, 32, seed=30)
    x = O.make_hidden(1, 8192, 4096, seed=31)
    with torch.no_grad():
        want, s, c = O.layer_forward(w, x, mode="chunk")
    layer = Qwen35GatedDeltaNet(weights=w, batch=1)
    got = layer(x)
    assert device_error() == 0
    check("cfg3 T=8192 out", got, want)
    check("cfg3 T=8192 final state", layer.get_recurrent_state(), s, max_rel=STATE_TOL)
    check("cfg3 T=8192 conv state", layer.get_conv_state(), c, max_rel=1e-4)
    # the last 64-token chunk alone (where accumulated error would show first)
    check("cfg3 T=8192 last chunk", got[:, -64:], want[:, -64:])


def test_config2_all_256_decode_steps():
    w = O.make_weights(4096, 16, 32, seed=32)
    B, steps = 64, 256
    x = O.make_hidden(B, steps, 4096, seed=33)
    s0 = torch.randn(B, 32, 128, 128, generator=torch.Generator().manual_seed(34)) * 0.1
    layer = Qwen35GatedDeltaNet(weights=w, batch=B)
    layer.set_state(rec_state=s0)
    xd = x.to("cuda", torch.bfloat16)
    outs = torch.empty(steps, B, 1, 4096, dtype=torch.bfloat16, device="cuda")
    for t in range(steps):
        layer.forward_into(xd[:, t:t + 1].contiguous(), outs[t])
    got = outs[:, :, 0].transpose(0, 1).float().cpu()
    assert device_error() == 0
    with torch.no_grad():
        want, s, c = O.layer_forward(w, x, rec_state=s0, mode="recurrent")
    check("cfg2 256 steps out", got, want)
    check("cfg2 256 steps final state", layer.get_recurrent_state(), s, max_rel=STATE_TOL)
    check("cfg2 256 steps conv state", layer.get_conv_state(), c, max_rel=1e-4)
    check("cfg2 last step", got[:, -1], want[:, -1])
