"""Recurrence-only op (mirror of GatedDeltaRuleL1) against the oracle and the reference.py golden vectors
(the cases of 9B/test_gated_delta_l1.py:48-92)."""
import numpy as np
import pytest
import torch

from linear_attention_op_b200 import GatedDeltaRule, device_error
from oracle import gdn_oracle as O
from tests._util import STATE_TOL, T, check, requires_b200

pytestmark = [pytest.mark.gpu, requires_b200]


@pytest.mark.parametrize("case", ["a", "b"])
def test_golden_reference_py(golden_dir, case):
    z = np.load(golden_dir / "recurrence_ref.npz")
    get = lambda k: T(z[f"{case}_{k}"])
    q, k, v, g, beta = get("q"), get("k"), get("v"), get("g"), get("beta")
    B, _, _, _ = q.shape
    Hv = v.shape[2]
    init = get("init")
    op = GatedDeltaRule(B * Hv, initial_state=None if init.numel() == 0 else init)
    o = op(q, k, v, g, beta)
    assert device_error() == 0
    check("output", o, get("o"), max_rel=1e-4)
    check("state", op.get_state(), get("state").reshape(B * Hv, 128, 128), max_rel=1e-4)


@pytest.mark.parametrize("B, Hk, Hv, T_", [(1, 16, 32, 1), (1, 16, 32, 45), (1, 8, 16, 7), (4, 16, 32, 3)])
def test_matches_reference(B, Hk, Hv, T_):
    q, k, v, g, beta = O.make_recurrence_inputs(B, T_, Hk, Hv)
    init = torch.randn(B, Hv, 128, 128, generator=torch.Generator().manual_seed(9)) * 0.1
    want_o, want_s = O.recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=init)
    op = GatedDeltaRule(B * Hv, initial_state=init.reshape(B * Hv, 128, 128))
    check("output", op(q, k, v, g, beta), want_o, max_rel=1e-4)
    check("state", op.get_state(), want_s.reshape(B * Hv, 128, 128), max_rel=STATE_TOL)


def test_long_sequence_slow_decay():
    B, Hk, Hv, T_ = 1, 16, 32, 1024
    q, k, v, _, beta = O.make_recurrence_inputs(B, T_, Hk, Hv, seed=3)
    g = torch.nn.functional.logsigmoid(torch.randn(B, T_, Hv, generator=torch.Generator().manual_seed(4)) + 5.0)
    want_o, want_s = O.recurrent_gated_delta_rule(q, k, v, g, beta)
    op = GatedDeltaRule(B * Hv)
    check("long output", op(q, k, v, g, beta), want_o, max_rel=1e-3)
    check("long state", op.get_state(), want_s.reshape(B * Hv, 128, 128), max_rel=STATE_TOL)


def test_decode_loop_keeps_state_in_place():
    B, Hk, Hv, steps = 1, 16, 32, 64
    q, k, v, g, beta = O.make_recurrence_inputs(B, steps, Hk, Hv, seed=1)
    want_o, want_s = O.recurrent_gated_delta_rule(q, k, v, g, beta)
    op = GatedDeltaRule(B * Hv)
    addr = op.state.data_ptr()
    outs = [op(q[:, t:t + 1], k[:, t:t + 1], v[:, t:t + 1], g[:, t:t + 1], beta[:, t:t + 1]) for t in range(steps)]
    assert op.state.data_ptr() == addr
    check("decode output", torch.cat(outs, dim=1), want_o, max_rel=1e-4)
    check("decode state", op.get_state(), want_s.reshape(B * Hv, 128, 128), max_rel=STATE_TOL)


def test_no_l2norm_and_custom_scale():
    q, k, v, g, beta = O.make_recurrence_inputs(2, 5, 2, 4, seed=7)
    k = torch.nn.functional.normalize(k, dim=-1)
    want_o, want_s = O.recurrent_gated_delta_rule(q, k, v, g, beta, use_qk_l2norm=False, scale=0.05)
    op = GatedDeltaRule(8)
    check("output", op(q, k, v, g, beta, use_qk_l2norm=False, scale=0.05), want_o, max_rel=1e-4)
    check("state", op.get_state(), want_s.reshape(8, 128, 128), max_rel=STATE_TOL)
