"""A whole multi-layer decode step captured in ONE CUDA graph (the reference records the stacked decode
step once and replays it: 0.8B/gdn_l1.py:309-325, 0.8B/bench_decode.py:44-60), with the stack's layers
sharing one workspace and a bounded prefill (row limit) before it."""
import pytest
import torch

from linear_attention_op_b200 import GDNStack, device_error
from oracle import gdn_oracle as O
from tests._util import STATE_TOL, check, requires_b200

pytestmark = [pytest.mark.gpu, requires_b200]


def test_stack_decode_step_in_one_graph_is_bit_identical_to_eager():
    L, B, H, T0, steps = 4, 8, 4096, 100, 6
    ws = [O.make_weights(H, 16, 32, seed=200 + i, a_max=64.0) for i in range(L)]
    x = O.make_hidden(B, T0 + steps, H, seed=201).to("cuda", torch.bfloat16)
    eager = GDNStack(ws, batch=B, max_rows=B * 64)
    graphed = GDNStack(ws, batch=B, max_rows=B * 64)
    for st in (eager, graphed):  # bounded prefill: 64-token pieces of all 8 sequences
        bufs = [torch.empty(B, T0, H, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
        st.forward_into(x[:, :T0].contiguous(), [bufs[i % 2] for i in range(L)])
    torch.cuda.synchronize()
    want = []
    for t in range(steps):
        outs = eager.allocate_activations(1)
        eager.forward_into(x[:, T0 + t:T0 + t + 1].contiguous(), outs)
        want.append(outs[-1].clone())

    xin = torch.empty(B, 1, H, dtype=torch.bfloat16, device="cuda")
    outs = graphed.allocate_activations(1)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        graphed.forward_into(xin, outs, stream=s)
    got = []
    for t in range(steps):
        xin.copy_(x[:, T0 + t:T0 + t + 1])
        g.replay()
        got.append(outs[-1].clone())
    torch.cuda.synchronize()
    assert device_error() == 0
    for t in range(steps):
        assert torch.equal(got[t], want[t]), f"step {t}: graph replay differs from eager"
    for i in range(L):
        assert torch.equal(graphed.layers[i].rec_state, eager.layers[i].rec_state), f"layer {i} state"
    # and the first layer against the oracle (prefill in pieces, then the decode steps)
    xc = x.float().cpu()
    with torch.no_grad():
        _, s0, c0 = O.layer_forward(ws[0], xc[:, :T0], mode="chunk")
        _, s0, c0 = O.layer_forward(ws[0], xc[:, T0:], s0, c0, mode="recurrent")
    check("stack layer 0 state vs oracle", graphed.get_recurrent_state(0), s0, max_rel=STATE_TOL)
