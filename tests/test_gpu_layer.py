"""Full GDN layer on the B200 against the HF golden fixtures and the CPU oracle (cases of
9B/test_gdn_layer.py:42-73 and 0.8B/test_gdn_l1.py:82-100, plus the benchmark configs at test size)."""
import numpy as np
import pytest
import torch

from linear_attention_op_b200 import GDNStack, Qwen35GatedDeltaNet, device_error
from oracle import gdn_oracle as O
from tests._util import OUT_TOL, STATE_TOL, T, check, fixture_weights, requires_b200

pytestmark = [pytest.mark.gpu, requires_b200]


@pytest.fixture(scope="module")
def hf_fixture(golden_dir):
    return np.load(golden_dir / "layer_hf.npz")


def test_hf_prefill_then_decode(hf_fixture):
    z = hf_fixture
    w = fixture_weights(z)
    x = T(z["x"])
    t0 = int(z["t0"][0])
    B = x.shape[0]
    layer = Qwen35GatedDeltaNet(weights=w, batch=B)
    y = layer(x[:, :t0])
    assert device_error() == 0
    check("prefill out", y, T(z["y_pre"]))
    check("prefill rec state", layer.get_recurrent_state(), T(z["rec_pre"]), max_rel=STATE_TOL)
    check("prefill conv state", layer.get_conv_state(), O.hf_conv_state_to_abi(T(z["conv_pre"])), max_rel=1e-4)
    ys = [layer(x[:, t:t + 1]) for t in range(t0, x.shape[1])]
    check("decode out", torch.cat(ys, 1), T(z["y_dec"]))
    check("decode rec state", layer.get_recurrent_state(), T(z["rec_dec"]), max_rel=STATE_TOL)
    check("decode conv state", layer.get_conv_state(), O.hf_conv_state_to_abi(T(z["conv_dec"])), max_rel=1e-4)


def test_hf_one_shot_and_single_token(hf_fixture):
    z = hf_fixture
    w = fixture_weights(z)
    x = T(z["x"])
    check("one-shot 43 tokens", Qwen35GatedDeltaNet(weights=w, batch=x.shape[0])(x), T(z["y_full"]))
    x1 = T(z["x1"])
    check("single token", Qwen35GatedDeltaNet(weights=w, batch=1)(x1), T(z["y_one"]))


@pytest.mark.parametrize("B, T_", [(1, 2), (3, 63), (2, 64), (3, 65), (1, 130), (4, 9), (1, 40)])
def test_ragged_prefill_shapes(hf_fixture, B, T_):
    w = fixture_weights(hf_fixture)
    x = O.make_hidden(B, T_, w.hidden, seed=B * 100 + T_)
    want, s, c = O.layer_forward(w, x, mode="chunk")
    layer = Qwen35GatedDeltaNet(weights=w, batch=B)
    check(f"out B={B} T={T_}", layer(x), want)
    check("state", layer.get_recurrent_state(), s, max_rel=STATE_TOL)
    check("conv", layer.get_conv_state(), c, max_rel=1e-4)


def test_long_prefill_split_across_calls(hf_fixture):
    """Prefill in pieces continues from the carried state exactly like one long call
    (9B/test_gdn_layer.py:66-73: 300 tokens over 3 launches)."""
    w = fixture_weights(hf_fixture)
    x = O.make_hidden(1, 300, w.hidden, seed=2)
    want, s, _ = O.layer_forward(w, x, mode="chunk")
    layer = Qwen35GatedDeltaNet(weights=w, batch=1)
    got = torch.cat([layer(x[:, :128]), layer(x[:, 128:256]), layer(x[:, 256:])], 1)
    check("split prefill", got, want)
    check("split prefill state", layer.get_recurrent_state(), s, max_rel=STATE_TOL)


def test_config0_08b_decode_128_tokens():
    """Config 0: 0.8B-shaped layer, batch 1, 128 sequential decode tokens from zero state."""
    w = O.make_weights(1024, 16, 16, seed=0)
    x = O.make_hidden(1, 128, 1024, seed=0)
    want, s, c = O.layer_forward(w, x, mode="recurrent")
    layer = Qwen35GatedDeltaNet(weights=w, batch=1)
    got = torch.cat([layer(x[:, t:t + 1]) for t in range(128)], 1)
    check("cfg0 decode out", got, want)
    check("cfg0 state", layer.get_recurrent_state(), s, max_rel=STATE_TOL)
    check("cfg0 conv", layer.get_conv_state(), c, max_rel=1e-4)


def test_config1_08b_prefill_2048_state_vs_sequential():
    """Config 1: 0.8B prefill T=2048, chunk 64; final state against 2048 sequential decode steps."""
    w = O.make_weights(1024, 16, 16, seed=0)
    x = O.make_hidden(1, 2048, 1024, seed=1)
    want, s_seq, c = O.layer_forward(w, x, mode="recurrent")
    layer = Qwen35GatedDeltaNet(weights=w, batch=1)
    check("cfg1 prefill out", layer(x), want)
    check("cfg1 final state vs sequential", layer.get_recurrent_state(), s_seq, max_rel=STATE_TOL)
    check("cfg1 conv", layer.get_conv_state(), c, max_rel=1e-4)


def test_config2_9b_decode_b64_random_state():
    """Config 2 at test length: 9B-shaped layer, batch 64, initial state N(0, 0.1), 3 decode steps."""
    w = O.make_weights(4096, 16, 32, seed=2)
    B = 64
    x = O.make_hidden(B, 3, 4096, seed=2)
    s0 = torch.randn(B, 32, 128, 128, generator=torch.Generator().manual_seed(3)) * 0.1
    want, s, c = O.layer_forward(w, x, rec_state=s0, mode="recurrent")
    layer = Qwen35GatedDeltaNet(weights=w, batch=B)
    layer.set_state(rec_state=s0)
    got = torch.cat([layer(x[:, t:t + 1]) for t in range(3)], 1)
    check("cfg2 decode out", got, want)
    check("cfg2 state", layer.get_recurrent_state(), s, max_rel=STATE_TOL)
    check("cfg2 conv", layer.get_conv_state(), c, max_rel=1e-4)


def test_config3_9b_prefill_at_test_size():
    """Config 3 geometry (9B, chunked prefill) at a size the oracle finishes quickly."""
    w = O.make_weights(4096, 16, 32, seed=3)
    x = O.make_hidden(2, 200, 4096, seed=3)
    want, s, c = O.layer_forward(w, x, mode="chunk")
    layer = Qwen35GatedDeltaNet(weights=w, batch=2)
    check("cfg3 prefill out", layer(x), want)
    check("cfg3 state", layer.get_recurrent_state(), s, max_rel=STATE_TOL)
    check("cfg3 conv", layer.get_conv_state(), c, max_rel=1e-4)


@pytest.mark.parametrize("hk, hv", [(4, 16), (8, 8)])
def test_gqa_ratios_prefill_then_decode(hk, hv):
    """GQA groups of 4 and 1 v-heads per k-head: the decode step keeps the conv in the in_proj epilogue for
    ratios other than 1 and 2 and runs it in the per-k-head decode kernel otherwise."""
    w = O.make_weights(1024, hk, hv, seed=40 + hk)
    B = 3
    x = O.make_hidden(B, 70, 1024, seed=41)
    want, s, c = O.layer_forward(w, x, mode="recurrent")
    layer = Qwen35GatedDeltaNet(weights=w, batch=B)
    got = torch.cat([layer(x[:, :67])] + [layer(x[:, t:t + 1]) for t in range(67, 70)], 1)
    check(f"gqa {hk}/{hv} out", got, want)
    check("state", layer.get_recurrent_state(), s, max_rel=STATE_TOL)
    check("conv", layer.get_conv_state(), c, max_rel=1e-4)


def test_strong_decay_prefill_then_decode():
    """A_log = log(U(1, 64)) (config 4's gate strength): chunk decay underflow must stay finite."""
    w = O.make_weights(1024, 16, 32, seed=4, a_max=64.0)
    x = O.make_hidden(2, 150, 1024, seed=4)
    want, s, _ = O.layer_forward(w, x, mode="recurrent")
    layer = Qwen35GatedDeltaNet(weights=w, batch=2)
    got = torch.cat([layer(x[:, :140])] + [layer(x[:, t:t + 1]) for t in range(140, 150)], 1)
    check("strong decay out", got, want)
    check("strong decay state", layer.get_recurrent_state(), s, max_rel=STATE_TOL)


def test_prefill_matches_decode_steps_on_gpu():
    """Size-independent property: the chunked prefill kernel and T decode steps agree on the device."""
    w = O.make_weights(2048, 16, 32, seed=5)
    x = O.make_hidden(2, 96, 2048, seed=5)
    a = Qwen35GatedDeltaNet(weights=w, batch=2)
    b = Qwen35GatedDeltaNet(weights=w, batch=2)
    ya = a(x)
    yb = torch.cat([b(x[:, t:t + 1]) for t in range(96)], 1)
    check("prefill vs decode out", ya, yb)
    check("prefill vs decode state", a.get_recurrent_state(), b.get_recurrent_state(), max_rel=STATE_TOL)


def test_reset_state():
    w = O.make_weights(1024, 16, 16, seed=6)
    x = O.make_hidden(1, 5, 1024, seed=6)
    layer = Qwen35GatedDeltaNet(weights=w, batch=1)
    y1 = layer(x)
    layer(x)
    layer.reset_state()
    y3 = layer(x)
    assert torch.equal(y1, y3)


def test_tp2_partial_sums_on_one_gpu():
    """Head-parallel shards: rank 0 + rank 1 partial outputs sum to the full layer (all-reduce skipped)."""
    w = O.make_weights(1024, 16, 32, seed=7)
    x = O.make_hidden(2, 70, 1024, seed=7)
    want, s, _ = O.layer_forward(w, x, mode="chunk")
    parts, states = [], []
    for r in range(2):
        L = Qwen35GatedDeltaNet(weights=w, batch=2, tp_rank=r, tp_size=2)
        parts.append(L(x).float())
        states.append(L.get_recurrent_state())
    check("tp2 sum of partials", parts[0] + parts[1], want)
    check("tp2 states", torch.cat(states, 1), s, max_rel=STATE_TOL)


def test_stack_decode_each_layer_keeps_state():
    """0.8B stack, 2 resident layers, batch 3: each layer decodes its own sequence one call at a time
    (0.8B/test_gdn_l1.py:56-73)."""
    ws = [O.make_weights(1024, 16, 16, seed=10 + i) for i in range(2)]
    B, steps = 3, 6
    x = O.make_hidden(B, steps, 1024, seed=11)
    want = [O.layer_forward(w, x, mode="recurrent")[0] for w in ws]
    stack = GDNStack(ws, batch=B)
    got = [[], []]
    for t in range(steps):
        for i in range(2):
            got[i].append(stack(x[:, t], layers=[i]))
    for i in range(2):
        check(f"stack layer {i}", torch.stack(got[i], 1), want[i])


def test_cuda_graph_decode_replay():
    w = O.make_weights(1024, 16, 16, seed=12)
    B = 4
    x = O.make_hidden(B, 4, 1024, seed=12)
    eager = Qwen35GatedDeltaNet(weights=w, batch=B)
    want = torch.cat([eager(x[:, t:t + 1]) for t in range(4)], 1)
    layer = Qwen35GatedDeltaNet(weights=w, batch=B, max_rows=B)
    xin = torch.zeros(B, 1, 1024, dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(xin)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        layer.forward_into(xin, out, stream=s)  # warm-up outside the capture
    torch.cuda.synchronize()
    layer.reset_state()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        layer.forward_into(xin, out, stream=s)
    layer.reset_state()
    outs = []
    for t in range(4):
        xin.copy_(x[:, t:t + 1].to("cuda", torch.bfloat16))
        graph.replay()
        outs.append(out.float().cpu().clone())
    check("graph replay", torch.cat(outs, 1), want, max_rel=1e-6, min_pcc=None, max_fro=None)


def test_tp8_shards_wide_batch_decode_on_one_gpu():
    """The eight head-parallel shards of the 9B layer at 512 sequences (64 per GPU, the 8-GPU benchmark's
    batch) run on one GPU without the all-reduce: their decode in_proj takes 256-token tiles with split-K,
    and the partial outputs sum to the full layer."""
    w = O.make_weights(4096, 16, 32, seed=13)
    B = 512
    x = O.make_hidden(B, 1, 4096, seed=13)
    s0 = torch.randn(B, 32, 128, 128, generator=torch.Generator().manual_seed(14)) * 0.1
    with torch.no_grad():
        want, s, _ = O.layer_forward(w, x, rec_state=s0, mode="recurrent")
    total = torch.zeros(B, 1, 4096)
    states = []
    for r in range(8):
        L = Qwen35GatedDeltaNet(weights=w, batch=B, tp_rank=r, tp_size=8)
        L.set_state(rec_state=s0[:, 4 * r:4 * (r + 1)])
        total += L(x).float()
        states.append(L.get_recurrent_state())
        del L
    assert device_error() == 0
    check("tp8 shards at B=512: sum of partials", total, want)
    check("tp8 shards at B=512: states", torch.cat(states, 1), s, max_rel=STATE_TOL)
