"""The decoder layer around the mixer (gdn_decoder_*: input RMSNorm, GDN mixer, residual, post RMSNorm,
SwiGLU MLP, residual) on the B200 against HF Qwen3_5DecoderLayer (the golden fixture, prefill then cached
decode) and against the CPU oracle at the 9B geometry (hidden 4096, intermediate 12288)."""
import numpy as np
import pytest
import torch

from linear_attention_op_b200 import DecoderMlpWeights, GDNError, Qwen35DecoderLayer, device_error
from oracle import gdn_oracle as O
from tests._util import STATE_TOL, T, bf16, check, fixture_weights, requires_b200

pytestmark = [pytest.mark.gpu, requires_b200]


def _mlp(dw: O.DecoderWeights) -> DecoderMlpWeights:
    return DecoderMlpWeights(dw.input_norm_w, dw.post_norm_w, dw.w_gate, dw.w_up, dw.w_down, dw.eps)


def _decoder_weights(hidden, hk, hv, inter, seed):
    gen = torch.Generator().manual_seed(seed + 1000)
    rn = lambda *s: O.bf16_round(torch.randn(*s, generator=gen) * 0.02)
    return O.DecoderWeights(
        gdn=O.make_weights(hidden, hk, hv, seed=seed),
        input_norm_w=torch.rand(hidden, generator=gen) - 0.5, post_norm_w=torch.rand(hidden, generator=gen) - 0.5,
        w_gate=rn(inter, hidden), w_up=rn(inter, hidden), w_down=rn(hidden, inter))


def test_decoder_matches_hf_fixture(golden_dir):
    z = np.load(golden_dir / "decoder_hf.npz")
    dw = O.DecoderWeights(gdn=fixture_weights(z), input_norm_w=T(z["input_norm_w"]), post_norm_w=T(z["post_norm_w"]),
                          w_gate=bf16(z["w_gate"]), w_up=bf16(z["w_up"]), w_down=bf16(z["w_down"]))
    x = T(z["x"])
    t0 = int(z["t0"][0])
    layer = Qwen35DecoderLayer(batch=x.shape[0], mixer_weights=dw.gdn, mlp_weights=_mlp(dw))
    y = layer(x[:, :t0])
    assert device_error() == 0
    check("decoder prefill vs HF", y, T(z["y_pre"]))
    ys = [layer(x[:, t:t + 1]) for t in range(t0, x.shape[1])]
    check("decoder decode vs HF", torch.cat(ys, 1), T(z["y_dec"]))
    # The fixture ran HF in fp32.  The library's decoder keeps its activations in bf16 as a bf16 HF model
    # does (the input RMSNorm's output is the mixer's input), so the fp32 state is held to the spec's 1e-3
    # against the oracle with the same bf16 activation roundings, and to 5e-3 against the fp32 fixture.
    check("decoder rec state vs HF (fp32 activations)", layer.get_recurrent_state(), T(z["rec_dec"]), max_rel=5e-3)
    with torch.no_grad():
        _, s, c = O.decoder_layer_forward(dw, x[:, :t0], mode="chunk", bf16_acts=True)
        for t in range(t0, x.shape[1]):
            _, s, c = O.decoder_layer_forward(dw, x[:, t:t + 1], s, c, mode="recurrent", bf16_acts=True)
    check("decoder rec state vs oracle (bf16 activations)", layer.get_recurrent_state(), s, max_rel=STATE_TOL)
    check("decoder conv state vs oracle (bf16 activations)", layer.get_conv_state(), c, max_rel=1e-4)


def test_decoder_9b_prefill_then_decode_vs_oracle():
    dw = _decoder_weights(4096, 16, 32, 12288, seed=70)
    B, t0, steps = 2, 130, 3
    x = O.make_hidden(B, t0 + steps, 4096, seed=71)
    with torch.no_grad():
        want_pre, s, c = O.decoder_layer_forward(dw, x[:, :t0], mode="chunk", bf16_acts=True)
        want_dec, s, c = O.decoder_layer_forward(dw, x[:, t0:], s, c, mode="recurrent", bf16_acts=True)
    layer = Qwen35DecoderLayer(batch=B, mixer_weights=dw.gdn, mlp_weights=_mlp(dw))
    got_pre = layer(x[:, :t0])
    got_dec = torch.cat([layer(x[:, t:t + 1]) for t in range(t0, t0 + steps)], 1)
    assert device_error() == 0
    check("9B decoder prefill", got_pre, want_pre)
    check("9B decoder decode", got_dec, want_dec)
    check("9B decoder state", layer.get_recurrent_state(), s, max_rel=STATE_TOL)


def test_decoder_9b_decode_batch64_vs_oracle():
    """Batch-64 decode: the gate/up GEMM's 192 weight tiles run two CTAs per SM, the down GEMM split-K."""
    dw = _decoder_weights(4096, 16, 32, 12288, seed=72)
    B = 64
    x = O.make_hidden(B, 2, 4096, seed=73)
    s0 = torch.randn(B, 32, 128, 128, generator=torch.Generator().manual_seed(74)) * 0.1
    with torch.no_grad():
        want, s, c = O.decoder_layer_forward(dw, x, rec_state=s0, mode="recurrent", bf16_acts=True)
    layer = Qwen35DecoderLayer(batch=B, mixer_weights=dw.gdn, mlp_weights=_mlp(dw))
    layer.set_state(rec_state=s0)
    got = torch.cat([layer(x[:, t:t + 1]) for t in range(2)], 1)
    assert device_error() == 0
    check("9B decoder decode B=64", got, want)
    check("9B decoder decode B=64 state", layer.get_recurrent_state(), s, max_rel=STATE_TOL)


def test_decoder_cuda_graph_decode_replay():
    dw = _decoder_weights(1024, 16, 16, 3072, seed=75)
    B = 4
    x = O.make_hidden(B, 3, 1024, seed=76)
    eager = Qwen35DecoderLayer(batch=B, mixer_weights=dw.gdn, mlp_weights=_mlp(dw))
    want = torch.cat([eager(x[:, t:t + 1]) for t in range(3)], 1)
    layer = Qwen35DecoderLayer(batch=B, mixer_weights=dw.gdn, mlp_weights=_mlp(dw), max_rows=B)
    xin = torch.zeros(B, 1, 1024, dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(xin)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        layer.forward_into(xin, out, stream=s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        layer.forward_into(xin, out, stream=s)
    layer.reset_state()
    outs = []
    for t in range(3):
        xin.copy_(x[:, t:t + 1].to("cuda", torch.bfloat16))
        g.replay()
        outs.append(out.float().cpu().clone())
    check("decoder graph replay", torch.cat(outs, 1), want, max_rel=1e-6, min_pcc=None, max_fro=None)


def test_decoder_rejects_tp_without_comm_and_aliasing():
    dw = _decoder_weights(1024, 16, 16, 3072, seed=77)
    with pytest.raises(ValueError):
        Qwen35DecoderLayer(batch=1, mixer_weights=dw.gdn, mlp_weights=_mlp(dw), tp_rank=0, tp_size=2)
    layer = Qwen35DecoderLayer(batch=1, mixer_weights=dw.gdn, mlp_weights=_mlp(dw))
    x = torch.zeros(1, 1, 1024, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(GDNError, match="alias"):
        layer.forward_into(x, x)
