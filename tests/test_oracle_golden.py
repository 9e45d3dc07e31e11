"""The CPU oracle against the golden fixtures made from the reference's own code (CPU only)."""
import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O


def T(a):
    return torch.from_numpy(np.asarray(a))


def bf16(a):
    return torch.from_numpy(np.asarray(a)).view(torch.bfloat16).float()


@pytest.mark.parametrize("case", ["a", "b"])
def test_recurrence_matches_reference_py(golden_dir, case):
    z = np.load(golden_dir / "recurrence_ref.npz")
    get = lambda k: T(z[f"{case}_{k}"])
    init = get("init")
    init = None if init.numel() == 0 else init
    o, s = O.recurrent_gated_delta_rule(get("q"), get("k"), get("v"), get("g"), get("beta"), initial_state=init)
    assert O.max_abs_rel(o, get("o")) < 1e-5
    assert O.max_abs_rel(s, get("state")) < 1e-5


@pytest.mark.parametrize("case", ["a", "b"])
def test_chunked_form_matches_reference_recurrence(golden_dir, case):
    z = np.load(golden_dir / "recurrence_ref.npz")
    get = lambda k: T(z[f"{case}_{k}"])
    init = get("init")
    init = None if init.numel() == 0 else init
    o, s = O.chunk_gated_delta_rule(get("q"), get("k"), get("v"), get("g"), get("beta"), initial_state=init, chunk=16)
    assert O.max_abs_rel(o, get("o")) < 1e-4
    assert O.max_abs_rel(s, get("state")) < 1e-4


def test_chunk_matches_hf_chunk(golden_dir):
    z = np.load(golden_dir / "chunk_hf.npz")
    o, s = O.chunk_gated_delta_rule(T(z["q"]), T(z["k"]), T(z["v"]), T(z["g"]), T(z["beta"]), chunk=64)
    assert O.max_abs_rel(o, T(z["o"])) < 1e-5
    assert O.max_abs_rel(s, T(z["state"])) < 1e-5


def layer_weights(z):
    hidden, hk, hv, dk, dv, _ = (int(v) for v in z["dims"])
    return O.GDNWeights(
        w_qkv=bf16(z["w_qkv"]), w_z=bf16(z["w_z"]), w_a=bf16(z["w_a"]), w_b=bf16(z["w_b"]),
        conv_w=T(z["conv_w"]), a_log=T(z["a_log"]), dt_bias=T(z["dt_bias"]), norm_w=T(z["norm_w"]),
        w_out=bf16(z["w_out"]), num_k_heads=hk, num_v_heads=hv, head_k_dim=dk, head_v_dim=dv,
    )


@pytest.mark.parametrize("mode", ["recurrent", "chunk"])
def test_layer_prefill_then_decode_matches_hf(golden_dir, mode):
    z = np.load(golden_dir / "layer_hf.npz")
    w = layer_weights(z)
    x = T(z["x"])
    t0 = int(z["t0"][0])
    y, s, c = O.layer_forward(w, x[:, :t0], mode=mode)
    assert O.max_abs_rel(y, T(z["y_pre"])) < 1e-4
    assert O.max_abs_rel(s, T(z["rec_pre"])) < 1e-4
    assert O.max_abs_rel(c, O.hf_conv_state_to_abi(T(z["conv_pre"]))) < 1e-6
    ys = []
    for t in range(t0, x.shape[1]):
        yt, s, c = O.layer_forward(w, x[:, t:t + 1], s, c, mode=mode)
        ys.append(yt)
    assert O.max_abs_rel(torch.cat(ys, 1), T(z["y_dec"])) < 1e-4
    assert O.max_abs_rel(s, T(z["rec_dec"])) < 1e-4
    assert O.max_abs_rel(c, O.hf_conv_state_to_abi(T(z["conv_dec"]))) < 1e-6


def test_layer_one_shot_and_single_token_match_hf(golden_dir):
    z = np.load(golden_dir / "layer_hf.npz")
    w = layer_weights(z)
    y, _, _ = O.layer_forward(w, T(z["x"]), mode="chunk")
    assert O.max_abs_rel(y, T(z["y_full"])) < 1e-4
    y1, _, _ = O.layer_forward(w, T(z["x1"]))
    assert O.max_abs_rel(y1, T(z["y_one"])) < 1e-4


def test_conv_state_roundtrip():
    s = torch.randn(2, 3, 10)
    assert torch.equal(O.hf_conv_state_to_abi(O.abi_conv_state_to_hf(s)), s)


def test_short_call_keeps_older_conv_history():
    w = torch.randn(6, 4)
    x = torch.randn(1, 5, 6)
    _, s_all = O.causal_conv1d(x, w, None)
    _, s1 = O.causal_conv1d(x[:, :4], w, None)
    _, s2 = O.causal_conv1d(x[:, 4:5], w, s1)
    assert torch.allclose(s_all, s2)


@pytest.mark.parametrize("mode", ["recurrent", "chunk"])
def test_decoder_layer_prefill_then_decode_matches_hf(golden_dir, mode):
    """The decoder layer around the mixer (input RMSNorm, residual, SwiGLU MLP) against HF's
    Qwen3_5DecoderLayer of the linear-attention type, prefill then cached decode."""
    z = np.load(golden_dir / "decoder_hf.npz")
    dw = O.DecoderWeights(gdn=layer_weights(z), input_norm_w=T(z["input_norm_w"]), post_norm_w=T(z["post_norm_w"]),
                          w_gate=bf16(z["w_gate"]), w_up=bf16(z["w_up"]), w_down=bf16(z["w_down"]))
    x = T(z["x"])
    t0 = int(z["t0"][0])
    y, s, c = O.decoder_layer_forward(dw, x[:, :t0], mode=mode)
    assert O.max_abs_rel(y, T(z["y_pre"])) < 1e-4
    ys = []
    for t in range(t0, x.shape[1]):
        yt, s, c = O.decoder_layer_forward(dw, x[:, t:t + 1], s, c, mode=mode)
        ys.append(yt)
    assert O.max_abs_rel(torch.cat(ys, 1), T(z["y_dec"])) < 1e-4
    assert O.max_abs_rel(s, T(z["rec_dec"])) < 1e-4
    assert O.max_abs_rel(c, O.hf_conv_state_to_abi(T(z["conv_dec"]))) < 1e-6
