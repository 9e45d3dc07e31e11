"""The oracle's e4m3 quantiser (the library's fp8 mode) on the CPU: power-of-two scales that keep every
row within e4m3's +-448, dequantised values exact in bf16 (so the prefill GEMMs can use them), rounding
error within half an e4m3 step, and the fp8 layer within a few percent of the bf16 one."""
import math

import torch

from oracle import gdn_oracle as O


def test_scales_are_tight_powers_of_two():
    g = torch.Generator().manual_seed(0)
    amax = torch.rand(4000, generator=g) * torch.exp2(torch.randint(-40, 20, (4000,), generator=g).float())
    amax[:3] = torch.tensor([0.0, 448.0, 56.0])
    s = O.e4m3_scale(amax)
    for a, sc in zip(amax.tolist(), s.tolist()):
        if a == 0:
            assert sc == 1.0
            continue
        m, _ = math.frexp(sc)
        assert m == 0.5, sc  # a power of two
        v = torch.tensor(a, dtype=torch.float32) / 448.0
        assert v.item() <= sc and (v.item() > sc / 2 or sc == 2.0**-126)


def test_row_quantisation_bounds():
    w = O.make_weights(1024, 16, 16, seed=3)
    for t in (w.w_qkv, w.w_out, O.make_hidden(2, 7, 1024, seed=4)[0]):
        q = O.quantize_rows_e4m3(t)
        assert torch.equal(q, O.bf16_round(q)), "dequantised values must be exact in bf16"
        s = O.e4m3_scale(t.abs().amax(-1))[..., None]
        assert (q.abs() / s <= 448).all()
        # round to nearest: |q - t| <= half an e4m3 step at |t| (3 mantissa bits; subnormal step 2^-9 s)
        step = torch.maximum(torch.exp2(torch.floor(torch.log2((t.abs() / s).clamp_min(2.0**-6))) - 3),
                             torch.full_like(t, 2.0**-9)) * s
        assert ((q - t).abs() <= step / 2 + 1e-12).all()


def test_fp8_layer_close_to_bf16_layer():
    w = O.make_weights(1024, 16, 16, seed=5)
    x = O.make_hidden(2, 6, 1024, seed=6)
    y_bf16 = O.layer_forward(w, x, mode="recurrent")[0]
    y_fp8 = O.layer_forward(O.fp8_weights(w), x, mode="recurrent", act_fp8=True)[0]
    # e4m3 keeps 3 mantissa bits: on random weights and activations both projections lose ~5% each
    assert O.rel_fro(y_fp8, y_bf16) < 0.12
