"""Shared helpers of the test suite (tolerances follow the benchmark spec and the reference's tests)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gdn_oracle as O

# bf16 outputs: max|d| / max|ref| <= 2e-2; fp32 final state: <= 1e-3 (benchmark spec).  The reference's own
# layer tests additionally require PCC > 0.9999 and rel-Frobenius < 1.5e-2 (9B/test_gdn_layer.py:35-39).
OUT_TOL = 2e-2
STATE_TOL = 1e-3


def cuda_ok() -> bool:
    return torch.cuda.is_available() and torch.cuda.get_device_capability(0)[0] >= 10


requires_b200 = pytest.mark.skipif(not cuda_ok(), reason="needs an sm_100 GPU")


def check(name, got, want, max_rel=OUT_TOL, min_pcc=0.9999, max_fro=1.5e-2):
    got, want = got.detach().float().cpu(), want.detach().float().cpu()
    assert got.shape == want.shape, f"{name}: shape {tuple(got.shape)} vs {tuple(want.shape)}"
    assert torch.isfinite(got).all(), f"{name}: non-finite values"
    mar, fro, p = O.max_abs_rel(got, want), O.rel_fro(got, want), O.pcc(got, want)
    print(f"{name}: max_abs_rel={mar:.2e} rel_fro={fro:.2e} pcc={p:.7f}")
    assert mar <= max_rel, f"{name}: max_abs_rel {mar:.3e} > {max_rel:.1e}"
    if min_pcc is not None:
        assert p > min_pcc, f"{name}: pcc {p:.6f}"
    if max_fro is not None:
        assert fro < max_fro, f"{name}: rel_fro {fro:.3e}"


def T(a):
    return torch.from_numpy(np.asarray(a))


def bf16(a):
    return torch.from_numpy(np.asarray(a)).view(torch.bfloat16).float()


def fixture_weights(z) -> O.GDNWeights:
    hidden, hk, hv, dk, dv, _ = (int(v) for v in z["dims"])
    return O.GDNWeights(
        w_qkv=bf16(z["w_qkv"]), w_z=bf16(z["w_z"]), w_a=bf16(z["w_a"]), w_b=bf16(z["w_b"]),
        conv_w=T(z["conv_w"]), a_log=T(z["a_log"]), dt_bias=T(z["dt_bias"]), norm_w=T(z["norm_w"]),
        w_out=bf16(z["w_out"]), num_k_heads=hk, num_v_heads=hv, head_k_dim=dk, head_v_dim=dv,
    )
