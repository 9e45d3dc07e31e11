"""tcgen05 GEMM building block (gdn_gemm_bf16) against a PyTorch fp32 reference of the same product."""
import ctypes

import pytest
import torch

from linear_attention_op_b200 import _lib
from tests._util import requires_b200

pytestmark = [pytest.mark.gpu, requires_b200]


def run_gemm(a, b, out_kind, ksplit=0):
    m, k = a.shape
    n = b.shape[0]
    transposed = out_kind >= 2
    dt = torch.bfloat16 if out_kind in (1, 3) else torch.float32
    out = torch.full((n, m) if transposed else (m, n), float("nan"), dtype=dt, device="cuda")
    _lib.call("gdn_gemm_bf16", ctypes.c_void_p(a.data_ptr()), a.stride(0), ctypes.c_void_p(b.data_ptr()),
              b.stride(0), m, n, k, out_kind, ctypes.c_void_p(out.data_ptr()), out.stride(0), ksplit,
              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert _lib.device_error() == 0
    return out


@pytest.mark.parametrize("m, n, k", [(128, 64, 256), (256, 256, 512), (200, 300, 512), (65, 17, 64),
                                     (1000, 48, 1024), (384, 1, 128)])
@pytest.mark.parametrize("out_kind", [0, 1, 2, 3])
def test_gemm_matches_fp32(m, n, k, out_kind):
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n * 3 + k)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    b = torch.randn(n, k, device="cuda", generator=g).bfloat16()
    want = a.float() @ b.float().T
    got = run_gemm(a, b, out_kind).float()
    if out_kind >= 2:
        got = got.T
    tol = 1e-4 if out_kind in (0, 2) else 1e-2
    err = ((got - want).abs().max() / want.abs().max()).item()
    assert err < tol, err


@pytest.mark.parametrize("ksplit", [1, 2, 3, 5, 8])
def test_gemm_split_k_cluster(ksplit):
    """Decode-shaped (weights as the 128-row operand, 64 tokens) with K split across a cluster."""
    g = torch.Generator(device="cuda").manual_seed(ksplit)
    w = torch.randn(1000, 2048, device="cuda", generator=g).bfloat16()
    x = torch.randn(64, 2048, device="cuda", generator=g).bfloat16()
    want = (w.float() @ x.float().T).T
    got = run_gemm(w, x, 2, ksplit)
    err = ((got - want).abs().max() / want.abs().max()).item()
    assert err < 1e-4, err


@pytest.mark.parametrize("tokens", [128, 256])
@pytest.mark.parametrize("ksplit", [2, 3, 5])
def test_gemm_split_k_wide_tiles(tokens, ksplit):
    """128- and 256-token tiles split over 2, 3 and 5 CTAs: chunks owned round-robin, more than one per CTA;
    the result is the same for every split up to the reduction order."""
    g = torch.Generator(device="cuda").manual_seed(tokens + ksplit)
    w = torch.randn(384, 1536, device="cuda", generator=g).bfloat16()
    x = torch.randn(tokens, 1536, device="cuda", generator=g).bfloat16()
    want = (w.float() @ x.float().T).T
    got = run_gemm(w, x, 2, ksplit)
    err = ((got - want).abs().max() / want.abs().max()).item()
    assert err < 1e-4, err
    assert torch.equal(got, run_gemm(w, x, 2, ksplit)), "split-K result not reproducible"


def test_gemm_9b_decode_inproj_shape():
    g = torch.Generator(device="cuda").manual_seed(1)
    w = (torch.randn(12352, 4096, device="cuda", generator=g) * 0.02).bfloat16()
    x = torch.randn(64, 4096, device="cuda", generator=g).bfloat16()
    want = (w.float() @ x.float().T).T
    got = run_gemm(w, x, 2, 0)
    err = ((got - want).abs().max() / want.abs().max()).item()
    assert err < 1e-4, err


def test_gemm_strided_operands():
    g = torch.Generator(device="cuda").manual_seed(3)
    big = torch.randn(300, 640, device="cuda", generator=g).bfloat16()
    a = big[:, :512]  # row stride 640
    b = torch.randn(96, 512, device="cuda", generator=g).bfloat16()
    want = a.float() @ b.float().T
    got = run_gemm(a, b, 0)
    assert ((got - want).abs().max() / want.abs().max()).item() < 1e-4
