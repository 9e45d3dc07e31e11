"""Failure detection without a GPU fault: every flag or barrier wait in the kernels is bounded (2 s) and
records an error code in the device error word instead of hanging or trapping.  Here the all-reduce's peer
wait is run on a flag that nothing sets (gdn_selftest_peer_wait): it must give up after its limit, the host
must read the peer-wait code, and the context must stay usable for a full layer call afterwards.  A flag that
is already set must pass without an error."""
import ctypes
import time

import pytest
import torch

from linear_attention_op_b200 import Qwen35GatedDeltaNet, device_error
from linear_attention_op_b200._lib import call
from oracle import gdn_oracle as O
from tests._util import check, requires_b200

pytestmark = [pytest.mark.gpu, requires_b200]

ERR_WAIT_PEER = 0x105


def _wait(flag: torch.Tensor, value: int):
    call("gdn_selftest_peer_wait", ctypes.c_void_p(flag.data_ptr()), value,
         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_peer_wait_on_set_flag_passes():
    flag = torch.full((1,), 5, dtype=torch.int64, device="cuda")
    _wait(flag, 5)
    assert device_error() == 0


def test_peer_wait_expires_records_status_and_context_survives():
    assert device_error() == 0
    flag = torch.zeros(1, dtype=torch.int64, device="cuda")  # no rank will ever set it
    t0 = time.perf_counter()
    _wait(flag, 1)
    code = device_error()  # synchronises: returns once the bounded wait has given up
    elapsed = time.perf_counter() - t0
    assert code == ERR_WAIT_PEER
    assert 1.5 < elapsed < 60, elapsed
    assert device_error() == 0  # reading the word cleared it
    # the context is intact: a layer call still runs and matches the oracle
    w = O.make_weights(1024, 16, 16, seed=70)
    x = O.make_hidden(2, 9, 1024, seed=71)
    want = O.layer_forward(w, x, mode="chunk")[0]
    check("layer after an expired wait", Qwen35GatedDeltaNet(weights=w, batch=2)(x), want)
    assert device_error() == 0
