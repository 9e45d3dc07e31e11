"""The work partition of the NVLink all-reduce (csrc/allreduce.cu), restated on the CPU and checked for
every rank count the library supports: in the reduce-scatter, rank r's CTA c sums the vectors
lo_r + c*256 + t + j*stride of slice r; in the all-gather, CTA c of every rank copies from each peer p the
vectors per*p + c*256 + t + j*stride.  Because CTA c of rank q waits only for the "reduced" flag of CTA c
of each peer, the vectors it copies must be exactly the ones that peer's CTA c reduced, and together the
two phases must fill every output vector exactly once.  The constants are read from the kernel header, so
the restatement tracks the code."""
import re
from pathlib import Path

import numpy as np
import pytest

HDR = (Path(__file__).resolve().parents[1] / "linear_attention_op_b200" / "csrc" / "kernels.cuh").read_text()
MAX_RANKS = int(re.search(r"kP2PMaxRanks = (\d+)", HDR).group(1))
MAX_CTAS = int(re.search(r"kP2PMaxCtas = (\d+)", HDR).group(1))
RED_OFF = int(re.search(r"kP2PReducedOff = (\d+)", HDR).group(1))
THREADS = 256  # allreduce_p2p_kernel's block size


def grid_of(nv, sms):
    return min(min(sms, MAX_CTAS), (nv + THREADS - 1) // THREADS)


def owner_cta(k, grid):
    """CTA that handles local offset k (k = c*256 + t + j*stride)."""
    return (k % (grid * THREADS)) // THREADS


@pytest.mark.parametrize("world", list(range(3, MAX_RANKS + 1)))
@pytest.mark.parametrize("n", [8 * 7, 4096 * 64, 4096 * 64 * 3 + 8 * 5, 4096 * 512, 8 << 20 >> 1])
@pytest.mark.parametrize("sms", [148, 132])
def test_two_shot_partition(world, n, sms):
    nv = n // 8
    grid = grid_of(nv, sms)
    per = (nv + world - 1) // world
    covered = np.zeros(nv, np.int64)
    for r in range(world):
        lo, hi = per * r, min(nv, per * r + per)
        # reduce-scatter: local offsets k = i - lo handled by CTA owner_cta(k)
        k = np.arange(hi - lo)
        rs_cta = owner_cta(k, grid)
        covered[lo:hi] += 1
        # all-gather on any other rank q: offset k of slice r is copied by CTA owner_cta(k) of rank q,
        # which waits on the flag of CTA owner_cta(k) of rank r: the same CTA index
        ag_k = np.arange(per)
        ag_k = ag_k[per * r + ag_k < nv]
        assert np.array_equal(owner_cta(ag_k, grid), rs_cta), "AG CTA must wait on the CTA that reduced it"
    assert (covered == 1).all(), "every vector reduced by exactly one rank"
    # flag page: reduced[rank][cta] lives below the first slot
    assert grid <= MAX_CTAS


def test_flag_page_fits_before_slot():
    api = (Path(__file__).resolve().parents[1] / "linear_attention_op_b200" / "csrc" / "gdn_api.cu").read_text()
    slot_off = int(re.search(r"kP2PSlotOffset = (\d+)", api).group(1))
    # arrive[8] at [0], epoch and cta_done at [16], [17], reduced at [RED_OFF ...)
    assert 2 * MAX_RANKS + 2 <= RED_OFF
    assert (RED_OFF + MAX_RANKS * MAX_CTAS) * 8 <= slot_off
