"""Head-parallel partition checked on CPU ranks (gloo, world size 2 and 4): every rank runs the oracle on its
shard of the weights, one all-reduce of the partial outputs reproduces the full layer, and the per-rank
states tile the full state.  This is the partition libgdn_b200.so applies in gdn_layer_create."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from linear_attention_op_b200.tp import shard_plan, shard_weights
from oracle import gdn_oracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        torch.set_num_threads(1)
        w = O.make_weights(256, 4, 8, seed=0)
        x = O.make_hidden(2, 37, 256, seed=1)
        s0 = torch.randn(2, 8, 128, 128, generator=torch.Generator().manual_seed(2)) * 0.1
        p = shard_plan(4, 8, rank, world)
        v0, v1 = p.v_heads
        ws = shard_weights(w, rank, world)
        part, s, c = O.layer_forward(ws, x, rec_state=s0[:, v0:v1].clone(), mode="chunk")
        dist.all_reduce(part)
        full, s_full, c_full = O.layer_forward(w, x, rec_state=s0, mode="chunk")
        states = [torch.empty_like(s) for _ in range(world)]
        dist.all_gather(states, s)
        q.put((rank, O.max_abs_rel(part, full), O.max_abs_rel(torch.cat(states, 1), s_full)))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), None))


@pytest.mark.parametrize("world", [2, 4])
def test_head_parallel_partition_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, out_err, state_err in results:
        assert state_err is not None, f"rank {rank} failed: {out_err}"
        assert out_err < 1e-5, (rank, out_err)
        assert state_err < 1e-6, (rank, state_err)


def test_shard_plan_rules():
    p = shard_plan(16, 32, 3, 8)
    assert p.k_heads == (6, 8) and p.v_heads == (12, 16)
    with pytest.raises(ValueError):
        shard_plan(16, 32, 0, 3)
    with pytest.raises(ValueError):
        shard_plan(16, 32, 8, 8)


def test_gqa_groups_stay_on_one_rank():
    for world in (1, 2, 4, 8):
        for r in range(world):
            p = shard_plan(16, 32, r, world)
            for h in range(*p.v_heads):
                assert p.k_heads[0] <= h // 2 < p.k_heads[1]
