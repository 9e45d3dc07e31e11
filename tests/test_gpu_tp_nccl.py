"""Head-parallel layer over 2, 4 or 8 GPUs with the library's communicator (NVLink all-reduce for small
outputs, NCCL above 8 MiB): every rank gets the full, all-reduced output, and the ranks' states tile the
single-GPU state -- for bf16 weights, for weight-only fp8 (whole-row out_proj scales) and for the decoder
layer around the mixer (two all-reduces per call).  Skipped with fewer GPUs."""
import os
import socket

import pytest
import torch

from tests._util import requires_b200

pytestmark = [pytest.mark.gpu, requires_b200]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        import datetime

        import torch.distributed as dist

        from linear_attention_op_b200 import Qwen35GatedDeltaNet, device_error
        from linear_attention_op_b200.tp import Communicator
        from oracle import gdn_oracle as O

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
        comm = Communicator.from_process_group()
        w = O.make_weights(1024, 16, 32, seed=7)
        x = O.make_hidden(2, 70, 1024, seed=7)
        want, s_want, c_want = O.layer_forward(w, x, mode="chunk")
        xd = O.make_hidden(2, 1, 1024, seed=8)
        want_d, s_want_d, _ = O.layer_forward(w, xd, s_want, c_want, mode="recurrent")
        layer = Qwen35GatedDeltaNet(weights=w, batch=2, tp_rank=rank, tp_size=world, comm=comm)
        y = layer(x)
        s_loc = layer.get_recurrent_state()
        yd = layer(xd)
        s_loc_d = layer.get_recurrent_state()
        # several decode calls in a row: the NVLink all-reduce's slots, epoch and push counters cycle
        xs = O.make_hidden(2, 5, 1024, seed=10)
        want_s, s_want_s, _ = O.layer_forward(w, xs, s_want_d, O.layer_forward(w, xd, s_want, c_want,
                                                                              mode="recurrent")[2], mode="recurrent")
        ys = torch.cat([layer(xs[:, t:t + 1]) for t in range(5)], 1)
        s_loc_s = layer.get_recurrent_state()
        # the pipelined host path with the ranks sharing the host copies (split_io): rank r's sequences of
        # the result equal forward_into's (8 sequences, so every group size divides the batch)
        x8 = O.make_hidden(8, 2, 1024, seed=11).to(torch.bfloat16)
        la = Qwen35GatedDeltaNet(weights=w, batch=8, tp_rank=rank, tp_size=world, comm=comm)
        lb = Qwen35GatedDeltaNet(weights=w, batch=8, tp_rank=rank, tp_size=world, comm=comm)
        rows = slice(rank * (8 // world), (rank + 1) * (8 // world))
        split_same = True
        for t in range(2):
            xt = x8[:, t:t + 1].contiguous()
            ya = la.forward_into(xt.cuda(), torch.empty(8, 1, 1024, dtype=torch.bfloat16, device="cuda")).cpu()
            yb = torch.zeros(8, 1, 1024, dtype=torch.bfloat16).pin_memory()
            lb.forward_host_async(xt.pin_memory(), yb, split_io=True).synchronize()
            split_same = split_same and bool(torch.equal(yb[rows], ya[rows]))
        # an output above the NVLink all-reduce's 8 MiB slot (4104 x 1024 bf16) takes the NCCL path
        xl = O.make_hidden(1, 4104, 1024, seed=9)
        yl = Qwen35GatedDeltaNet(weights=w, batch=1, tp_rank=rank, tp_size=world, comm=comm)(xl)
        # weight-only fp8: every shard quantises out_proj with the whole rows' scales, so the all-reduced
        # decode output matches the single-GPU quantised layer
        wq = O.fp8_weights(w)
        want_q, _, _ = O.layer_forward(wq, xd, s_want, c_want, mode="recurrent")
        lq = Qwen35GatedDeltaNet(weights=w, batch=2, tp_rank=rank, tp_size=world, comm=comm, weight_dtype="fp8")
        hvl = 32 // world
        lq.set_state(rec_state=s_want[:, rank * hvl:(rank + 1) * hvl])
        conv_idx = torch.cat([torch.arange(rank * 128 * (16 // world), (rank + 1) * 128 * (16 // world)),
                              2048 + torch.arange(rank * 128 * (16 // world), (rank + 1) * 128 * (16 // world)),
                              4096 + torch.arange(rank * 128 * hvl, (rank + 1) * 128 * hvl)])
        lq.set_state(conv_state=c_want[:, :, conv_idx])
        yq = lq(xd)
        # the decoder layer around the mixer: two all-reduces per call (mixer output, MLP output)
        from linear_attention_op_b200 import DecoderMlpWeights, Qwen35DecoderLayer
        gen = torch.Generator().manual_seed(90)
        rn = lambda *sz: O.bf16_round(torch.randn(*sz, generator=gen) * 0.02)
        dw = O.DecoderWeights(gdn=w, input_norm_w=torch.rand(1024, generator=gen) - 0.5,
                              post_norm_w=torch.rand(1024, generator=gen) - 0.5, w_gate=rn(2048, 1024),
                              w_up=rn(2048, 1024), w_down=rn(1024, 2048))
        want_dp, sd, cd = O.decoder_layer_forward(dw, x, mode="chunk", bf16_acts=True)
        want_dd, sd, cd = O.decoder_layer_forward(dw, xd, sd, cd, mode="recurrent", bf16_acts=True)
        dec = Qwen35DecoderLayer(batch=2, mixer_weights=w, comm=comm, tp_rank=rank, tp_size=world,
                                 mlp_weights=DecoderMlpWeights(dw.input_norm_w, dw.post_norm_w, dw.w_gate, dw.w_up,
                                                               dw.w_down))
        ydp = dec(x)
        ydd = dec(xd)
        err = device_error()
        hv = 32 // world
        res = dict(
            out=O.max_abs_rel(y.float(), want), state=O.max_abs_rel(s_loc, s_want[:, rank * hv:(rank + 1) * hv]),
            out_dec=O.max_abs_rel(yd.float(), want_d),
            state_dec=O.max_abs_rel(s_loc_d, s_want_d[:, rank * hv:(rank + 1) * hv]), err=err,
            out_fp8=O.max_abs_rel(yq.float(), want_q), dec_pre=O.max_abs_rel(ydp.float(), want_dp),
            dec_dec=O.max_abs_rel(ydd.float(), want_dd),
            dec_state=O.max_abs_rel(dec.get_recurrent_state(), sd[:, rank * hv:(rank + 1) * hv]),
            out_steps=O.max_abs_rel(ys.float(), want_s), split_io_same=split_same,
            state_steps=O.max_abs_rel(s_loc_s, s_want_s[:, rank * hv:(rank + 1) * hv]))
        if rank == 0:
            res["out_large"] = O.max_abs_rel(yl.float(), O.layer_forward(w, xl, mode="chunk")[0])
        comm.close()
        dist.destroy_process_group()
        q.put((rank, res))
    except Exception as e:  # report instead of hanging the parent
        import traceback

        q.put((rank, {"exc": traceback.format_exc()}))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_layer_nccl(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    for rank in range(world):
        r = results[rank]
        assert "exc" not in r, r.get("exc")
        print(rank, r)
        assert r["err"] == 0
        assert r["out"] <= 2e-2 and r["out_dec"] <= 2e-2 and r["out_steps"] <= 2e-2, r
        assert r["state_steps"] <= 1e-3, r
        assert r["split_io_same"], r
        assert r["state"] <= 1e-3 and r["state_dec"] <= 1e-3, r
        assert r["out_fp8"] <= 2e-2, r
        assert r["dec_pre"] <= 2e-2 and r["dec_dec"] <= 2e-2 and r["dec_state"] <= 1e-3, r
        if rank == 0:
            assert r["out_large"] <= 2e-2, r
