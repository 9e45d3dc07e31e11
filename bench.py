"""Benchmark of the Qwen3.5 Gated DeltaNet layer on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-prefill]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 --master-port P bench.py --gpus N

Headline (``value``): config 2 of the benchmark spec -- a Qwen3.5-9B-shaped GDN layer (hidden 4096, 16 QK heads,
32 V heads, dk = dv = 128, conv 4), batch-64 decode, fp32 state ~ N(0, 0.1), as tokens/s of the whole job,
16 consecutive decode steps per CUDA-graph replay (a model's graph holds many layers per token; the host's
graph launches then do not pace the GPU).  Heads are sharded over N GPUs (one all-reduce per step) and the
batch grows with N (64 sequences per GPU, 64 N in all), so every GPU streams the same 268 MB of recurrent
state per step as one GPU does at batch 64: weak scaling.  The same line carries config 3 (batch 8 x 8192-token
chunked prefill, fixed size: strong scaling) under ``prefill``, the
per-stage timing, the roofline of the dominant kernel, the end-to-end number through the public API with
host buffers, and the CPU baseline (the oracle port on the host cores, rank 0 at N = 1 only).

``--impl reference`` times the reference's CPU path (the oracle restatement of HF Qwen3_5GatedDeltaNet /
reference.py; the reference's own device code is Tenstorrent-only) on the host cores for the same config.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "GDN layer tokens/s (decode & 8K prefill), % HBM/tensor roofline, 1-8 B200"
H, HK, HV, D = 4096, 16, 32, 128          # Qwen3.5-9B GDN geometry
DECODE_B = 64                              # config 2 (override: --decode-b, for profiling smaller cases)
PREFILL_B, PREFILL_T = 8, 8192             # config 3 (override: --prefill-b / --prefill-t)
STAGES = ["in_proj", "conv", "chunk_prep", "recurrence", "out_proj", "allreduce"]
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return dict(FALLBACK_PEAKS, source="fallback")


def ncu_traffic(key: str, geometry: str):
    """Per-launch DRAM bytes of one kernel from the committed ncu summary (profiles/ncu_traffic.json), or None
    when that capture was made on another geometry (shard or batch) than the one being reported."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    return d.get(key) if d.get("_geometry", {}).get(key.split("_")[0]) == geometry else None


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def workload_config(world: int) -> dict:
    """The benchmark configuration, the same dict in both arms (ours and --impl reference)."""
    B = DECODE_B * world
    return {"workload": f"cfg2: Qwen3.5-9B GDN layer decode, batch {DECODE_B} per GPU (global {B}), "
                        "fp32 state ~N(0,0.1)",
            "model": "Qwen3.5-9B GDN layer (random init)", "global_batch": B, "seq_len": 1,
            "parallelism": f"tp{world} head-parallel" if world > 1 else "tp1",
            "l2": "inputs larger than L2: 417 MB of weights + state per GPU per step > 126 MB"}


# ---------------------------------------------------------------------------------------------------
# Synthetic layer (the benchmark spec's distributions), generated on the GPU
# ---------------------------------------------------------------------------------------------------
def synthetic_weights(seed: int, device, a_max: float = 16.0):
    from linear_attention_op_b200 import LayerWeights

    g = torch.Generator(device=device).manual_seed(seed)
    kd, vd = HK * D, HV * D
    conv_dim = 2 * kd + vd
    rn = lambda *s: (torch.randn(*s, generator=g, device=device) * 0.02).to(torch.bfloat16)
    return LayerWeights(
        w_qkv=rn(conv_dim, H), w_z=rn(vd, H), w_a=rn(HV, H), w_b=rn(HV, H),
        conv_w=((torch.rand(conv_dim, 4, generator=g, device=device) * 2 - 1) * 0.5).bfloat16().float(),
        a_log=torch.log(1 + torch.rand(HV, generator=g, device=device) * (a_max - 1)),
        dt_bias=torch.randn(HV, generator=g, device=device) * 0.1,
        norm_w=0.5 + torch.rand(D, generator=g, device=device),
        w_out=rn(H, vd), num_k_heads=HK, num_v_heads=HV)


def decode_bytes(B: int, world: int = 1, wbytes: int = 2) -> dict:
    """Algorithmic HBM bytes of one decode step (the per-unit figures of the design notes), per GPU;
    wbytes = bytes per weight (2 bf16, 1 with fp8 weights)."""
    hv, kd, vd = HV // world, HK * D // world, HV * D // world
    conv_dim = 2 * kd + vd
    rows = conv_dim + vd + 2 * hv
    w_in, w_out = rows * H * wbytes, H * vd * wbytes
    state = 2 * B * hv * D * D * 4
    conv = 2 * B * conv_dim * 3 * 4
    act = 2 * B * H * 2
    proj = B * rows * 4
    return {
        # in_proj writes the raw fp32 projections; the conv (history read, state roll) runs in the step kernel
        "in_proj": w_in + B * H * 2 + proj,
        "recurrence": state + conv + proj + B * vd * 2,
        "out_proj": w_out + B * vd * 2 + B * H * 2,
        "step": w_in + w_out + state + conv + act,
    }


def prefill_flops(B: int, T: int, world: int = 1) -> dict:
    n = B * T
    hv, kd, vd = HV // world, HK * D // world, HV * D // world
    rows = 2 * kd + 2 * vd + 2 * hv
    rec = 182955 * n * hv  # per token per head at C = 64, dk = dv = 128
    return {"in_proj": 2 * n * H * rows, "recurrence": rec, "out_proj": 2 * n * vd * H,
            "step": 2 * n * H * rows + 2 * n * vd * H + rec}


# ---------------------------------------------------------------------------------------------------
# Clocks sampled during the timed region
# ---------------------------------------------------------------------------------------------------
class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled through NVML in a background thread while the
    timed region runs (the fields of nvidia-smi's clocks line; read-only queries).  One sampler for the
    whole job -- rank 0, its own GPU: external nvidia-smi processes polling several GPUs contend for driver
    locks and stall the ranks' kernel launches.  indices None: no sampling."""

    def __init__(self, indices, period_s: float | None = 0.05):
        # period None: only the samples taken as the region starts and ends (used with several ranks, whose
        # all-reduces make every rank wait out any stall an in-region query causes on one of them).  NVML is
        # initialised here, before the caller's barrier: nvmlInit takes long enough that doing it as the
        # region starts would delay rank 0 behind the others.
        self.indices = indices
        self.period = period_s
        self.rows = []
        self.thread = None
        self.handles = None
        if indices is not None:
            try:
                import pynvml as nv

                nv.nvmlInit()
                self.nv = nv
                self.handles = [nv.nvmlDeviceGetHandleByIndex(i) for i in indices]
            except Exception:
                self.handles = None

    def _sample(self, nv):
        for h in self.handles:
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.rows.append((sm, mx, rs))
            except Exception:
                pass

    def __enter__(self):
        if not self.handles:
            return self
        try:
            import threading

            nv = self.nv
            self._sample(nv)
            self.stop = threading.Event()

            def loop():
                while self.period is not None and not self.stop.wait(self.period):
                    self._sample(nv)

            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
        except Exception:
            self.thread = None
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)
            self._sample(self.nv)

    def summary(self):
        if self.thread is None or not self.rows:
            return None
        nv = self.nv
        bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
        reasons = sorted({name for _, _, rs in self.rows for name, bit in bits.items() if rs & bit})
        return {"sm_mhz": statistics.median(r[0] for r in self.rows), "sm_max_mhz": max(r[1] for r in self.rows),
                "reasons": reasons, "samples": len(self.rows), "source": "NVML (nvidia-smi's clocks fields)",
                "mode": "every 50 ms" if self.period else "region start and end (several ranks)"}


# ---------------------------------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------------------------------
def setup_dist(n: int):
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=datetime.timedelta(seconds=300))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def stage_times(layer, run_step, steps: int) -> list[float]:
    """Average ms per stage over `steps` eager calls, with the library's stage events."""
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(7)] for _ in range(2)]
    tot = [0.0] * 6
    for i in range(steps):
        e = evs[i % 2]
        layer.set_stage_events(e)
        run_step()
        torch.cuda.synchronize()
        for j in range(6):
            tot[j] += e[j].elapsed_time(e[j + 1])
    layer.set_stage_events(None)
    return [t / steps for t in tot]


def max_abs_rel(got: torch.Tensor, want: torch.Tensor) -> float:
    """max|got - want| / max|want| (the benchmark spec's tolerance metric)."""
    got, want = got.double(), want.double()
    return float((got - want).abs().max() / want.abs().max().clamp_min(1e-30))


def tp_parity(layer, W, rank: int, world: int, dev, weight_dtype: str = "bf16") -> dict:
    """Multi-GPU correctness, checked before the timed region: the head-parallel layer (this rank's shard and
    the library communicator) against a single-GPU layer (tp_size 1, the path the GPU test suite pins to the
    CPU oracle) built from the same weights on this rank's GPU, on the same inputs.
    * decode: one step at the benchmark's global batch from a random N(0, 0.1) state -- the NVLink
      all-reduce at the timed message size;
    * prefill: 2 sequences x 130 tokens from zero state -- the NCCL all-reduce, ragged last chunk.
    Every rank compares its all-reduced output and its state shards; the worst error over the ranks is
    reported, plus whether every rank received bit-identical outputs."""
    import torch.distributed as dist

    from linear_attention_op_b200 import Qwen35GatedDeltaNet

    hv, kd, vd = HV // world, HK * D // world, HV * D // world
    k0, v0 = rank * kd, rank * vd
    conv_idx = torch.cat([torch.arange(k0, k0 + kd), HK * D + torch.arange(k0, k0 + kd),
                          2 * HK * D + torch.arange(v0, v0 + vd)]).to(dev)
    B = layer.batch
    ref = Qwen35GatedDeltaNet(weights=W, batch=B, device=dev, weight_dtype=weight_dtype)
    g = torch.Generator(device=dev).manual_seed(77)  # identical on every rank
    s0 = torch.randn(B, HV, D, D, generator=g, device=dev) * 0.1
    c0 = torch.randn(B, 3, 2 * HK * D + HV * D, generator=g, device=dev)
    x = torch.randn(B, 1, H, generator=g, device=dev).to(torch.bfloat16)
    xp = torch.randn(2, 130, H, generator=g, device=dev).to(torch.bfloat16)
    res = {}
    tp = layer.with_batch(B)
    tp.set_state(rec_state=s0[:, rank * hv:(rank + 1) * hv], conv_state=c0[:, :, conv_idx])
    ref.set_state(rec_state=s0, conv_state=c0)
    out_tp = tp.forward_into(x, torch.empty_like(x))
    out_ref = ref.forward_into(x, torch.empty_like(x))
    torch.cuda.synchronize()
    res["decode_out"] = max_abs_rel(out_tp.float(), out_ref.float())
    res["decode_state"] = max_abs_rel(tp.rec_state, ref.rec_state[:, rank * hv:(rank + 1) * hv])
    res["decode_conv_state"] = max_abs_rel(tp.conv_state, ref.conv_state[:, :, conv_idx])
    sums = [out_tp.float().sum().double()]
    del tp, s0
    tp2, ref2 = layer.with_batch(2), ref.with_batch(2)
    outp_tp = tp2.forward_into(xp, torch.empty_like(xp))
    outp_ref = ref2.forward_into(xp, torch.empty_like(xp))
    torch.cuda.synchronize()
    res["prefill_out"] = max_abs_rel(outp_tp.float(), outp_ref.float())
    res["prefill_state"] = max_abs_rel(tp2.rec_state, ref2.rec_state[:, rank * hv:(rank + 1) * hv])
    res["prefill_conv_state"] = max_abs_rel(tp2.conv_state, ref2.conv_state[:, :, conv_idx])
    sums.append(outp_tp.float().sum().double())
    del tp2, ref2, ref
    t = torch.tensor([res[k] for k in sorted(res)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    res = {k: float(v) for k, v in zip(sorted(res), t.tolist())}
    cs = torch.stack(sums).to(dev)
    allcs = [torch.empty_like(cs) for _ in range(world)]
    dist.all_gather(allcs, cs)
    res["ranks_identical"] = all(torch.equal(allcs[0], c) for c in allcs)
    res["tolerance"] = {"out": 2e-2, "state": 1e-3, "conv_state": 1e-4}
    res["ok"] = bool(res["ranks_identical"] and res["decode_out"] <= 2e-2 and res["prefill_out"] <= 2e-2
                     and res["decode_state"] <= 1e-3 and res["prefill_state"] <= 1e-3
                     and res["decode_conv_state"] <= 1e-4 and res["prefill_conv_state"] <= 1e-4)
    res["against"] = "single-GPU layer (tp1) with the same weights and inputs on each rank's GPU"
    return res


def graph_steps_for(steps: int, want: int) -> int:
    """The largest divisor of `steps` not above `want`: every replay holds the same number of steps and the
    timed region holds exactly `steps` of them."""
    return max(d for d in range(1, max(1, min(want, steps)) + 1) if steps % d == 0)


def run_ours(args):
    from linear_attention_op_b200 import Qwen35GatedDeltaNet, device_error, launch_count
    from linear_attention_op_b200.tp import Communicator

    rank, world, local = setup_dist(args.gpus)
    dev = torch.device("cuda", local)
    pk = peaks()
    comm = Communicator.from_process_group() if world > 1 else None
    W = synthetic_weights(0, dev)
    B = DECODE_B * world  # 64 sequences per GPU: each GPU holds all of them for its 1/N of the heads
    layer = Qwen35GatedDeltaNet(weights=W, batch=B, device=dev, tp_rank=rank, tp_size=world, comm=comm,
                                max_rows=max(B, PREFILL_B * PREFILL_T if args.prefill else B),
                                weight_dtype=args.weights)
    if args.only == "prefill":  # profiling case: the prefill workload alone
        res = run_prefill(args, layer, dev, world, pk)
        if rank == 0:
            print(json.dumps({"metric": METRIC, "only": "prefill", "prefill": res}), flush=True)
        if comm is not None:
            comm.close()
        return
    parity = tp_parity(layer, W, rank, world, dev, args.weights) if world > 1 else None
    g = torch.Generator(device=dev).manual_seed(1000 + rank)  # this rank's heads of the N(0, 0.1) state
    layer.set_state(rec_state=torch.randn(B, HV // world, D, D, generator=g, device=dev) * 0.1)
    gx = torch.Generator(device=dev).manual_seed(1)  # the replicated input, identical on every rank
    x = torch.randn(B, 1, H, generator=gx, device=dev).to(torch.bfloat16)
    out = torch.empty_like(x)
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream())

    # eager warm-up, launch count per step
    n0 = launch_count()
    with torch.cuda.stream(stream):
        layer.forward_into(x, out, stream=stream)
    torch.cuda.synchronize()
    launches_per_step = launch_count() - n0
    if device_error() != 0:
        raise SystemExit("device error during warm-up")

    # G consecutive decode steps per graph (as a model's graph holds many layers per token), so that the
    # host's graph launches do not pace the GPU; K timed steps = K / G replays.
    gsteps = graph_steps_for(args.steps, args.graph_steps)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(gsteps):
            layer.forward_into(x, out, stream=stream)
    for _ in range(max(1, -(-args.warmup // gsteps))):
        graph.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler([local] if rank == 0 else None, 0.05 if world == 1 else None)
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with sampler as clk:
        torch.cuda.synchronize()
        if world > 1:
            # One more untimed replay: its all-reduces line the ranks' devices up, so the timed region starts
            # at the same moment on every rank whatever host-side skew follows the barrier.
            with torch.cuda.stream(stream):
                graph.replay()
        start.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(args.steps // gsteps):
                graph.replay()
        end.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    if max_over_ranks(float(device_error()), world) != 0:  # e.g. a peer wait that ran out: no number
        raise SystemExit("device error during the timed decode steps")
    ms = max_over_ranks(start.elapsed_time(end), world)
    ms_step = ms / args.steps
    value = B * args.steps / (ms / 1e3)

    # per-stage timing (eager, same step), roofline of the dominant kernel
    def dec_step():
        layer.forward_into(x, out, stream=torch.cuda.current_stream())

    st = stage_times(layer, dec_step, min(max(args.steps, 20), 50))
    names = STAGES
    byt = decode_bytes(B, world, 1 if args.weights.startswith("fp8") else 2)
    dec_stage = {n: round(t * 1e3, 2) for n, t in zip(names, st) if n not in ("conv", "chunk_prep")}
    dom = max(["in_proj", "recurrence", "out_proj"], key=lambda n: dec_stage[n])
    achieved = byt[dom] / (dec_stage[dom] * 1e-6) / 1e9
    geom = f"9B B={B} tp{world} {args.weights}"
    roofline = {"kernel": dom, "bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"],
                "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                "traffic": ncu_traffic(f"decode_{dom}", geom), "algorithmic_bytes": byt[dom],
                "peak_source": pk["source"] + " (HBM copy)"}
    step_achieved = byt["step"] / (ms_step * 1e-3) / 1e9
    decode_detail = {"stage_us": dec_stage, "step_bytes": byt["step"], "step_gbs": round(step_achieved, 1),
                     "step_hbm_frac": round(step_achieved / pk["hbm_gbs"], 4),
                     "graph": f"{gsteps} consecutive decode steps per CUDA-graph replay"}

    # End to end through the public API with pinned host buffers: every step copies its input host->device
    # and its result device->host inside the timed region (forward_host_async: the copies run on copy streams
    # with double-buffered device rows, overlapping the neighbouring steps' compute).
    # With 4 or more GPUs the ranks share the host traffic (split_io): rank r copies its 1/N of the sequences
    # in and out, and the communicator all-gathers the input over NVLink, so the job moves each step's input
    # and result across PCIe once instead of N times (8 GPUs copying the whole batch each: 1.13 M tok/s, bound
    # by the host side).  At 2 GPUs the all-gather on the call's stream costs more than it saves (1.11 against
    # 1.28 M tok/s), so each rank copies the whole batch.
    xh = x.detach().cpu().pin_memory()
    yh = [torch.empty_like(xh).pin_memory() for _ in range(2)]
    split = world >= 4
    for i in range(3):
        layer.forward_host_async(xh, yh[i % 2], split_io=split)
    torch.cuda.synchronize()
    barrier(world)
    e2e_steps = max(args.steps, 20)
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    es.record()
    for i in range(e2e_steps):
        ev = layer.forward_host_async(xh, yh[i % 2], split_io=split)
    ev.synchronize()
    ee.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(max(es.elapsed_time(ee), (time.perf_counter() - t0) * 1e3), world)
    e2e = {"value": round(B * e2e_steps / (e2e_ms / 1e3), 1), "unit": "tokens/s",
           "h2d_bytes_per_step": xh.numel() * xh.element_size(),
           "d2h_bytes_per_step": yh[0].numel() * yh[0].element_size(), "steps": e2e_steps,
           "path": "Qwen35GatedDeltaNet.forward_host_async (C-ABI gdn_layer_forward), pinned host in/out, "
                   "copies on copy streams overlapping the neighbouring steps" +
                   (f"; split_io: each of the {world} ranks copies 1/{world} of the sequences in and out and "
                    "all-gathers the input over NVLink (bytes above = the whole job's)" if split else ""),
           "timing": "max of host wall clock and CUDA events around all steps, max over ranks"}

    result = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": {
            "bf16": "bf16 (fp32 state, fp32 accumulation)",
            "fp8": "fp8 e4m3 projection weights, bf16 activations (fp32 state, fp32 accumulation)",
            "fp8_w8a8": "fp8 e4m3 projection weights and decode activations, bf16 elsewhere (fp32 state, fp32 accumulation)",
        }[args.weights], "data": "synthetic",
        "config": workload_config(world),
        "roofline": roofline, "decode": decode_detail, "e2e": e2e,
        "gpu_launches": launches_per_step * args.steps, "launches_per_step": launches_per_step,
        "clocks": clk.summary(),
    }
    if parity is not None:
        result["parity"] = parity
    if args.prefill:
        result["prefill"] = run_prefill(args, layer, dev, world, pk)
    if args.variants or args.stack:
        del graph, layer
        graph = None
        torch.cuda.empty_cache()
    if args.variants:
        result.update(run_variants(args, rank, world, comm, dev, pk))
    if args.stack:
        result["stack"] = run_stack(args, rank, world, comm, dev, pk)
    if device_error() != 0:
        raise SystemExit("device error during the benchmark")
    if rank == 0 and world == 1 and not args.no_cpu:
        result["cpu_baseline"] = cpu_baseline()
    del graph
    if comm is not None:
        comm.close()
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if parity is not None and not parity["ok"]:
        raise SystemExit(f"tensor-parallel parity failed: {parity}")


def run_prefill(args, layer_dec, dev, world, pk):
    """Config 3: batch 8 x 8192-token chunked prefill (weights shared with the decode layer)."""
    B, T = PREFILL_B, PREFILL_T
    layer_p = layer_dec.with_batch(B)  # same device weights, own batch and state
    g = torch.Generator(device=dev).manual_seed(5)
    x = torch.randn(B, T, H, generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty_like(x)
    steps = max(1, min(args.steps, args.prefill_steps))
    for _ in range(3):
        layer_p.forward_into(x, out)
    torch.cuda.synchronize()
    sampler = ClockSampler([dev.index] if int(os.environ.get("RANK", 0)) == 0 else None, 0.05 if world == 1 else None)
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with sampler as clk:
        torch.cuda.synchronize()
        if world > 1:  # an untimed step whose all-reduce lines the ranks' devices up (as in decode)
            layer_p.forward_into(x, out)
        s.record()
        for _ in range(steps):
            layer_p.forward_into(x, out)
        e.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(s.elapsed_time(e), world) / steps
    st = stage_times(layer_p, lambda: layer_p.forward_into(x, out), min(steps, 3))
    stage = {n: round(t, 3) for n, t in zip(STAGES, st)}
    fl = prefill_flops(B, T, world)
    tf = lambda n: fl[n] / (stage[n] * 1e-3) / 1e12
    rec_ms = stage["chunk_prep"] + stage["recurrence"]
    peak = pk["bf16_tflops"]  # burst: a ~10 ms kernel in a region well under a second
    geom = f"9B B={B} T={T} tp{world} {args.weights}"
    return {
        "workload": "cfg3: Qwen3.5-9B GDN layer chunked prefill, batch 8 x 8192 tokens, chunk 64",
        "value": round(B * T / (ms / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(ms, 3), "steps": steps,
        "scaling": "strong", "stage_ms": stage,
        "roofline": {"kernel": "in_proj", "bound": "tensor", "achieved": round(tf("in_proj"), 1),
                     "peak": peak, "unit": "TFLOP/s", "frac": round(tf("in_proj") / peak, 4),
                     "traffic": ncu_traffic("prefill_in_proj", geom), "algorithmic_flops": fl["in_proj"],
                     "peak_source": pk["source"] + " (burst bf16)"},
        "step_tflops": round(fl["step"] / (ms * 1e-3) / 1e12, 1),
        "step_tensor_frac": round(fl["step"] / (ms * 1e-3) / 1e12 / peak, 4),
        "recurrence_tflops": round(fl["recurrence"] / (rec_ms * 1e-3) / 1e12, 2),
        "clocks": clk.summary(),
    }


def graph_decode_us(forward, x, out, steps: int, world: int, dev) -> float:
    """Per-step device time (us) of `forward(x, out, stream)` replayed from a CUDA graph of 8 steps, max over
    ranks, after an eager warm-up and one graph replay."""
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        forward(x, out, stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(8):
            forward(x, out, stream)
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        if world > 1:
            graph.replay()
        s.record(stream)
        for _ in range(max(1, steps // 8)):
            graph.replay()
        e.record(stream)
    torch.cuda.synchronize()
    us = max_over_ranks(s.elapsed_time(e) * 1e3 / (8 * max(1, steps // 8)), world)
    del graph
    return us


def run_variants(args, rank, world, comm, dev, pk):
    """Rows f3 and f4 of the hot-path scope at the benchmark's decode batch (64 sequences per GPU, 9B
    geometry, head-parallel over the N GPUs): the layer with weight-only fp8 weights, and the whole decoder
    layer around the mixer (input RMSNorm, mixer, residual, post RMSNorm, SwiGLU MLP with intermediate 12288,
    residual; two all-reduces per call with N > 1), decode from CUDA graphs and a config-3-sized prefill."""
    from linear_attention_op_b200 import DecoderMlpWeights, Qwen35DecoderLayer, Qwen35GatedDeltaNet

    B, I = DECODE_B * world, 12288
    W = synthetic_weights(0, dev)
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(B, 1, H, generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty_like(x)
    res = {}
    lq = Qwen35GatedDeltaNet(weights=W, batch=B, device=dev, tp_rank=rank, tp_size=world, comm=comm, max_rows=B,
                             weight_dtype="fp8")
    us = graph_decode_us(lambda a, o, st: lq.forward_into(a, o, stream=st), x, out, args.steps, world, dev)
    byt = decode_bytes(B, world, 1)["step"]
    res["fp8_weight_only"] = {
        "workload": f"cfg2 decode with weight-only fp8 (e4m3) projection weights, batch {B}, tp{world}",
        "us_per_step": round(us, 2), "tokens_per_s": round(B / (us * 1e-6), 1), "step_bytes": byt,
        "step_hbm_frac": round(byt / (us * 1e-6) / 1e9 / pk["hbm_gbs"], 4)}
    del lq
    rn = lambda *sz: (torch.randn(*sz, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    mlp = DecoderMlpWeights(input_norm_w=torch.rand(H, generator=g, device=dev) - 0.5,
                            post_norm_w=torch.rand(H, generator=g, device=dev) - 0.5,
                            w_gate=rn(I, H), w_up=rn(I, H), w_down=rn(H, I))
    dec = Qwen35DecoderLayer(batch=B, mixer_weights=W, mlp_weights=mlp, device=dev, tp_rank=rank, tp_size=world,
                             comm=comm, max_rows=B)
    us = graph_decode_us(lambda a, o, st: dec.forward_into(a, o, stream=st), x, out, args.steps, world, dev)
    byt = decode_bytes(B, world)["step"] + 3 * H * (I // world) * 2 + 4 * B * H * 2
    entry = {"workload": f"Qwen3.5-9B linear-attention decoder layer (mixer + SwiGLU MLP, intermediate {I}), "
                         f"batch {B} decode, tp{world}",
             "decode_us_per_step": round(us, 2), "decode_tokens_per_s": round(B / (us * 1e-6), 1),
             "decode_step_bytes": byt, "decode_step_hbm_frac": round(byt / (us * 1e-6) / 1e9 / pk["hbm_gbs"], 4)}
    del dec
    dp = Qwen35DecoderLayer(batch=PREFILL_B, mixer_weights=W, mlp_weights=mlp, device=dev, tp_rank=rank,
                            tp_size=world, comm=comm, max_rows=PREFILL_B * PREFILL_T)
    xp = torch.randn(PREFILL_B, PREFILL_T, H, generator=g, device=dev).to(torch.bfloat16)
    op = torch.empty_like(xp)
    for _ in range(2):
        dp.forward_into(xp, op)
    torch.cuda.synchronize()
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dp.forward_into(xp, op)
    s.record()
    for _ in range(3):
        dp.forward_into(xp, op)
    e.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(s.elapsed_time(e), world) / 3
    fl = prefill_flops(PREFILL_B, PREFILL_T, world)["step"] + 6 * PREFILL_B * PREFILL_T * H * (I // world)
    entry.update({"prefill_workload": f"batch {PREFILL_B} x {PREFILL_T} tokens", "prefill_ms": round(ms, 3),
                  "prefill_tokens_per_s": round(PREFILL_B * PREFILL_T / (ms * 1e-3), 1),
                  "prefill_tflops": round(fl / (ms * 1e-3) / 1e12, 1),
                  "prefill_tensor_frac": round(fl / (ms * 1e-3) / 1e12 / pk["bf16_tflops"], 4)})
    res["decoder"] = entry
    del dp, xp, op
    torch.cuda.empty_cache()
    return res


def run_stack(args, rank, world, comm, dev, pk):
    """Config 4: a stack of 24 Qwen3.5-9B GDN layers (random init, per-layer seeds, A_log = log U(1, 64)),
    batch 128, a 4096-token prefill then 512 decode steps, head-parallel over the N GPUs (fixed total work:
    strong scaling).  The layers share one workspace, bounded by a 65536-row limit (the prefill runs in
    pieces of 512 tokens of all 128 sequences); every decode step of the whole stack is ONE CUDA-graph
    replay (24 layers, one all-reduce each)."""
    from linear_attention_op_b200 import GDNStack

    L, B, T0, steps = args.stack_layers, 128, args.stack_prefill, args.stack_steps
    weights = [synthetic_weights(1000 + i, dev, a_max=64.0) for i in range(L)]
    stack = GDNStack(weights, batch=B, device=dev, tp_rank=rank, tp_size=world, comm=comm, max_rows=65536)
    del weights
    g = torch.Generator(device=dev).manual_seed(9)
    x = torch.randn(B, T0, H, generator=g, device=dev).to(torch.bfloat16)
    bufs = [torch.empty_like(x), torch.empty_like(x)]
    outs = [bufs[i % 2] for i in range(L)]
    xd = torch.randn(B, 1, H, generator=g, device=dev).to(torch.bfloat16)
    douts = [torch.empty_like(xd) for _ in range(2)]
    dlist = [douts[i % 2] for i in range(L)]
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream())
    wb = [torch.empty(B, 128, H, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    with torch.cuda.stream(stream):  # warm-up: a short prefill and a decode step, then back to zero state
        stack.forward_into(x[:, :128].contiguous(), [wb[i % 2] for i in range(L)], stream=stream)
        stack.forward_into(xd, dlist, stream=stream)
    del wb
    torch.cuda.synchronize()
    stack.reset_state()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    barrier(world)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        ev[0].record(stream)
        stack.forward_into(x, outs, stream=stream)
        ev[1].record(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        stack.forward_into(xd, dlist, stream=stream)
    barrier(world)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        if world > 1:
            graph.replay()  # lines the ranks' devices up (its all-reduces); one extra untimed step
        ev[2].record(stream)
        for _ in range(steps):
            graph.replay()
        ev[3].record(stream)
    torch.cuda.synchronize()
    pre_ms = max_over_ranks(ev[0].elapsed_time(ev[1]), world)
    dec_ms = max_over_ranks(ev[2].elapsed_time(ev[3]), world)
    del graph
    byt = decode_bytes(B, world)["step"] * L  # per GPU per step
    fl = prefill_flops(B, T0, world)["step"] * L
    res = {
        "workload": f"cfg4: {L} Qwen3.5-9B GDN layers, batch {B}, {T0}-token prefill then {steps} decode steps, "
                    f"A_log = log U(1,64), tp{world} head-parallel",
        "scaling": "strong", "prefill_ms": round(pre_ms, 2), "prefill_tokens_per_s": round(B * T0 / (pre_ms / 1e3), 1),
        "prefill_tflops": round(fl / (pre_ms * 1e-3) / 1e12, 1),
        "decode_ms_per_step": round(dec_ms / steps, 4), "decode_tokens_per_s": round(B * steps / (dec_ms / 1e3), 1),
        "decode_step_gbs_per_gpu": round(byt / (dec_ms / steps * 1e-3) / 1e9, 1),
        "decode_step_hbm_frac": round(byt / (dec_ms / steps * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
        "tokens_per_s": round(B * (T0 + steps) / ((pre_ms + dec_ms) / 1e3), 1),
        "graph": f"one CUDA graph per decode step of all {L} layers",
        "prefill_row_limit": 65536,
    }
    del stack
    return res


# ---------------------------------------------------------------------------------------------------
# CPU baseline / reference arm: the oracle port on the host cores
# ---------------------------------------------------------------------------------------------------
def cpu_decode_rate(budget_s: float = 15.0, max_steps: int | None = None, warmup: int = 1):
    from oracle import gdn_oracle as O  # the CPU restatement of the reference path

    torch.set_num_threads(os.cpu_count() or 1)
    w = O.make_weights(H, HK, HV, seed=0)
    B = DECODE_B
    x = O.make_hidden(B, 1, H, seed=1)
    s = torch.randn(B, HV, D, D, generator=torch.Generator().manual_seed(1)) * 0.1
    c = torch.zeros(B, 3, 2 * HK * D + HV * D)
    with torch.no_grad():
        for _ in range(warmup):
            O.layer_forward(w, x, s, c)
        n, t0 = 0, time.perf_counter()
        while True:
            _, s, c = O.layer_forward(w, x, s, c)
            n += 1
            el = time.perf_counter() - t0
            if (max_steps is not None and n >= max_steps) or (max_steps is None and el >= budget_s):
                break
    return B * n / el, n, el, torch.get_num_threads()


def cpu_baseline():
    rate, n, el, cores = cpu_decode_rate()
    return {"value": round(rate, 1), "unit": "tokens/s", "cores": cores, "kind": "port", "cpu": cpu_model(),
            "sample": f"{n} cfg2 decode steps (batch 64, 9B GDN layer, fp32) in {el:.1f} s on the host cores"}


def run_reference(args):
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return
    rate_w = cpu_decode_rate(max_steps=args.warmup, warmup=0) if args.warmup > 0 else None
    del rate_w
    rate, n, el, cores = cpu_decode_rate(max_steps=args.steps, warmup=0)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(rate, 1), "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": n, "warmup": args.warmup, "ms_per_step": round(el / n * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": workload_config(args.gpus),
        "cpu_baseline": {"value": round(rate, 1), "unit": "tokens/s", "cores": cores, "kind": "port",
                         "cpu": cpu_model(),
                         "sample": f"{n} cfg2 decode steps of batch 64 on the host cores, each a bounded sample "
                                   f"of the workload's {DECODE_B * args.gpus} sequences (the reference's device "
                                   f"code is Tenstorrent-only; this is its CPU golden path restated)"},
        "e2e": {"value": round(rate, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-prefill", dest="prefill", action="store_false")
    ap.add_argument("--prefill-steps", type=int, default=5)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--only", choices=["all", "decode", "prefill"], default="all",
                    help="profiling: run only one workload (the headline line needs 'all')")
    ap.add_argument("--decode-b", type=int, default=DECODE_B)
    ap.add_argument("--graph-steps", type=int, default=16, help="decode steps captured per CUDA graph")
    ap.add_argument("--prefill-b", type=int, default=PREFILL_B)
    ap.add_argument("--prefill-t", type=int, default=PREFILL_T)
    ap.add_argument("--no-stack", dest="stack", action="store_false", help="skip the config-4 stack line")
    ap.add_argument("--no-variants", dest="variants", action="store_false",
                    help="skip the weight-only fp8 and decoder-layer lines")
    ap.add_argument("--stack-layers", type=int, default=24)
    ap.add_argument("--stack-prefill", type=int, default=4096)
    ap.add_argument("--stack-steps", type=int, default=512)
    ap.add_argument("--weights", choices=["bf16", "fp8", "fp8_w8a8"], default="bf16",
                    help="fp8: e4m3 projection weights, bf16 activations; fp8_w8a8: e4m3 decode activations too "
                         "(not the benchmark config's bf16 weights; reported beside it)")
    args = ap.parse_args()
    globals()["DECODE_B"], globals()["PREFILL_B"], globals()["PREFILL_T"] = args.decode_b, args.prefill_b, args.prefill_t
    if args.only == "decode":
        args.prefill = False
    if args.only != "all":
        args.stack = False
        args.variants = False
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
