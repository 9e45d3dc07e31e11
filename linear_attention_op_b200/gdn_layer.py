"""Host-side mirror of the reference's per-layer op API, on top of the C-ABI (``include/gdn_b200.h``).

* ``Qwen35GatedDeltaNet``  <- ``Qwen35GatedDeltaNetTT`` (9B/gdn_layer.py:54-292): full layer, prefill and
  decode, state kept on the device across calls, ``reset_state`` / ``get_recurrent_state``.
* ``GDNStack``             <- ``Qwen35_08B_GDNStackL1`` (0.8B/gdn_l1.py:147-341): several layers back to
  back with one state per layer, ``layers=[i]`` selection, ``allocate_activations`` / ``forward_into``
  for CUDA-graph replay (the reference's trace capture, 0.8B/bench_decode.py:44-57).
* ``GatedDeltaRule``       <- ``GatedDeltaRuleL1`` (9B/gated_delta_l1.py:131-272): the recurrence alone.
* ``Qwen35DecoderLayer``   <- Hugging Face ``Qwen3_5DecoderLayer`` of the linear-attention type: input RMSNorm,
  the mixer, residual, post RMSNorm, SwiGLU MLP, residual (the surroundings the reference names as its next
  step, 0.8B/OPTIMIZATION.md:258-259).

Everything runs in libgdn_b200.so; PyTorch only provides device memory and the current stream.  Errors
raise ``GDNError`` (the reference uses asserts / ValueError, which callers may also catch as RuntimeError).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import Dims, LayerInfo, MlpWeights, Weights, call

HEAD_DIM = 128


# The reference's weight_dtype (ttnn.bfloat16 / bfloat8_b) -> gdn_layer_set_weight_format's formats:
# "fp8" = e4m3 weights with bf16 activations (the reference's weight-only semantics, any tp_size);
# "fp8_w8a8" = e4m3 weights and per-token e4m3 decode activations (tp_size 1).
WEIGHT_FORMATS = {"bf16": 0, "fp8_w8a8": 1, "fp8": 2}


def _stream_handle(stream: torch.cuda.Stream | None = None) -> ctypes.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _to_device(t: torch.Tensor, device: torch.device) -> tuple[torch.Tensor, bool]:
    """Contiguous bf16 copy of t on device; a pinned host tensor is copied without blocking the host
    (the caller synchronises before it returns)."""
    pinned = t.device.type == "cpu" and t.is_pinned()
    return t.to(device=device, dtype=torch.bfloat16, non_blocking=pinned).contiguous(), pinned


def _to_caller(out: torch.Tensor, like: torch.Tensor, pinned: bool) -> torch.Tensor:
    """out (device bf16) in like's device and dtype.  For a pinned host input the result comes back into
    pinned host memory (a direct DMA, where a pageable destination would be staged) and the current stream
    is synchronised before returning."""
    if not pinned:
        return out.to(device=like.device, dtype=like.dtype)
    src = out if like.dtype == out.dtype else out.to(like.dtype)
    res = torch.empty(src.shape, dtype=src.dtype, pin_memory=True)
    res.copy_(src, non_blocking=True)
    torch.cuda.current_stream().synchronize()
    return res


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


@dataclass
class LayerWeights:
    """HF-layout weights of one layer (host or device tensors).  Projections are converted to bf16."""

    w_qkv: torch.Tensor
    w_z: torch.Tensor
    w_a: torch.Tensor
    w_b: torch.Tensor
    conv_w: torch.Tensor  # [conv_dim, K]
    a_log: torch.Tensor
    dt_bias: torch.Tensor
    norm_w: torch.Tensor
    w_out: torch.Tensor
    num_k_heads: int
    num_v_heads: int
    head_k_dim: int = HEAD_DIM
    head_v_dim: int = HEAD_DIM
    eps: float = 1e-6

    @property
    def hidden(self) -> int:
        return int(self.w_qkv.shape[1])

    @classmethod
    def from_hf(cls, layer) -> "LayerWeights":
        """From a Hugging Face ``Qwen3_5GatedDeltaNet`` (the reference's constructor argument)."""
        g = lambda t: t.detach()
        eps = getattr(layer.norm, "variance_epsilon", None) or getattr(layer, "layer_norm_epsilon", 1e-6)
        return cls(g(layer.in_proj_qkv.weight), g(layer.in_proj_z.weight), g(layer.in_proj_a.weight),
                   g(layer.in_proj_b.weight), g(layer.conv1d.weight)[:, 0, :], g(layer.A_log), g(layer.dt_bias),
                   g(layer.norm.weight), g(layer.out_proj.weight), int(layer.num_k_heads), int(layer.num_v_heads),
                   int(layer.head_k_dim), int(layer.head_v_dim), float(eps))

    @classmethod
    def from_any(cls, w) -> "LayerWeights":
        if isinstance(w, cls):
            return w
        if hasattr(w, "in_proj_qkv"):
            return cls.from_hf(w)
        fields = ("w_qkv", "w_z", "w_a", "w_b", "conv_w", "a_log", "dt_bias", "norm_w", "w_out", "num_k_heads",
                  "num_v_heads")
        get = (lambda k: w[k]) if isinstance(w, dict) else (lambda k: getattr(w, k))
        kw = {k: get(k) for k in fields}
        for k in ("head_k_dim", "head_v_dim", "eps"):
            try:
                kw[k] = get(k)
            except (KeyError, AttributeError):
                pass
        return cls(**kw)


class _LayerHandle:
    """Owns one gdn_layer* (this rank's head shard of one layer's weights, on the current device)."""

    def __init__(self, weights: LayerWeights, tp_rank: int = 0, tp_size: int = 1):
        w = weights
        bf = lambda t: t.detach().to(torch.bfloat16).contiguous()
        f32 = lambda t: t.detach().to(torch.float32).contiguous()
        keep = dict(w_qkv=bf(w.w_qkv), w_z=bf(w.w_z), w_a=bf(w.w_a), w_b=bf(w.w_b), conv_w=f32(w.conv_w),
                    a_log=f32(w.a_log), dt_bias=f32(w.dt_bias), norm_w=f32(w.norm_w), w_out=bf(w.w_out))
        self.dims = Dims(w.hidden, w.num_k_heads, w.num_v_heads, w.head_k_dim, w.head_v_dim,
                         int(keep["conv_w"].shape[1]), float(w.eps), 64)
        cw = Weights(*(ctypes.c_void_p(keep[k].data_ptr()) for k in
                       ("w_qkv", "w_z", "w_a", "w_b", "conv_w", "a_log", "dt_bias", "norm_w", "w_out")))
        handle = ctypes.c_void_p()
        call("gdn_layer_create", ctypes.byref(self.dims), ctypes.byref(cw), tp_rank, tp_size, ctypes.byref(handle))
        self.handle = handle
        self.info = LayerInfo()
        call("gdn_layer_get_info", self.handle, ctypes.byref(self.info))
        self.hidden = w.hidden

    def reserve(self, max_tokens: int, max_batch: int = 64) -> None:
        call("gdn_layer_reserve_batch", self.handle, int(max_tokens), int(max_batch))

    def set_max_rows(self, max_rows: int) -> None:
        call("gdn_layer_set_max_rows", self.handle, int(max_rows))

    def forward(self, x: torch.Tensor, B: int, T: int, rec: torch.Tensor, conv: torch.Tensor, out: torch.Tensor,
                comm=None, stream=None) -> None:
        call("gdn_layer_forward", self.handle, _ptr(x), B, T, _ptr(rec), _ptr(conv), _ptr(out),
             ctypes.c_void_p(comm.handle.value if comm is not None else 0), _stream_handle(stream))

    def close(self) -> None:
        if getattr(self, "handle", None) is not None and self.handle.value:
            _lib.lib().gdn_layer_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Qwen35GatedDeltaNet:
    """One Gated DeltaNet layer on a B200, continuing from its on-device state across calls.

    Drop-in for ``Qwen35GatedDeltaNetTT(device, hf_layer, batch)``: ``layer(x)`` with x ``[B, T, hidden]``
    (any device/dtype) returns ``[B, T, hidden]`` on x's device in x's dtype; T == 1 is a decode step,
    T > 1 a chunked prefill.  ``tp_rank``/``tp_size``/``comm`` shard the heads over GPUs (one NCCL
    all-reduce per call); with ``tp_size > 1`` and ``comm=None`` the call returns this rank's partial sum.
    ``weight_dtype="fp8"`` (the reference's ``weight_dtype=ttnn.bfloat8_b`` mode: weights quantised, activations
    not) quantises the projection weights to e4m3 with per-row power-of-two scales: decode steps stream half
    the weight bytes, prefill uses the dequantised weights; it works head-parallel too.
    ``weight_dtype="fp8_w8a8"`` also quantises the decode activations per token (e4m3 x e4m3 GEMMs, one GPU).
    """

    def __init__(self, hf_layer=None, batch: int = 1, *, weights=None, device=None, tp_rank: int = 0,
                 tp_size: int = 1, comm=None, max_rows: int | None = None, weight_dtype: str = "bf16"):
        if (hf_layer is None) == (weights is None):
            raise ValueError("pass exactly one of hf_layer or weights")
        if batch <= 0:
            raise ValueError("batch must be > 0")
        if weight_dtype not in WEIGHT_FORMATS:
            raise ValueError(f"weight_dtype must be one of {sorted(WEIGHT_FORMATS)}")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.batch = batch
        self.comm = comm
        self.tp_rank, self.tp_size = tp_rank, tp_size
        w = LayerWeights.from_any(hf_layer if hf_layer is not None else weights)
        with torch.cuda.device(self.device):
            self._h = _LayerHandle(w, tp_rank, tp_size)
            if weight_dtype != "bf16":  # before any reserve: fp8 decode calls need more workspace
                call("gdn_layer_set_weight_format", self._h.handle, WEIGHT_FORMATS[weight_dtype])
        self.weight_dtype = weight_dtype
        info = self._h.info
        self.hidden = info.hidden
        self.nk, self.nv = w.num_k_heads, w.num_v_heads
        self.nk_local, self.nv_local = info.num_k_heads_local, info.num_v_heads_local
        self.conv_dim_local = info.conv_dim_local
        self.dk = self.dv = HEAD_DIM
        if max_rows:
            # the reference's max_rows (9B/gdn_layer.py:55-66, 282-292): longer prefill calls run in pieces of
            # at most max_rows rows, and the workspace is reserved for them once
            if max_rows < batch:
                raise ValueError(f"max_rows {max_rows} must be >= batch {batch}")
            self._h.set_max_rows(max_rows)
            with torch.cuda.device(self.device):
                self._h.reserve(max_rows, batch)
        self.max_rows = max_rows
        self._io = None
        self.reset_state()

    # ---- state (9B/gdn_layer.py:137-157) -----------------------------------------------------------
    def reset_state(self) -> None:
        """Zero both states in place (their device addresses never change, so captured graphs stay valid)."""
        B = self.batch
        if getattr(self, "rec_state", None) is None:
            self.rec_state = torch.zeros(B, self.nv_local, self.dk, self.dv, dtype=torch.float32, device=self.device)
            self.conv_state = torch.zeros(B, 3, self.conv_dim_local, dtype=torch.float32, device=self.device)
        else:
            self.rec_state.zero_()
            self.conv_state.zero_()

    def set_state(self, rec_state: torch.Tensor | None = None, conv_state: torch.Tensor | None = None) -> None:
        if rec_state is not None:
            self.rec_state.copy_(rec_state.reshape(self.rec_state.shape))
        if conv_state is not None:
            self.conv_state.copy_(conv_state.reshape(self.conv_state.shape))

    def get_recurrent_state(self) -> torch.Tensor:
        """[B, Hv_local, dk, dv] host copy (for checks)."""
        return self.rec_state.detach().float().cpu()

    def get_conv_state(self) -> torch.Tensor:
        """[B, 3, conv_dim_local] host copy: rows hold the last 3 pre-conv inputs, oldest first."""
        return self.conv_state.detach().float().cpu()

    # ---- forward -----------------------------------------------------------------------------------
    def forward_into(self, x: torch.Tensor, out: torch.Tensor, stream=None) -> torch.Tensor:
        """Device bf16 x [B, T, hidden] -> device bf16 out (preallocated); allocates nothing once the
        workspace is reserved, so it can be captured in a CUDA graph."""
        B, T, H = x.shape
        if B != self.batch or H != self.hidden:
            raise ValueError(f"x is {tuple(x.shape)}, layer expects [{self.batch}, T, {self.hidden}]")
        if x.dtype != torch.bfloat16 or out.dtype != torch.bfloat16 or not x.is_contiguous() or not out.is_contiguous():
            raise ValueError("forward_into wants contiguous bf16 tensors")
        self._h.forward(x, B, T, self.rec_state, self.conv_state, out, self.comm, stream)
        return out

    def __call__(self, hidden_states: torch.Tensor) -> torch.Tensor:
        B, T, H = hidden_states.shape
        if B != self.batch or H != self.hidden:
            raise ValueError(f"hidden_states is {tuple(hidden_states.shape)}, layer expects [{self.batch}, T, {self.hidden}]")
        with torch.cuda.device(self.device):
            x, pinned = _to_device(hidden_states, self.device)
            out = torch.empty_like(x)
            self.forward_into(x, out)
            return _to_caller(out, hidden_states, pinned)

    def forward_host_async(self, x_host: torch.Tensor, out_host: torch.Tensor,
                           split_io: bool = False) -> torch.cuda.Event:
        """Pinned host bf16 x [B, T, hidden] -> pinned host bf16 out, without waiting: the host-to-device copy,
        the layer call and the device-to-host copy are queued and the returned event completes when out_host
        holds the result.  Copies run on two copy streams with double-buffered device rows, so a call's
        input copy overlaps the previous call's compute and its result copy the next call's compute (the
        calls themselves stay in order on the current stream).  x_host must not change, and out_host must
        not be read, before the event completes.

        split_io (tensor-parallel layer with its communicator, batch divisible by the group size): the
        ranks share the host traffic instead of each moving the whole batch -- rank r copies only sequences
        [r B / G, (r + 1) B / G) of x_host in, the communicator all-gathers the other ranks' sequences over
        NVLink before the call, and only rank r's sequences of the (identical) result are copied out to
        out_host.  Every rank passes the whole input; the whole output is the union of the ranks' shares."""
        B, T, H = x_host.shape
        G, r = self.tp_size, self.tp_rank
        if split_io and (G == 1 or self.comm is None or B % G):
            raise ValueError("split_io needs a tensor-parallel layer with its communicator and batch % tp_size == 0")
        if B != self.batch or H != self.hidden or tuple(out_host.shape) != (B, T, H):
            raise ValueError(f"x {tuple(x_host.shape)} / out {tuple(out_host.shape)} do not match [{self.batch}, T, {self.hidden}]")
        if x_host.dtype != torch.bfloat16 or out_host.dtype != torch.bfloat16 or not (x_host.is_pinned() and out_host.is_pinned()):
            raise ValueError("forward_host_async wants pinned host bf16 tensors")
        with torch.cuda.device(self.device):
            io = self._io
            if io is None or io["shape"] != (B, T, H):
                dev = lambda: torch.empty(B, T, H, dtype=torch.bfloat16, device=self.device)
                io = self._io = {"shape": (B, T, H), "xin": [dev(), dev()], "xout": [dev(), dev()], "i": 0,
                                 "h2d_stream": torch.cuda.Stream(self.device), "d2h_stream": torch.cuda.Stream(self.device),
                                 "h2d": [torch.cuda.Event(), torch.cuda.Event()], "d2h": [torch.cuda.Event(), torch.cuda.Event()],
                                 "done": [torch.cuda.Event(), torch.cuda.Event()]}
            i = io["i"]
            io["i"] = i ^ 1
            cur = torch.cuda.current_stream()
            hs, ds = io["h2d_stream"], io["d2h_stream"]
            rows = slice(r * (B // G), (r + 1) * (B // G)) if split_io else slice(0, B)
            hs.wait_event(io["done"][i])  # the call that last read xin[i] has finished
            with torch.cuda.stream(hs):
                io["xin"][i][rows].copy_(x_host[rows], non_blocking=True)
                io["h2d"][i].record(hs)
            cur.wait_event(io["h2d"][i])
            cur.wait_event(io["d2h"][i])  # the copy that last read xout[i] has finished
            if split_io:
                self.comm.allgather_(io["xin"][i], stream=cur)
            self.forward_into(io["xin"][i], io["xout"][i], stream=cur)
            io["done"][i].record(cur)
            ds.wait_event(io["done"][i])
            with torch.cuda.stream(ds):
                out_host[rows].copy_(io["xout"][i][rows], non_blocking=True)
                io["d2h"][i].record(ds)
            return io["d2h"][i]

    def reserve(self, max_tokens: int, max_batch: int | None = None) -> None:
        with torch.cuda.device(self.device):
            self._h.reserve(max_tokens, max_batch if max_batch is not None else max(self.batch, 64))

    def share_workspace(self, owner: "Qwen35GatedDeltaNet") -> None:
        """Use owner's device workspace instead of this layer's own (gdn_layer_share_workspace); the two
        must then run on one stream."""
        call("gdn_layer_share_workspace", self._h.handle, owner._h.handle)

    def workspace_bytes(self) -> int:
        info = LayerInfo()
        call("gdn_layer_get_info", self._h.handle, ctypes.byref(info))
        return int(info.workspace_bytes)

    def with_batch(self, batch: int) -> "Qwen35GatedDeltaNet":
        """Another op over the same device weights (and workspace) with its own batch size and zeroed state.
        The two ops must not run concurrently on different streams (they share the workspace)."""
        other = object.__new__(Qwen35GatedDeltaNet)
        other.__dict__.update({k: v for k, v in self.__dict__.items() if k not in ("rec_state", "conv_state")})
        other.batch = batch
        other.rec_state = other.conv_state = None
        other._io = None
        other.reset_state()
        return other

    def set_stage_events(self, events: list | None) -> None:
        """Have every forward record up to 7 timing events at its stage boundaries (see
        gdn_layer_set_stage_events); None disables."""
        if not events:
            call("gdn_layer_set_stage_events", self._h.handle, None, 0)
            self._stage_events = None
            return
        for e in events:  # torch creates the CUDA event lazily on first record
            e.record()
        arr = (ctypes.c_void_p * len(events))(*[ctypes.c_void_p(e.cuda_event) for e in events])
        call("gdn_layer_set_stage_events", self._h.handle, arr, len(events))
        self._stage_events = (events, arr)


class GDNStack:
    """Several GDN layers run back to back, each with its own state (decode or prefill).

    Drop-in for ``Qwen35_08B_GDNStackL1(device, hf_layers, batch)``: ``stack(x, layers=None)`` applies the
    selected layers in order (GDN mixers only: no norms, residuals or MLP, like the reference).  The layers
    run on one stream and share one device workspace (sized by the largest call), as the reference's stack
    shares its scratch buffers."""

    def __init__(self, hf_layers, batch: int = 1, *, device=None, tp_rank: int = 0, tp_size: int = 1, comm=None,
                 max_rows: int | None = None, weight_dtype: str = "bf16"):
        self.batch = batch
        self.layers = [Qwen35GatedDeltaNet(weights=LayerWeights.from_any(L), batch=batch, device=device,
                                           tp_rank=tp_rank, tp_size=tp_size, comm=comm, weight_dtype=weight_dtype)
                       for L in hf_layers]
        for L in self.layers[1:]:
            L.share_workspace(self.layers[0])
        if max_rows:
            if max_rows < batch:
                raise ValueError(f"max_rows {max_rows} must be >= batch {batch}")
            for L in self.layers:
                L._h.set_max_rows(max_rows)
                L.max_rows = max_rows
            self.layers[0].reserve(max_rows, batch)
        self.hidden = self.layers[0].hidden
        self.device = self.layers[0].device

    def reset_state(self) -> None:
        for L in self.layers:
            L.reset_state()

    def get_recurrent_state(self, i: int) -> torch.Tensor:
        return self.layers[i].get_recurrent_state()

    def allocate_activations(self, seq_len: int = 1) -> list[torch.Tensor]:
        """One persistent bf16 output buffer per layer, for forward_into / CUDA-graph capture."""
        return [torch.empty(self.batch, seq_len, self.hidden, dtype=torch.bfloat16, device=self.device)
                for _ in self.layers]

    def forward_into(self, x: torch.Tensor, outs: list[torch.Tensor], stream=None) -> torch.Tensor:
        for L, out in zip(self.layers, outs):
            L.forward_into(x, out, stream)
            x = out
        return x

    def __call__(self, hidden_states: torch.Tensor, layers=None) -> torch.Tensor:
        shape = hidden_states.shape
        x = hidden_states.reshape(self.batch, -1, shape[-1])
        idx = range(len(self.layers)) if layers is None else layers
        with torch.cuda.device(self.device):
            cur, pinned = _to_device(x, self.device)
            for i in idx:
                out = torch.empty_like(cur)
                self.layers[i].forward_into(cur, out)
                cur = out
            return _to_caller(cur, hidden_states, pinned).reshape(shape)


class GatedDeltaRule:
    """The recurrence alone with its state resident on the device across calls.

    Drop-in for ``GatedDeltaRuleL1(device, num_heads, head_k_dim, head_v_dim, initial_state=...)``:
    ``op(q, k, v, g, beta, use_qk_l2norm=True, scale=None)`` with q, k ``[B, T, Hk, dk]``, v
    ``[B, T, Hv, dv]``, g, beta ``[B, T, Hv]`` returns o ``[B, T, Hv, dv]``; ``num_heads`` = B * Hv."""

    def __init__(self, num_heads: int, head_k_dim: int = HEAD_DIM, head_v_dim: int = HEAD_DIM, *, device=None,
                 initial_state: torch.Tensor | None = None):
        if head_k_dim != HEAD_DIM or head_v_dim != HEAD_DIM:
            raise ValueError("only head dims of 128 are supported")
        self.num_heads = num_heads
        self.dk, self.dv = head_k_dim, head_v_dim
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.state = torch.zeros(num_heads, self.dk, self.dv, dtype=torch.float32, device=self.device)
        self.reset_state(initial_state)

    def reset_state(self, initial_state: torch.Tensor | None = None) -> None:
        """Reset in place (the buffer address never changes, like the reference's L1 state)."""
        if initial_state is None:
            self.state.zero_()
        else:
            self.state.copy_(initial_state.reshape(self.state.shape))

    def get_state(self) -> torch.Tensor:
        """[num_heads, dk, dv] host copy (for checks)."""
        return self.state.detach().cpu()

    def __call__(self, q, k, v, g, beta, use_qk_l2norm: bool = True, scale: float | None = None) -> torch.Tensor:
        B, T, Hk, dk = q.shape
        Hv = v.shape[2]
        if B * Hv != self.num_heads or dk != self.dk or v.shape[3] != self.dv or Hv % Hk:
            raise ValueError(f"shapes q {tuple(q.shape)} v {tuple(v.shape)} do not match num_heads={self.num_heads}")
        dev = lambda t: t.to(device=self.device, dtype=torch.float32).contiguous()
        with torch.cuda.device(self.device):
            qd, kd, vd, gd, bd = dev(q), dev(k), dev(v), dev(g), dev(beta)
            o = torch.empty(B, T, Hv, self.dv, dtype=torch.float32, device=self.device)
            call("gdn_recurrence_forward", _ptr(qd), _ptr(kd), _ptr(vd), _ptr(gd), _ptr(bd), B, T, Hk, Hv,
                 1 if use_qk_l2norm else 0, float(scale) if scale else 0.0, _ptr(self.state), _ptr(o),
                 _stream_handle())
        return o.to(q.device)


@dataclass
class DecoderMlpWeights:
    """The decoder layer's weights around the mixer (host or device tensors): RMSNorm weights [hidden]
    (applied as 1 + w), gate/up [intermediate, hidden], down [hidden, intermediate]."""

    input_norm_w: torch.Tensor
    post_norm_w: torch.Tensor
    w_gate: torch.Tensor
    w_up: torch.Tensor
    w_down: torch.Tensor
    eps: float = 1e-6

    @classmethod
    def from_hf(cls, layer) -> "DecoderMlpWeights":
        """From a Hugging Face ``Qwen3_5DecoderLayer`` (linear-attention type)."""
        g = lambda t: t.detach()
        return cls(g(layer.input_layernorm.weight), g(layer.post_attention_layernorm.weight),
                   g(layer.mlp.gate_proj.weight), g(layer.mlp.up_proj.weight), g(layer.mlp.down_proj.weight),
                   float(layer.input_layernorm.eps))


class Qwen35DecoderLayer:
    """A whole Qwen3.5 decoder layer of the linear-attention type on a B200, continuing from the mixer's
    on-device state across calls: ``layer(x)`` with x ``[B, T, hidden]`` returns ``[B, T, hidden]``
    (T == 1 decode, T > 1 prefill), as HF ``Qwen3_5DecoderLayer`` with its cache does.  ``mixer`` is the
    ``Qwen35GatedDeltaNet`` inside (its state, ``reset_state``, ``get_recurrent_state``, weight format and row
    limit).  With ``tp_size > 1`` a communicator is required: every rank gets the full output."""

    def __init__(self, hf_layer=None, batch: int = 1, *, mixer_weights=None, mlp_weights=None, device=None,
                 tp_rank: int = 0, tp_size: int = 1, comm=None, max_rows: int | None = None,
                 weight_dtype: str = "bf16"):
        if hf_layer is not None:
            mixer_weights, mlp_weights = hf_layer.linear_attn, DecoderMlpWeights.from_hf(hf_layer)
        if mixer_weights is None or mlp_weights is None:
            raise ValueError("pass hf_layer, or mixer_weights and mlp_weights")
        if tp_size > 1 and comm is None:
            raise ValueError("a tensor-parallel decoder layer needs its communicator")
        self.mixer = Qwen35GatedDeltaNet(weights=mixer_weights, batch=batch, device=device, tp_rank=tp_rank,
                                         tp_size=tp_size, comm=comm, max_rows=max_rows, weight_dtype=weight_dtype)
        self.device, self.batch, self.hidden, self.comm = self.mixer.device, batch, self.mixer.hidden, comm
        m = mlp_weights
        bf = lambda t: t.detach().to(torch.bfloat16).contiguous()
        f32 = lambda t: t.detach().to(torch.float32).contiguous()
        keep = dict(input_norm_w=f32(m.input_norm_w), post_norm_w=f32(m.post_norm_w), w_gate=bf(m.w_gate),
                    w_up=bf(m.w_up), w_down=bf(m.w_down))
        self.intermediate = int(keep["w_gate"].shape[0])
        cw = MlpWeights(*(ctypes.c_void_p(keep[k].data_ptr()) for k in
                          ("input_norm_w", "post_norm_w", "w_gate", "w_up", "w_down")), self.intermediate, float(m.eps))
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            call("gdn_decoder_create", self.mixer._h.handle, ctypes.byref(cw), ctypes.byref(handle))
            if max_rows:
                call("gdn_decoder_reserve", handle, int(max_rows))
        self.handle = handle

    # state: the mixer's
    def reset_state(self) -> None:
        self.mixer.reset_state()

    def set_state(self, rec_state=None, conv_state=None) -> None:
        self.mixer.set_state(rec_state, conv_state)

    def get_recurrent_state(self) -> torch.Tensor:
        return self.mixer.get_recurrent_state()

    def get_conv_state(self) -> torch.Tensor:
        return self.mixer.get_conv_state()

    def forward_into(self, x: torch.Tensor, out: torch.Tensor, stream=None) -> torch.Tensor:
        """Device bf16 x [B, T, hidden] -> device bf16 out (preallocated, not aliasing x)."""
        B, T, H = x.shape
        if B != self.batch or H != self.hidden:
            raise ValueError(f"x is {tuple(x.shape)}, layer expects [{self.batch}, T, {self.hidden}]")
        if x.dtype != torch.bfloat16 or out.dtype != torch.bfloat16 or not x.is_contiguous() or not out.is_contiguous():
            raise ValueError("forward_into wants contiguous bf16 tensors")
        mx = self.mixer
        call("gdn_decoder_forward", self.handle, _ptr(x), B, T, _ptr(mx.rec_state), _ptr(mx.conv_state), _ptr(out),
             ctypes.c_void_p(self.comm.handle.value if self.comm is not None else 0), _stream_handle(stream))
        return out

    def __call__(self, hidden_states: torch.Tensor) -> torch.Tensor:
        with torch.cuda.device(self.device):
            x, pinned = _to_device(hidden_states, self.device)
            out = torch.empty_like(x)
            self.forward_into(x, out)
            return _to_caller(out, hidden_states, pinned)

    def close(self) -> None:
        if getattr(self, "handle", None) is not None and self.handle.value:
            _lib.lib().gdn_decoder_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
