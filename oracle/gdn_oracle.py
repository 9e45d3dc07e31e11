"""CPU oracle for the Qwen3.5 Gated DeltaNet (GDN) layer -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.  The CUDA library under
``linear_attention_op_b200/`` never calls into it and has no CPU fallback.

It restates, in plain fp32 torch on the CPU, the algorithm of the reference's CPU golden path:

* ``wormhole_n150/qwen3.5_9B/reference.py`` -- the reference's own recurrence (``l2norm`` :7-8,
  ``recurrent_gated_delta_rule`` :11-35);
* the Hugging Face ``Qwen3_5GatedDeltaNet`` forward that every reference test compares against
  (``9B/test_gdn_layer.py:42-73``, ``0.8B/test_gdn_l1.py:82-93``), whose algorithm lives in the
  third-party package transformers 5.5.0 (``models/qwen3_5/modeling_qwen3_5.py``:
  ``Qwen3_5RMSNormGated`` :175-190, ``torch_causal_conv1d_update`` :210-225, ``l2norm`` :228-231,
  ``torch_chunk_gated_delta_rule`` :234-311, ``torch_recurrent_gated_delta_rule`` :314-353,
  ``Qwen3_5GatedDeltaNet.forward`` :422-533);
* the reference layer op's state semantics (``9B/gdn_layer.py:244-292``): weights in, hidden states plus
  the fp32 recurrent state and the rolling conv state in and out, long inputs continued from the state.

Parity pinning: ``tests/golden/make_golden.py`` imports the reference's ``reference.py`` and the HF layer in
the build container and stores their outputs as fixtures; ``tests/test_oracle_golden.py`` checks this
module against every fixture.

Conventions (the same as the C-ABI in ``include/gdn_b200.h``):

* hidden states ``x``: ``[B, T, hidden]``; rows are sequence-major (``b*T + t``), as in
  ``9B/kernels/layer_reader.cpp:108-110``;
* recurrent state ``S``: ``[B, Hv, dk, dv]`` fp32, indexed ``S[k_index, v_index]``
  (``reference.py:26-34``);
* conv state: ``[B, K-1, conv_dim]`` fp32, row ``j`` holds the pre-conv input at time ``T-(K-1)+j``
  (the reference keeps the last 3 inputs, ``9B/kernels/layer_reader.cpp:184-197``; Hugging Face keeps the
  last K = 4 inputs as ``[B, conv_dim, K]``; ``hf_conv_state_to_abi`` converts).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

# ------------------------------------------------------------------------------------------------
# Elementary pieces
# ------------------------------------------------------------------------------------------------


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """x * rsqrt(sum(x^2) + eps) over the last dim (``reference.py:7-8``; HF ``l2norm`` eps 1e-6)."""
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def gating(a: torch.Tensor, b: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor):
    """Per (token, v-head) decay and write strength.

    g = -exp(A_log) * softplus(a + dt_bias)   (softplus threshold 20, ``9B/kernels/layer_compute.cpp:160-166``)
    beta = sigmoid(b)                          (``layer_compute.cpp:176-177``)
    """
    g = -a_log.float().exp() * F.softplus(a.float() + dt_bias.float(), beta=1.0, threshold=20.0)
    return g, torch.sigmoid(b.float())


def causal_conv1d(x: torch.Tensor, weight: torch.Tensor, conv_state: torch.Tensor | None):
    """Depthwise causal conv + SiLU with a rolling state.

    x: [B, T, C] pre-conv channels; weight: [C, K] (tap j multiplies the input at time t-(K-1)+j, the
    layout of HF ``conv1d.weight[:, 0, :]`` and of the reference's tap diagonals, ``9B/gdn_layer.py:101-103``);
    conv_state: [B, K-1, C] (zeros if None).
    Returns (SiLU(conv(x)) [B, T, C], new_state [B, K-1, C]).  The new state holds the last K-1 inputs of
    the concatenation [state; x] (``layer_reader.cpp:184-197``), so a short call keeps older history.
    """
    B, T, C = x.shape
    K = weight.shape[1]
    if conv_state is None:
        conv_state = torch.zeros(B, K - 1, C, dtype=torch.float32)
    xs = torch.cat([conv_state.float(), x.float()], dim=1)  # [B, K-1+T, C]
    out = torch.zeros(B, T, C, dtype=torch.float32)
    w = weight.float()
    for j in range(K):
        out += xs[:, j:j + T, :] * w[:, j]
    return F.silu(out), xs[:, T:, :].clone()


def rmsnorm_gated(o: torch.Tensor, z: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6):
    """RMSNorm over the head dim, times weight, times SiLU(z), all in fp32
    (HF ``Qwen3_5RMSNormGated``; ``9B/kernels/layer_compute.cpp:287-395``)."""
    o = o.float()
    var = (o * o).mean(-1, keepdim=True)
    return (o * torch.rsqrt(var + eps)) * weight.float() * F.silu(z.float())


def expand_heads(x: torch.Tensor, hv: int) -> torch.Tensor:
    """GQA: v-head h reads k-head h // (Hv/Hk) (``reference.py:21-23``, ``9B/gdn_layer.py:48-51``)."""
    hk = x.shape[2]
    return x if hk == hv else x.repeat_interleave(hv // hk, dim=2)


# ------------------------------------------------------------------------------------------------
# The recurrence: sequential and chunked forms
# ------------------------------------------------------------------------------------------------


def recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=None, use_qk_l2norm=True, scale=None):
    """Token-by-token gated delta rule in fp32 (``reference.py:11-35``).

    q, k: [B, T, Hk, dk]; v: [B, T, Hv, dv]; g (log decay), beta: [B, T, Hv].
    Per token:  S <- exp(g) S;  u = beta (v - S^T k);  S <- S + k u^T;  o = S^T q.
    Returns (o [B, T, Hv, dv], S [B, Hv, dk, dv]).
    """
    q, k, v, g, beta = (t.float() for t in (q, k, v, g, beta))
    if use_qk_l2norm:
        q, k = l2norm(q), l2norm(k)
    B, T, _, dk = q.shape
    Hv, dv = v.shape[2], v.shape[3]
    q, k = expand_heads(q, Hv), expand_heads(k, Hv)
    q = q * (dk ** -0.5 if scale is None else scale)
    S = torch.zeros(B, Hv, dk, dv) if initial_state is None else initial_state.float().clone()
    o = torch.empty(B, T, Hv, dv)
    for t in range(T):
        S = S * g[:, t].exp()[..., None, None]
        kt = k[:, t]
        u = (v[:, t] - torch.einsum("bhkv,bhk->bhv", S, kt)) * beta[:, t][..., None]
        S = S + kt[..., :, None] * u[..., None, :]
        o[:, t] = torch.einsum("bhkv,bhk->bhv", S, q[:, t])
    return o, S


def chunk_gated_delta_rule(q, k, v, g, beta, initial_state=None, chunk=64, use_qk_l2norm=True, scale=None):
    """Chunked (WY/UT) form of the same recurrence, fp32.

    Follows the algorithm of HF ``torch_chunk_gated_delta_rule`` (modeling_qwen3_5.py:234-311; Yang et al.,
    "Parallelizing Linear Transformers with the Delta Rule over Sequence Length", 2024), restated with a
    triangular solve and an explicit initial state (HF's layer always starts prefill from zero).
    Per chunk of C tokens with in-chunk cumulative log decay G_i = sum_{j<=i} g_j:
        M_ij = beta_i (k_i . k_j) exp(G_i - G_j)   for j < i            (strictly lower)
        T    = (I + M)^-1
        U    = T (beta * v),   W = T (beta * exp(G) * k)
        Vn   = U - W S
        O    = (exp(G) * q) S + [(q k^T) * exp(G_i - G_j)]_{j<=i} Vn
        S   <- exp(G_C) S + (exp(G_C - G) * k)^T Vn
    Returns (o [B, T, Hv, dv], S [B, Hv, dk, dv]).
    """
    q, k, v, g, beta = (t.float() for t in (q, k, v, g, beta))
    if use_qk_l2norm:
        q, k = l2norm(q), l2norm(k)
    B, T, _, dk = q.shape
    Hv, dv = v.shape[2], v.shape[3]
    q, k = expand_heads(q, Hv), expand_heads(k, Hv)
    q = q * (dk ** -0.5 if scale is None else scale)
    pad = (-T) % chunk
    # [B, H, n, C, d]
    def to_chunks(x):
        x = x.transpose(1, 2)
        x = F.pad(x, (0, 0, 0, pad)) if x.dim() == 4 else F.pad(x, (0, pad))
        return x.reshape(B, Hv, -1, chunk, *x.shape[3:])
    qc, kc, vc = to_chunks(q), to_chunks(k), to_chunks(v)
    gc, bc = to_chunks(g), to_chunks(beta)
    G = gc.cumsum(-1)
    n = qc.shape[2]
    eye = torch.eye(chunk)
    strict = torch.tril(torch.ones(chunk, chunk, dtype=torch.bool), -1)
    causal = torch.tril(torch.ones(chunk, chunk, dtype=torch.bool), 0)
    diff = G[..., :, None] - G[..., None, :]
    decay = torch.where(causal, diff, torch.full_like(diff, -torch.inf)).exp()  # exp(G_i - G_j), j <= i
    kb = kc * bc[..., None]
    M = (kb @ kc.transpose(-1, -2)) * decay * strict
    Tm = torch.linalg.solve_triangular(eye + M, eye.expand_as(M), upper=False, unitriangular=True)
    U = Tm @ (vc * bc[..., None])
    W = Tm @ (kb * G.exp()[..., None])
    A = (qc @ kc.transpose(-1, -2)) * decay  # decay is zero above the diagonal
    S = torch.zeros(B, Hv, dk, dv) if initial_state is None else initial_state.float().clone()
    o = torch.empty(B, Hv, n, chunk, dv)
    for i in range(n):
        vn = U[:, :, i] - W[:, :, i] @ S
        o[:, :, i] = (qc[:, :, i] * G[:, :, i, :, None].exp()) @ S + A[:, :, i] @ vn
        gl = G[:, :, i, -1]
        S = S * gl.exp()[..., None, None] + (kc[:, :, i] * (gl[..., None] - G[:, :, i]).exp()[..., None]).transpose(-1, -2) @ vn
    o = o.reshape(B, Hv, n * chunk, dv)[:, :, :T].transpose(1, 2).contiguous()
    return o, S


# ------------------------------------------------------------------------------------------------
# The full layer
# ------------------------------------------------------------------------------------------------


@dataclass
class GDNWeights:
    """One layer's weights in HF layout, fp32 tensors holding bf16-representable values for the projections.

    w_qkv [2*kd + vd, hidden], w_z [vd, hidden], w_a [Hv, hidden], w_b [Hv, hidden], conv_w [conv_dim, K],
    a_log [Hv], dt_bias [Hv], norm_w [dv], w_out [hidden, vd].
    """

    w_qkv: torch.Tensor
    w_z: torch.Tensor
    w_a: torch.Tensor
    w_b: torch.Tensor
    conv_w: torch.Tensor
    a_log: torch.Tensor
    dt_bias: torch.Tensor
    norm_w: torch.Tensor
    w_out: torch.Tensor
    num_k_heads: int
    num_v_heads: int
    head_k_dim: int = 128
    head_v_dim: int = 128
    eps: float = 1e-6

    @property
    def hidden(self) -> int:
        return self.w_qkv.shape[1]

    @property
    def key_dim(self) -> int:
        return self.num_k_heads * self.head_k_dim

    @property
    def value_dim(self) -> int:
        return self.num_v_heads * self.head_v_dim

    @property
    def conv_dim(self) -> int:
        return 2 * self.key_dim + self.value_dim

    @property
    def conv_k(self) -> int:
        return self.conv_w.shape[1]

    @classmethod
    def from_hf(cls, layer) -> "GDNWeights":
        """Copy the weights of a HF ``Qwen3_5GatedDeltaNet`` (fp32 copies)."""
        f = lambda t: t.detach().float().clone()
        return cls(
            w_qkv=f(layer.in_proj_qkv.weight), w_z=f(layer.in_proj_z.weight), w_a=f(layer.in_proj_a.weight),
            w_b=f(layer.in_proj_b.weight), conv_w=f(layer.conv1d.weight[:, 0, :]), a_log=f(layer.A_log),
            dt_bias=f(layer.dt_bias), norm_w=f(layer.norm.weight), w_out=f(layer.out_proj.weight),
            num_k_heads=layer.num_k_heads, num_v_heads=layer.num_v_heads, head_k_dim=layer.head_k_dim,
            head_v_dim=layer.head_v_dim, eps=layer.norm.variance_epsilon,
        )


@dataclass
class LayerTrace:
    """Intermediates of one oracle layer call (for stage-by-stage checks)."""

    qkv_pre: torch.Tensor  # [B, T, conv_dim] in_proj output before the conv
    z: torch.Tensor  # [B, T, vd]
    g: torch.Tensor  # [B, T, Hv]
    beta: torch.Tensor  # [B, T, Hv]
    qkv: torch.Tensor  # [B, T, conv_dim] after conv + SiLU
    o: torch.Tensor  # [B, T, Hv, dv] recurrence output
    y: torch.Tensor  # [B, T, vd] gated RMSNorm output


def layer_forward(w: GDNWeights, x: torch.Tensor, rec_state=None, conv_state=None, mode: str = "recurrent",
                  chunk: int = 64, trace: bool = False, act_fp8: bool = False):
    """One GDN layer call that continues from (rec_state, conv_state), in fp32.

    x: [B, T, hidden].  mode "recurrent" runs the token-by-token rule, "chunk" the chunked form.
    Returns (out [B, T, hidden], new rec_state [B, Hv, dk, dv], new conv_state [B, K-1, conv_dim]
    [, LayerTrace]).  Same sequence of steps as HF ``Qwen3_5GatedDeltaNet.forward`` and the reference's
    ``Qwen35GatedDeltaNetTT._forward_rows`` (``9B/gdn_layer.py:244-280``).
    act_fp8: the projections' inputs are quantised per token to e4m3 (quantize_rows_e4m3; the out_proj
    input after rounding to bf16) -- the library's fp8 decode; pair it with fp8_weights(w).
    """
    x = x.float()
    x_in = quantize_rows_e4m3(x) if act_fp8 else x
    B, T, _ = x.shape
    kd, vd, Hk, Hv = w.key_dim, w.value_dim, w.num_k_heads, w.num_v_heads
    qkv_pre = x_in @ w.w_qkv.float().T
    z = x_in @ w.w_z.float().T
    a = x_in @ w.w_a.float().T
    b = x_in @ w.w_b.float().T
    qkv, new_conv = causal_conv1d(qkv_pre, w.conv_w, conv_state)
    q = qkv[..., :kd].reshape(B, T, Hk, w.head_k_dim)
    k = qkv[..., kd:2 * kd].reshape(B, T, Hk, w.head_k_dim)
    v = qkv[..., 2 * kd:].reshape(B, T, Hv, w.head_v_dim)
    g, beta = gating(a, b, w.a_log, w.dt_bias)
    if mode == "recurrent":
        o, S = recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=rec_state)
    elif mode == "chunk":
        o, S = chunk_gated_delta_rule(q, k, v, g, beta, initial_state=rec_state, chunk=chunk)
    else:
        raise ValueError(f"unknown mode {mode!r}")
    y = rmsnorm_gated(o, z.reshape(B, T, Hv, w.head_v_dim), w.norm_w, w.eps).reshape(B, T, vd)
    out = (quantize_rows_e4m3(bf16_round(y)) if act_fp8 else y) @ w.w_out.float().T
    if trace:
        return out, S, new_conv, LayerTrace(qkv_pre, z, g, beta, qkv, o, y)
    return out, S, new_conv


# ------------------------------------------------------------------------------------------------
# Conversions and synthetic inputs
# ------------------------------------------------------------------------------------------------


def hf_conv_state_to_abi(hf_state: torch.Tensor) -> torch.Tensor:
    """HF cache conv state [B, conv_dim, K] (last K inputs) -> [B, K-1, conv_dim] (last K-1 inputs)."""
    return hf_state[:, :, 1:].transpose(1, 2).contiguous().float()


def abi_conv_state_to_hf(state: torch.Tensor, oldest: torch.Tensor | None = None) -> torch.Tensor:
    """[B, K-1, conv_dim] -> HF [B, conv_dim, K]; the oldest column (never read again) is zero unless given."""
    B, km1, C = state.shape
    out = torch.zeros(B, C, km1 + 1)
    out[:, :, 1:] = state.transpose(1, 2)
    if oldest is not None:
        out[:, :, 0] = oldest
    return out


def bf16_round(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).float()


# ------------------------------------------------------------------------------------------------
# The decoder layer around the mixer (linear-attention layer type): input RMSNorm, GDN mixer, residual,
# post-mixer RMSNorm, SwiGLU MLP, residual -- HF transformers 5.5.0 ``Qwen3_5DecoderLayer.forward``,
# ``Qwen3_5RMSNorm`` and ``Qwen3_5MLP`` (modeling_qwen3_5.py).  The reference stacks GDN mixers only
# (0.8B/gdn_l1.py:295-325); its optimisation notes name these surroundings as the next step
# (0.8B/OPTIMIZATION.md:258-259).
# ------------------------------------------------------------------------------------------------


@dataclass
class DecoderWeights:
    """One linear-attention decoder layer: the GDN mixer's weights plus its surroundings (fp32 tensors;
    projections bf16-representable).  input_norm_w, post_norm_w [hidden] (applied as 1 + w);
    w_gate, w_up [intermediate, hidden]; w_down [hidden, intermediate]."""

    gdn: GDNWeights
    input_norm_w: torch.Tensor
    post_norm_w: torch.Tensor
    w_gate: torch.Tensor
    w_up: torch.Tensor
    w_down: torch.Tensor
    eps: float = 1e-6


def rmsnorm_offset(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """Qwen3_5RMSNorm: x * rsqrt(mean(x^2) + eps) * (1 + w), in fp32."""
    x = x.float()
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * (1.0 + w.float())


def swiglu_mlp(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor:
    """Qwen3_5MLP with hidden_act silu: down(silu(gate(x)) * up(x))."""
    return (F.silu(x @ w_gate.float().T) * (x @ w_up.float().T)) @ w_down.float().T


def decoder_layer_forward(dw: DecoderWeights, x: torch.Tensor, rec_state=None, conv_state=None,
                          mode: str = "recurrent", chunk: int = 64, bf16_acts: bool = False):
    """One decoder-layer call that continues from (rec_state, conv_state), in fp32; returns
    (out [B, T, hidden], new rec_state, new conv_state).

    bf16_acts: the activations between the steps are rounded to bf16 as a bf16 HF model stores them --
    ``Qwen3_5RMSNorm.forward`` casts its result back to the input dtype (``output.type_as(x)``), the mixer
    returns its out_proj output in that dtype and the residual sums of ``Qwen3_5DecoderLayer.forward`` run in
    it; the MLP's SiLU(gate) * up product is rounded before the down projection.  The recurrent state still
    evolves in fp32 from the rounded mixer input."""
    r = bf16_round if bf16_acts else (lambda t: t)
    x = x.float()
    mixed, S, conv = layer_forward(dw.gdn, r(rmsnorm_offset(x, dw.input_norm_w, dw.eps)), rec_state, conv_state,
                                   mode=mode, chunk=chunk)
    h = r(x + r(mixed))
    hn = r(rmsnorm_offset(h, dw.post_norm_w, dw.eps))
    act = r(F.silu(hn @ dw.w_gate.float().T) * (hn @ dw.w_up.float().T))
    out = h + act @ dw.w_down.float().T
    return out, S, conv


# ------------------------------------------------------------------------------------------------
# fp8 (e4m3) weights and activations: the library's fp8 mode, the B200 counterpart of the reference's
# block-float weight modes (weight_dtype=ttnn.bfloat8_b, 9B/gdn_layer.py:55,90-119; 0.8B/gdn_l1.py:155).
# ------------------------------------------------------------------------------------------------


def e4m3_scale(amax: torch.Tensor) -> torch.Tensor:
    """Per-row scale: the smallest power of two 2^e with amax / 2^e <= 448 (e4m3's largest finite value),
    read from the bits of the fp32 quotient amax / 448 (that value when it is a power of two, else the next
    power up; 2^-126 below the normal range); 1 where amax is 0."""
    v = (amax.float() / 448.0).contiguous()
    bits = v.view(torch.int32)
    ex = (bits >> 23) & 0xFF
    up = torch.where((bits & 0x7FFFFF) != 0, (ex + 1) << 23, bits)
    up = torch.where(ex == 0, torch.full_like(bits, 1 << 23), up)
    s = up.view(torch.float32)
    return torch.where(amax > 0, s, torch.ones_like(s))


def quantize_rows_e4m3(t: torch.Tensor) -> torch.Tensor:
    """Row-wise (last dim) e4m3 round trip with e4m3_scale: round-to-nearest-even e4m3 of t / scale, times
    the scale (exact: the scale is a power of two)."""
    t = t.float()
    s = e4m3_scale(t.abs().amax(dim=-1))[..., None]
    return (t / s).to(torch.float8_e4m3fn).float() * s


def fp8_weights(w: GDNWeights) -> GDNWeights:
    """The weights the library's fp8 mode computes with: every output row of the projections quantised by
    quantize_rows_e4m3 (conv taps, gates and norm weight unchanged)."""
    from dataclasses import replace

    return replace(w, w_qkv=quantize_rows_e4m3(w.w_qkv), w_z=quantize_rows_e4m3(w.w_z),
                   w_a=quantize_rows_e4m3(w.w_a), w_b=quantize_rows_e4m3(w.w_b), w_out=quantize_rows_e4m3(w.w_out))


def make_weights(hidden: int, num_k_heads: int, num_v_heads: int, head_dim: int = 128, conv_k: int = 4,
                 seed: int = 0, a_max: float = 16.0, std: float = 0.02) -> GDNWeights:
    """Synthetic layer weights with the benchmark's distributions, projections rounded to bf16.

    Projections ~ N(0, std); A_log = log(U(1, a_max)); dt_bias ~ N(0, 0.1); conv taps follow the
    PyTorch Conv1d default init U(-1/sqrt(K), 1/sqrt(K)) rounded to bf16 (the convention of
    ``0.8B/test_gdn_l1.py:50``); norm weight ~ U(0.5, 1.5) (``9B/test_gdn_layer.py:23``).
    """
    gen = torch.Generator().manual_seed(seed)
    kd, vd = num_k_heads * head_dim, num_v_heads * head_dim
    conv_dim = 2 * kd + vd
    rn = lambda *s: bf16_round(torch.randn(*s, generator=gen) * std)
    bound = 1.0 / conv_k ** 0.5
    return GDNWeights(
        w_qkv=rn(conv_dim, hidden), w_z=rn(vd, hidden), w_a=rn(num_v_heads, hidden), w_b=rn(num_v_heads, hidden),
        conv_w=bf16_round((torch.rand(conv_dim, conv_k, generator=gen) * 2 - 1) * bound),
        a_log=torch.log(1.0 + torch.rand(num_v_heads, generator=gen) * (a_max - 1.0)),
        dt_bias=torch.randn(num_v_heads, generator=gen) * 0.1,
        norm_w=0.5 + torch.rand(head_dim, generator=gen),
        w_out=rn(hidden, vd), num_k_heads=num_k_heads, num_v_heads=num_v_heads,
        head_k_dim=head_dim, head_v_dim=head_dim,
    )


def make_hidden(B: int, T: int, hidden: int, seed: int = 0) -> torch.Tensor:
    """x ~ N(0, 1) rounded to bf16, as fp32."""
    gen = torch.Generator().manual_seed(seed)
    return bf16_round(torch.randn(B, T, hidden, generator=gen))


def make_recurrence_inputs(B, T, Hk, Hv, dk=128, dv=128, seed=0, decay_shift=2.0):
    """q, k, v ~ N(0,1); g = logsigmoid(N(0,1) + shift); beta = sigmoid(N(0,1))
    (``9B/test_gated_delta_l1.py:17-24``)."""
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, Hk, dk, generator=gen)
    k = torch.randn(B, T, Hk, dk, generator=gen)
    v = torch.randn(B, T, Hv, dv, generator=gen)
    g = F.logsigmoid(torch.randn(B, T, Hv, generator=gen) + decay_shift)
    beta = torch.sigmoid(torch.randn(B, T, Hv, generator=gen))
    return q, k, v, g, beta


# ------------------------------------------------------------------------------------------------
# Metrics
# ------------------------------------------------------------------------------------------------


def max_abs_rel(got: torch.Tensor, want: torch.Tensor) -> float:
    """max|got - want| / max|want| -- the tolerance metric of the benchmark spec."""
    got, want = got.double(), want.double()
    return ((got - want).abs().max() / want.abs().max().clamp_min(1e-30)).item()


def rel_fro(got: torch.Tensor, want: torch.Tensor) -> float:
    """||got - want||_F / ||want||_F (``9B/test_gdn_layer.py:35-39``)."""
    got, want = got.double(), want.double()
    return ((got - want).norm() / want.norm().clamp_min(1e-30)).item()


def pcc(got: torch.Tensor, want: torch.Tensor) -> float:
    """Pearson correlation (``9B/test_gdn_layer.py:31-32``)."""
    return torch.corrcoef(torch.stack([got.flatten().double(), want.flatten().double()]))[0, 1].item()
