"""Generate the golden fixtures that pin the CPU oracle to the reference's own CPU code.

Run in the build container, where the reference checkout and Hugging Face transformers 5.5.0 are present:

    python tests/golden/make_golden.py --reference-dir <checkout>/wormhole_n150/qwen3.5_9B

Sources of truth (nothing here is re-implemented; every expected value comes from the reference's code):

* ``recurrence_ref.npz`` -- ``wormhole_n150/qwen3.5_9B/reference.py::recurrent_gated_delta_rule`` (imported
  from the reference checkout) on the input recipe of ``9B/test_gated_delta_l1.py:17-24,60-61``;
* ``chunk_hf.npz`` -- HF ``torch_chunk_gated_delta_rule`` (the prefill path every reference layer test
  compares against) with ``output_final_state=True``;
* ``layer_hf.npz`` -- HF ``Qwen3_5GatedDeltaNet`` (torch fallback path, fp32) built the way
  ``9B/test_gdn_layer.py:19-28`` builds it (bf16-rounded projections, norm weight U(0.5, 1.5), dt_bias
  U(-1, 1)), at a small geometry with the Qwen3.5 head size (dk = dv = 128): a 2-sequence 40-token prefill
  followed by 3 cached decode steps, plus a one-token call;
* ``decoder_hf.npz`` -- HF ``Qwen3_5DecoderLayer`` of the linear-attention type (input RMSNorm, the GDN mixer,
  residual, post-mixer RMSNorm, SwiGLU MLP, residual) at the same geometry with a 512-wide MLP: a 2-sequence
  40-token prefill followed by 3 cached decode steps.  The reference stacks GDN mixers only; these are the
  surroundings its optimisation notes name as the next step (0.8B/OPTIMIZATION.md:258-259).

The fixtures are small (< 2 MB together) and committed; the GPU box never needs the reference checkout.
"""

from __future__ import annotations

import argparse
import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def load_reference_module(ref_dir: str):
    spec = importlib.util.spec_from_file_location("gdn_reference_py", Path(ref_dir) / "reference.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().contiguous().numpy()


def recurrence_cases(ref) -> dict:
    out = {}
    cases = [("a", 1, 2, 4, 45, True, 0), ("b", 2, 1, 2, 7, False, 1)]
    for name, B, Hk, Hv, T, with_init, seed in cases:
        gen = torch.Generator().manual_seed(seed)
        q = torch.randn(B, T, Hk, 128, generator=gen)
        k = torch.randn(B, T, Hk, 128, generator=gen)
        v = torch.randn(B, T, Hv, 128, generator=gen)
        g = torch.nn.functional.logsigmoid(torch.randn(B, T, Hv, generator=gen) + 2.0)
        beta = torch.sigmoid(torch.randn(B, T, Hv, generator=gen))
        init = torch.randn(B, Hv, 128, 128, generator=gen) * 0.1 if with_init else None
        o, s = ref.recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=init)
        for key, val in dict(q=q, k=k, v=v, g=g, beta=beta, o=o, state=s).items():
            out[f"{name}_{key}"] = f32(val)
        out[f"{name}_init"] = f32(init) if init is not None else np.zeros((0,), np.float32)
    return out


def chunk_case() -> dict:
    from transformers.models.qwen3_5.modeling_qwen3_5 import torch_chunk_gated_delta_rule

    gen = torch.Generator().manual_seed(5)
    B, T, H = 1, 100, 2
    q = torch.randn(B, T, H, 128, generator=gen)
    k = torch.randn(B, T, H, 128, generator=gen)
    v = torch.randn(B, T, H, 128, generator=gen)
    g = torch.nn.functional.logsigmoid(torch.randn(B, T, H, generator=gen) + 2.0)
    beta = torch.sigmoid(torch.randn(B, T, H, generator=gen))
    o, s = torch_chunk_gated_delta_rule(q, k, v, g, beta, chunk_size=64, initial_state=None,
                                        output_final_state=True, use_qk_l2norm_in_kernel=True)
    return dict(q=f32(q), k=f32(k), v=f32(v), g=f32(g), beta=f32(beta), o=f32(o), state=f32(s))


def layer_case() -> dict:
    from transformers.cache_utils import DynamicCache
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5GatedDeltaNet

    cfg = Qwen3_5TextConfig(hidden_size=256, linear_num_key_heads=2, linear_num_value_heads=4,
                            linear_key_head_dim=128, linear_value_head_dim=128, linear_conv_kernel_dim=4,
                            rms_norm_eps=1e-6, num_hidden_layers=1)
    torch.manual_seed(0)
    L = Qwen3_5GatedDeltaNet(cfg, layer_idx=0).eval()
    with torch.no_grad():
        L.norm.weight.uniform_(0.5, 1.5)
        L.dt_bias.uniform_(-1.0, 1.0)
        for lin in (L.in_proj_qkv, L.in_proj_z, L.in_proj_a, L.in_proj_b, L.out_proj):
            lin.weight.copy_(lin.weight.bfloat16().float())
        L.conv1d.weight.copy_(L.conv1d.weight.bfloat16().float())
    gen = torch.Generator().manual_seed(1)
    B, T0, steps = 2, 40, 3
    x = torch.randn(B, T0 + steps, 256, generator=gen).bfloat16().float()
    x1 = torch.randn(1, 1, 256, generator=gen).bfloat16().float()
    with torch.no_grad():
        cache = DynamicCache(config=cfg)
        y_pre = L(x[:, :T0], cache_params=cache)
        conv_pre = cache.layers[0].conv_states.clone()
        rec_pre = cache.layers[0].recurrent_states.clone()
        y_dec = [L(x[:, t:t + 1], cache_params=cache) for t in range(T0, T0 + steps)]
        conv_dec = cache.layers[0].conv_states.clone()
        rec_dec = cache.layers[0].recurrent_states.clone()
        y_full = L(x)  # one-shot, no cache: the chunked path over all 43 tokens
        y_one = L(x1)
    bf = lambda t: t.detach().to(torch.bfloat16).view(torch.int16).numpy()
    return dict(
        w_qkv=bf(L.in_proj_qkv.weight), w_z=bf(L.in_proj_z.weight), w_a=bf(L.in_proj_a.weight),
        w_b=bf(L.in_proj_b.weight), w_out=bf(L.out_proj.weight), conv_w=f32(L.conv1d.weight[:, 0, :]),
        a_log=f32(L.A_log), dt_bias=f32(L.dt_bias), norm_w=f32(L.norm.weight),
        dims=np.array([256, 2, 4, 128, 128, 4], np.int32), x=f32(x), x1=f32(x1),
        y_pre=f32(y_pre), conv_pre=f32(conv_pre), rec_pre=f32(rec_pre), y_dec=f32(torch.cat(y_dec, 1)),
        conv_dec=f32(conv_dec), rec_dec=f32(rec_dec), y_full=f32(y_full), y_one=f32(y_one),
        t0=np.array([T0], np.int32),
    )


def decoder_case() -> dict:
    from transformers.cache_utils import DynamicCache
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5DecoderLayer

    cfg = Qwen3_5TextConfig(hidden_size=256, linear_num_key_heads=2, linear_num_value_heads=4,
                            linear_key_head_dim=128, linear_value_head_dim=128, linear_conv_kernel_dim=4,
                            rms_norm_eps=1e-6, num_hidden_layers=1, intermediate_size=512)
    assert cfg.layer_types == ["linear_attention"] and cfg.hidden_act == "silu"
    torch.manual_seed(2)
    D = Qwen3_5DecoderLayer(cfg, layer_idx=0).eval()
    L = D.linear_attn
    with torch.no_grad():
        L.norm.weight.uniform_(0.5, 1.5)
        L.dt_bias.uniform_(-1.0, 1.0)
        D.input_layernorm.weight.uniform_(-0.5, 0.5)  # applied as (1 + w)
        D.post_attention_layernorm.weight.uniform_(-0.5, 0.5)
        for lin in (L.in_proj_qkv, L.in_proj_z, L.in_proj_a, L.in_proj_b, L.out_proj, D.mlp.gate_proj,
                    D.mlp.up_proj, D.mlp.down_proj):
            lin.weight.copy_(lin.weight.bfloat16().float())
        L.conv1d.weight.copy_(L.conv1d.weight.bfloat16().float())
    gen = torch.Generator().manual_seed(3)
    B, T0, steps = 2, 40, 3
    x = torch.randn(B, T0 + steps, 256, generator=gen).bfloat16().float()
    with torch.no_grad():
        cache = DynamicCache(config=cfg)
        y_pre = D(x[:, :T0], position_embeddings=None, past_key_values=cache)
        y_dec = [D(x[:, t:t + 1], position_embeddings=None, past_key_values=cache) for t in range(T0, T0 + steps)]
        conv_dec = cache.layers[0].conv_states.clone()
        rec_dec = cache.layers[0].recurrent_states.clone()
    bf = lambda t: t.detach().to(torch.bfloat16).view(torch.int16).numpy()
    return dict(
        w_qkv=bf(L.in_proj_qkv.weight), w_z=bf(L.in_proj_z.weight), w_a=bf(L.in_proj_a.weight),
        w_b=bf(L.in_proj_b.weight), w_out=bf(L.out_proj.weight), conv_w=f32(L.conv1d.weight[:, 0, :]),
        a_log=f32(L.A_log), dt_bias=f32(L.dt_bias), norm_w=f32(L.norm.weight),
        dims=np.array([256, 2, 4, 128, 128, 4], np.int32),
        input_norm_w=f32(D.input_layernorm.weight), post_norm_w=f32(D.post_attention_layernorm.weight),
        w_gate=bf(D.mlp.gate_proj.weight), w_up=bf(D.mlp.up_proj.weight), w_down=bf(D.mlp.down_proj.weight),
        x=f32(x), y_pre=f32(y_pre), y_dec=f32(torch.cat(y_dec, 1)), conv_dec=f32(conv_dec),
        rec_dec=f32(rec_dec), t0=np.array([T0], np.int32),
    )


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-dir", required=True,
                    help="the reference checkout's wormhole_n150/qwen3.5_9B directory (holds reference.py)")
    ap.add_argument("--only", choices=["recurrence", "chunk", "layer", "decoder"], default=None,
                    help="regenerate one fixture only (the others keep their committed bytes)")
    args = ap.parse_args(argv)
    torch.set_num_threads(max(1, torch.get_num_threads()))
    ref = load_reference_module(args.reference_dir)
    if args.only in (None, "recurrence"):
        np.savez_compressed(HERE / "recurrence_ref.npz", **recurrence_cases(ref))
    if args.only in (None, "chunk"):
        np.savez_compressed(HERE / "chunk_hf.npz", **chunk_case())
    if args.only in (None, "layer"):
        np.savez_compressed(HERE / "layer_hf.npz", **layer_case())
    if args.only in (None, "decoder"):
        np.savez_compressed(HERE / "decoder_hf.npz", **decoder_case())
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    sys.exit(main())
