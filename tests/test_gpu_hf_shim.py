"""The Hugging Face integration shim: a patched ``Qwen3_5GatedDeltaNet`` (module on the CPU, as the
reference's tests keep it) against the unpatched module on the same inputs, through HF's own cache --
prefill, cached decode, and the cache contents (9B/test_gdn_layer.py:42-73 is the reference's check of the
same boundary)."""
import copy

import pytest
import torch

from tests._util import OUT_TOL, STATE_TOL, check, requires_b200

pytestmark = [pytest.mark.gpu, requires_b200]


def _hf_layer():
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5GatedDeltaNet

    cfg = Qwen3_5TextConfig(hidden_size=256, linear_num_key_heads=2, linear_num_value_heads=4,
                            linear_key_head_dim=128, linear_value_head_dim=128, linear_conv_kernel_dim=4,
                            rms_norm_eps=1e-6, num_hidden_layers=1)
    from transformers.models.qwen3_5 import modeling_qwen3_5 as hf

    torch.manual_seed(3)
    L = Qwen3_5GatedDeltaNet(cfg, layer_idx=0).eval()
    # HF's own torch path (the one the reference's tests run): with a GPU present transformers picks the
    # flash-linear-attention kernels (conv, delta rule, gated norm), which do not take CPU tensors.
    L.causal_conv1d_fn = None
    L.causal_conv1d_update = hf.torch_causal_conv1d_update
    L.chunk_gated_delta_rule = hf.torch_chunk_gated_delta_rule
    L.recurrent_gated_delta_rule = hf.torch_recurrent_gated_delta_rule
    if not isinstance(L.norm, hf.Qwen3_5RMSNormGated):  # the fused norm is a Triton kernel too
        norm = hf.Qwen3_5RMSNormGated(L.head_v_dim, eps=cfg.rms_norm_eps)
        norm.weight.data.copy_(L.norm.weight.data)
        L.norm = norm
    with torch.no_grad():
        L.norm.weight.uniform_(0.5, 1.5)
        L.dt_bias.uniform_(-1.0, 1.0)
        for lin in (L.in_proj_qkv, L.in_proj_z, L.in_proj_a, L.in_proj_b, L.out_proj):
            lin.weight.copy_(lin.weight.bfloat16().float())
        L.conv1d.weight.copy_(L.conv1d.weight.bfloat16().float())
    return cfg, L


def test_patched_module_matches_hf_with_cache():
    from transformers.cache_utils import DynamicCache

    from linear_attention_op_b200.hf import patch_gated_deltanet, patch_model

    cfg, ref = _hf_layer()
    ours = patch_gated_deltanet(copy.deepcopy(ref))
    gen = torch.Generator().manual_seed(4)
    B, T0, steps = 2, 37, 4
    x = torch.randn(B, T0 + steps, 256, generator=gen).bfloat16().float()
    with torch.no_grad():
        c_ref, c_ours = DynamicCache(config=cfg), DynamicCache(config=cfg)
        check("prefill", ours(x[:, :T0], cache_params=c_ours), ref(x[:, :T0], cache_params=c_ref), OUT_TOL)
        for t in range(T0, T0 + steps):
            check(f"decode {t}", ours(x[:, t:t + 1], cache_params=c_ours), ref(x[:, t:t + 1], cache_params=c_ref),
                  OUT_TOL)
        check("recurrent cache", c_ours.layers[0].recurrent_states, c_ref.layers[0].recurrent_states, STATE_TOL)
        check("conv cache (the columns HF reads)", c_ours.layers[0].conv_states[:, :, 1:],
              c_ref.layers[0].conv_states[:, :, 1:], 1e-4)
        check("no cache", ours(x), ref(x), OUT_TOL)
    assert patch_model(torch.nn.ModuleList([copy.deepcopy(ref), ours])) == 1  # the patched one is skipped
