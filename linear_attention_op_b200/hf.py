"""Hugging Face integration: route ``Qwen3_5GatedDeltaNet.forward`` through the B200 library.

``patch_gated_deltanet(module)`` replaces one module's ``forward`` (the one the reference's layer op is checked
against, 9B/test_gdn_layer.py:19-47); ``patch_model(model)`` does it for every GDN layer of a model.  The
patched forward keeps HF's semantics and cache protocol (transformers ``LinearAttentionLayer``):

* ``cache_params`` absent or without previous state, or T > 1: a prefill from zero state (HF passes
  ``initial_state=None`` to its chunked rule); with a cache, the final recurrent state and the conv window
  are stored through ``update_recurrent_state`` / ``update_conv_state`` as HF does;
* cached decode (previous state, T == 1): continues from the cache's recurrent state and conv window and
  writes both back in place.

HF's conv cache keeps the last K = 4 pre-conv inputs per channel, ``[B, conv_dim, 4]``; the library keeps the
last K - 1 = 3, ``[B, 3, conv_dim]`` (the reference's layout, 9B/kernels/layer_reader.cpp:184-197).  The
oldest of HF's four columns is never read by its update; after a prefill through this shim it holds zeros,
after a decode step the previous window's second column (exactly what HF stores).

The module may live on the CPU (as in the reference's tests); inputs and states move to the layer's GPU for
the call and back.  Errors raise ``GDNError``; there is no CPU path.
"""

from __future__ import annotations

import torch

from ._lib import call
from .gdn_layer import WEIGHT_FORMATS, LayerWeights, _LayerHandle


class _PatchedGDN:
    def __init__(self, module, device, weight_dtype: str = "bf16"):
        if weight_dtype not in WEIGHT_FORMATS:
            raise ValueError(f"weight_dtype must be one of {sorted(WEIGHT_FORMATS)}")
        self.module = module
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.layer_idx = getattr(module, "layer_idx", 0)
        with torch.cuda.device(self.device):
            self.handle = _LayerHandle(LayerWeights.from_hf(module))
            if weight_dtype != "bf16":
                call("gdn_layer_set_weight_format", self.handle.handle, WEIGHT_FORMATS[weight_dtype])
        info = self.handle.info
        self.hv, self.conv_dim = info.num_v_heads_local, info.conv_dim_local
        self.hidden = info.hidden

    def __call__(self, hidden_states: torch.Tensor, cache_params=None, attention_mask=None):
        from transformers.models.qwen3_5.modeling_qwen3_5 import apply_mask_to_padding_states

        hidden_states = apply_mask_to_padding_states(hidden_states, attention_mask)
        B, T, H = hidden_states.shape
        dev, idx = self.device, self.layer_idx
        decode = cache_params is not None and cache_params.has_previous_state(idx) and T == 1
        with torch.cuda.device(dev):
            x = hidden_states.to(device=dev, dtype=torch.bfloat16).contiguous()
            out = torch.empty_like(x)
            if decode:
                layer = cache_params.layers[idx]
                rec = layer.recurrent_states.to(device=dev, dtype=torch.float32).contiguous()
                window = layer.conv_states.to(device=dev, dtype=torch.float32)
                conv = window[:, :, 1:].transpose(1, 2).contiguous()
            else:
                rec = torch.zeros(B, self.hv, 128, 128, dtype=torch.float32, device=dev)
                conv = torch.zeros(B, 3, self.conv_dim, dtype=torch.float32, device=dev)
            self.handle.forward(x, B, T, rec, conv, out)
            if cache_params is not None:
                if decode:
                    new_window = torch.cat([window[:, :, 1:2], conv.transpose(1, 2)], dim=2)
                    layer.conv_states.copy_(new_window.to(layer.conv_states.device, layer.conv_states.dtype))
                    layer.recurrent_states.copy_(rec.to(layer.recurrent_states.device, layer.recurrent_states.dtype))
                else:
                    new_window = torch.cat([torch.zeros_like(conv[:, :1]), conv], dim=1).transpose(1, 2)
                    cache_params.update_conv_state(new_window.to(hidden_states.device, hidden_states.dtype), idx)
                    cache_params.update_recurrent_state(rec.to(hidden_states.device), idx)
        return out.to(device=hidden_states.device, dtype=hidden_states.dtype)


def patch_gated_deltanet(module, device=None, weight_dtype: str = "bf16"):
    """Make ``module`` (a HF ``Qwen3_5GatedDeltaNet``) run on the B200 library; returns the module.
    weight_dtype "fp8": the library's e4m3 weight mode (see Qwen35GatedDeltaNet)."""
    module._gdn_b200 = _PatchedGDN(module, device, weight_dtype)
    module.forward = module._gdn_b200
    return module


def patch_model(model, device=None, weight_dtype: str = "bf16") -> int:
    """Patch every ``Qwen3_5GatedDeltaNet`` inside ``model``; returns how many were patched."""
    n = 0
    for m in model.modules():
        if type(m).__name__ == "Qwen3_5GatedDeltaNet" and not hasattr(m, "_gdn_b200"):
            patch_gated_deltanet(m, device, weight_dtype)
            n += 1
    return n
