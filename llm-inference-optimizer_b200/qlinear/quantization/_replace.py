"""Module replacement shared by the INT8 and INT4 quantizers.

The reference's engines fetch each projection from its parent module on
every call (``src/engine/paged_engine.py:98-105``,
``src/engine/graphed_decode_engine.py:81,105,110``), so swapping the
``nn.Linear`` objects under ``model.model.layers`` for quantized modules is
the whole integration: nothing else in the model or the engines changes.
The statistics returned are those of ``quantize_model_int8`` /
``quantize_model_int4`` (``src/quantization/int8.py:73-100``,
``src/quantization/int4.py:72-97``).
"""
from __future__ import annotations

import gc
from typing import Callable

import torch
import torch.nn as nn


def tensor_bytes(*tensors) -> int:
    """Storage bytes of the given tensors; None entries count as zero."""
    return sum(t.numel() * t.element_size() for t in tensors if t is not None)


def replace_linears(model: nn.Module, quantize: Callable[[nn.Linear], nn.Module]) -> dict:
    """Swap every ``nn.Linear`` found below ``model.model.layers`` for
    ``quantize(linear)``.  The embeddings and the lm_head sit outside the
    decoder layers and are left alone.

    Returns ``{"layers_quantized", "bytes_before", "bytes_after"}``: how many
    projections were swapped, their dense weight + bias bytes, and the bytes
    of the modules that replaced them (``num_bytes()``).  A result of zero
    layers means the model did not have the expected layout."""
    sites = [(owner, attr, mod)
             for owner in model.model.layers.modules()
             for attr, mod in owner.named_children()
             if isinstance(mod, nn.Linear)]
    dense = packed = 0
    for owner, attr, mod in sites:
        dense += tensor_bytes(mod.weight, mod.bias)
        q = quantize(mod)
        packed += q.num_bytes()
        setattr(owner, attr, q)
    swapped = len(sites)
    sites = owner = mod = q = None   # drop the last references to the dense layers
    # the fp16 weights just dropped are released back to the device
    gc.collect()
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    return {"layers_quantized": swapped, "bytes_before": dense, "bytes_after": packed}
