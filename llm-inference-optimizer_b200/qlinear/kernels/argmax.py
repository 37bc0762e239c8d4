"""Row-wise argmax of fp16 logits through packed 64-bit keys (libqlinear).

The reference's engines take ``argmax`` of the lm_head's logits for greedy
decoding (src/engine/paged_engine.py:146-147, 202-203;
src/engine/graphed_decode_engine.py:114-115).  ``argmax_keys`` reduces each
row to one key ``(ord(value) << 32) | (0xFFFFFFFF - column)``; keys of
column shards combine with a max, so a sharded lm_head exchanges 8 bytes per
row and rank instead of its logits.  Ties resolve to the smallest column,
as ``torch.argmax`` does.
"""
from __future__ import annotations

import torch

from .. import _lib
from ._launch import ld, on_device

_SIGN = -(1 << 63)          # bit 63 as an int64


def argmax_keys(logits: torch.Tensor, col_offset: int = 0) -> torch.Tensor:
    """logits fp16 [M, N] (CUDA, unit inner stride) -> int64 [M] raw key bits."""
    assert logits.is_cuda and logits.dtype == torch.float16 and logits.dim() == 2
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    M, N = logits.shape
    keys = torch.empty(M, dtype=torch.int64, device=logits.device)
    if M == 0:
        return keys
    with on_device(logits.device):
        stream = torch.cuda.current_stream(logits.device)
        st = _lib.load().ql_argmax_rows_f16(logits.data_ptr(), M, N, ld(logits, N), col_offset, keys.data_ptr(),
                                            stream.cuda_stream)
    _lib.check(st)
    return keys


def combine_keys(keys: torch.Tensor, dim: int = 0) -> torch.Tensor:
    """Max of raw (unsigned) key bits along `dim` (torch compares int64 as
    signed, so bit 63 is flipped around the max)."""
    return (keys ^ _SIGN).amax(dim=dim) ^ _SIGN


def key_columns(keys: torch.Tensor) -> torch.Tensor:
    """Column index held by each key (int64)."""
    return 0xFFFFFFFF - (keys & 0xFFFFFFFF)


def key_values(keys: torch.Tensor) -> torch.Tensor:
    """fp16 value held by each key."""
    ordv = (keys >> 32) & 0xFFFF
    bits = torch.where(ordv >= 0x8000, ordv - 0x8000, 0xFFFF - ordv)
    return bits.to(torch.int32).to(torch.int16).view(torch.float16)


def argmax_f16(logits: torch.Tensor) -> torch.Tensor:
    """torch.argmax(logits, dim=-1) for fp16 CUDA logits of any leading shape."""
    N = logits.shape[-1]
    keys = argmax_keys(logits.reshape(-1, N))
    return key_columns(keys).reshape(logits.shape[:-1])


__all__ = ["argmax_keys", "combine_keys", "key_columns", "key_values", "argmax_f16"]
