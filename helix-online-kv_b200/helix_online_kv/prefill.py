"""Exact multi-token attention on the tensor cores (hokv_prefill_attention).

The reference's cache hands exact K/V to the model's own attention for every
prefill and for the layers it keeps exact (compressed_cache.py:72-105).  This
module is that attention as one CUDA launch per layer: causal (query i at
position kv_len - q_len + i) or full, grouped-query heads read from their
shared KV head, f16/bf16, head_dim 64 or 128, (batch, head, token) strides that
nest (any permutation of a packed layout, or a slice of one: the CDC-03 store's
views and the transposed projections a model passes need no copy), contiguous
head dims, key and value with the same strides.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib as L

_DTYPES = {torch.float16: L.F16, torch.bfloat16: L.BF16}


def supported(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor) -> bool:
    """True when hokv_prefill_attention takes these tensors as they are."""
    if query.dtype not in _DTYPES or key.dtype != query.dtype or value.dtype != query.dtype:
        return False
    if query.dim() != 4 or key.dim() != 4 or value.dim() != 4 or query.shape[-1] not in (64, 128):
        return False
    if key.shape != value.shape or key.shape[-1] != query.shape[-1] or query.shape[0] != key.shape[0]:
        return False
    if query.shape[1] % key.shape[1] != 0:
        return False
    for t in (query, key, value):
        if not t.is_cuda or t.stride(-1) != 1 or t.data_ptr() % 16 or any(s % 8 for s in t.stride()[:3]):
            return False
        if not _nests(t):
            return False
    return key.stride() == value.stride()


def _nests(t: torch.Tensor) -> bool:
    """The (token, head, batch) dims, in ascending stride order, each cover the
    dims inside them (the tensor maps the kernel loads through need this;
    dims of extent 1 always fit)."""
    dims = sorted(((t.stride(i), t.shape[i]) for i in (2, 1, 0) if t.shape[i] > 1))
    need = t.shape[3]
    for stride, extent in dims:
        if stride < need:
            return False
        need = stride * extent
    return True


def prefill_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, scaling: Optional[float] = None,
                      is_causal: bool = True, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """softmax(query key^T * scaling [causal]) value.

    query [B, H_q, q_len, D], key/value [B, H_kv, kv_len, D] (H_q a multiple of
    H_kv) -> [B, q_len, H_q, D] (the layout a Hugging Face attention function
    returns), in the query's dtype."""
    if not supported(query, key, value):
        raise ValueError(f"Expected f16/bf16 CUDA tensors [B, H, S, 64|128] with contiguous head dims and "
                         f"strides in multiples of 8 elements, got {tuple(query.shape)} {query.dtype}, "
                         f"{tuple(key.shape)} {key.dtype}")
    B, Hq, Sq, D = query.shape
    Hkv, Skv = key.shape[1], key.shape[2]
    if is_causal and Skv < Sq:
        raise ValueError(f"causal attention needs kv_len >= q_len, got {Skv} < {Sq}")
    scale = float(scaling) if scaling is not None else D ** -0.5
    if out is None:
        out = torch.empty((B, Sq, Hq, D), dtype=query.dtype, device=query.device)
    elif out.shape != (B, Sq, Hq, D) or out.dtype != query.dtype or out.stride(-1) != 1:
        raise ValueError(f"Expected out [{B}, {Sq}, {Hq}, {D}] {query.dtype}, got {tuple(out.shape)} {out.dtype}")
    lib = L.lib()
    L.check(lib.hokv_prefill_attention(
        L.ptr(query), L.ptr(key), L.ptr(value), L.ptr(out), _DTYPES[query.dtype], B, Hq, Hkv, Sq, Skv, D,
        query.stride(0), query.stride(1), query.stride(2), key.stride(0), key.stride(1), key.stride(2),
        value.stride(0), value.stride(1), value.stride(2), out.stride(0), out.stride(2), out.stride(1),
        scale, 1 if is_causal else 0, L.stream()), "prefill_attention")
    return out
