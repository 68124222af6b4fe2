"""Fused scalar-VQ Q.K^T without materialising K (Path A).

Drop-in for the reference module (helix_online_kv/triton_attention.py).  The
reference compiles a Triton kernel; this build calls the hand-written sm_100a
kernel ``k_scalar_vq_qkt`` of libhokv instead, which reads uint8 (or int32)
indices directly -- no int32 copy -- and looks them up in a codebook held 32
times in shared memory so that lookups never bank-conflict.

``_HAS_TRITON`` keeps its name for callers that test it: it is True when the
fused device kernel is available (CUDA device + built library).
"""

from __future__ import annotations

import numpy as np

from . import _lib as L

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None

_HAS_TRITON = L.available()


def fused_scalar_vq_qkt(q, k_indices, codebook, scale: float, block_t: int = 64):
    """(q @ K_reconstructed.T) * scale on the device (triton_attention.py:69-120).

    Args:
        q: [head_dim] float32 CUDA tensor.
        k_indices: [seq_len, head_dim] uint8 or int32 CUDA tensor.
        codebook: [256] float32 CUDA tensor.
        scale: attention scale.
        block_t: accepted for compatibility (the CUDA kernel sizes its own blocks).

    Returns:
        [seq_len] float32 CUDA tensor.
    """
    assert q.is_cuda, "q must be on CUDA"
    assert k_indices.is_cuda, "k_indices must be on CUDA"
    assert codebook.is_cuda, "codebook must be on CUDA"
    seq_len, head_dim = k_indices.shape
    q = q.contiguous().float()
    codebook = codebook.contiguous().float()
    if k_indices.dtype not in (torch.uint8, torch.int32):
        k_indices = k_indices.to(torch.int32)
    k_indices = k_indices.contiguous()
    scores = torch.empty(seq_len, dtype=torch.float32, device=q.device)
    L.check(L.lib().hokv_scalar_vq_qkt(L.ptr(q), L.ptr(k_indices), L.dtype_code(k_indices), seq_len, head_dim,
                                       k_indices.stride(0), L.ptr(codebook), min(codebook.numel(), 256),
                                       float(scale), 0, L.ptr(scores), L.stream()), "scalar_vq_qkt")
    return scores


def fused_scalar_vq_qkt_numpy(q, k_indices, codebook, scale: float):
    """NumPy-facing form (triton_attention.py:123-141): same kernel, f64 accumulation.

    Returns [seq_len] float32 NumPy array.
    """
    L.require_device()
    idx = np.asarray(k_indices)
    it = torch.uint8 if idx.dtype == np.uint8 else torch.int32
    qd = L.to_dev(np.asarray(q, dtype=np.float32).ravel())
    idd = L.to_dev(idx, it)
    cb = L.to_dev(np.asarray(codebook, dtype=np.float32).ravel())
    seq_len, head_dim = idx.shape
    scores = torch.empty(seq_len, dtype=torch.float32, device=qd.device)
    L.check(L.lib().hokv_scalar_vq_qkt(L.ptr(qd), L.ptr(idd), L.dtype_code(idd), seq_len, head_dim, head_dim,
                                       L.ptr(cb), min(cb.numel(), 256), float(scale), 1, L.ptr(scores), L.stream()),
            "scalar_vq_qkt")
    L.device_status()
    return scores.cpu().numpy()
