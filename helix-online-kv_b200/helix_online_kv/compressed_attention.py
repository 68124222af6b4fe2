"""Compressed-domain attention, single head and single query (NumPy in/out).

Drop-in for the reference module (helix_online_kv/compressed_attention.py):
the same functions, arguments, return values and NumPy dtype rules (a Python
float scale keeps float32 scores, a NumPy float64 scale promotes them).  Every
path runs on the device through libhokv; Path G (``hybrid_pq_attention``,
CDC-03) uses the same kernels as the batched decode in ``cdc03.py``.
Batched multi-head decode lives in ``cdc03.CDC03Store``.
"""

from __future__ import annotations

import numpy as np

from . import _lib as L

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None


def _f32(a):
    return L.to_dev(np.asarray(a, dtype=np.float32))


def _u8(a):
    return L.to_dev(np.asarray(a), torch.uint8)


def _score_dtype(scale, *arrays):
    """dtype NumPy gives ``(q @ K.T) * scale`` for these operands."""
    base = np.result_type(*[np.asarray(a).dtype for a in arrays]) if arrays else np.dtype(np.float32)
    return np.result_type(base, scale)


def _softmax_dev(s):
    """scipy.special.softmax of a CUDA f32/f64 vector (compressed_attention.py:31-33)."""
    out = torch.empty_like(s)
    L.check(L.lib().hokv_softmax(L.ptr(s), int(s.dtype == torch.float64), s.numel(), L.ptr(out), None, 0,
                                 L.stream()), "softmax")
    return out


def _softmax(x):
    """Numerically stable softmax (compressed_attention.py:31-33)."""
    L.require_device()
    arr = np.asarray(x)
    dt = torch.float64 if arr.dtype == np.float64 else torch.float32
    return _softmax_dev(L.to_dev(arr, dt)).cpu().numpy()


def _dense(q, K, V, scale, mask=None, scores_f32=False, out_f32=False):
    L.require_device()
    sdt = _score_dtype(scale, q, K)
    f64 = sdt == np.float64
    mul_f64 = f64 or isinstance(scale, (np.floating,)) and np.dtype(type(scale)) == np.float64
    store_scores_f64 = f64 and not scores_f32
    out_f64 = (np.result_type(sdt, np.asarray(V).dtype) == np.float64) and not out_f32
    qd, Kd, Vd = _f32(q).reshape(-1), _f32(K), _f32(V)
    S, D = Kd.shape
    scores = torch.empty(S, dtype=torch.float64 if store_scores_f64 else torch.float32, device=qd.device)
    out = torch.empty(D, dtype=torch.float64 if out_f64 else torch.float32, device=qd.device)
    ws = L.workspace(8 * S)
    L.check(L.lib().hokv_dense_attention(L.ptr(qd), L.ptr(Kd), L.ptr(Vd), D, S, int(mul_f64), float(scale),
                                         int(store_scores_f64) | (int(out_f64) << 1),
                                         L.ptr(mask) if mask is not None else None, L.ptr(scores), L.ptr(out),
                                         L.ptr(ws), ws.numel(), L.stream()), "dense_attention")
    return scores.cpu().numpy(), out.cpu().numpy()


# -- Reference --

def standard_attention(q, K, V, scale):
    """Dense single-query attention (compressed_attention.py:38-55).

    Returns (scores [seq_len], output [head_dim]).
    """
    return _dense(q, K, V, scale)


# -- Path A: scalar VQ --

def scalar_vq_attention(q, k_indices, k_codebook, V, scale):
    """Decompress K from the scalar codebook, then standard attention
    (compressed_attention.py:60-80)."""
    L.require_device()
    idx = np.asarray(k_indices)
    cb = _f32(k_codebook).reshape(-1)
    flat = _u8(idx).reshape(-1)
    K = torch.empty(flat.numel(), dtype=torch.float32, device=flat.device)
    L.check(L.lib().hokv_scalar_decode(L.ptr(flat), flat.numel(), L.ptr(cb), cb.numel(), L.ptr(K), L.stream()),
            "scalar_decode")
    L.device_status()
    K = K.reshape(idx.shape).cpu().numpy()
    return standard_attention(q, K, V, scale)


# -- Path B: vector VQ --

def _cents_dev(codebook):
    """[k, d] centroid array -> ([1, 256, d] zero-padded CUDA tensor, [1] counts)."""
    c = np.asarray(codebook, dtype=np.float32)
    k, d = c.shape
    pad = np.zeros((1, 256, d), np.float32)
    pad[0, :k] = c
    return L.to_dev(pad), L.to_dev(np.array([k], np.int32), torch.int32)


def _vq_scores_dev(q, k_indices, codebook, scale):
    from .product_codebook import tables_for, gather_scores
    cents, kc = _cents_dev(codebook)
    k = int(np.asarray(codebook).shape[0])
    T = tables_for(_f32(q).reshape(-1), cents, kc, 1, k)
    idx = _u8(k_indices).reshape(-1, 1)
    if _score_dtype(scale, q, codebook) == np.float64:
        raw = gather_scores(T, idx)
        out = torch.empty(raw.numel(), dtype=torch.float64, device=raw.device)
        L.check(L.lib().hokv_scale_f32_to_f64(L.ptr(raw), raw.numel(), float(scale), L.ptr(out), L.stream()), "scale")
        return out
    return gather_scores(T, idx, scale)


def vector_vq_attention_scores(q, k_indices, k_vector_codebook, scale):
    """(q @ codebook.T)[indices] * scale (compressed_attention.py:85-107)."""
    L.require_device()
    s = _vq_scores_dev(q, k_indices, k_vector_codebook, scale)
    L.device_status()
    return s.cpu().numpy()


def _value_output_dev(weights_dev, codes_dev, cents_dev, k_dev, M, sd):
    w = weights_dev
    if w.dtype != torch.float64:
        w64 = torch.empty(w.numel(), dtype=torch.float64, device=w.device)
        L.check(L.lib().hokv_scale_f32_to_f64(L.ptr(w.contiguous()), w.numel(), 1.0, L.ptr(w64), L.stream()), "cast")
        w = w64
    out = torch.empty(M * sd, dtype=torch.float32, device=w.device)
    ws = L.workspace(L.lib().hokv_pq_value_output_workspace_size(M))
    L.check(L.lib().hokv_pq_value_output(L.ptr(w), codes_dev.shape[0], L.ptr(codes_dev), codes_dev.stride(0), M, sd,
                                         L.ptr(cents_dev), 256, L.ptr(k_dev), L.ptr(out), L.ptr(ws), ws.numel(),
                                         L.stream()), "pq_value_output")
    return out


def vector_vq_value_output(attn_weights, v_indices, v_vector_codebook):
    """Bin weights by V cluster (f64), weighted centroid sum (compressed_attention.py:110-133)."""
    L.require_device()
    w = np.asarray(attn_weights)
    wd = L.to_dev(w, torch.float64 if w.dtype == np.float64 else torch.float32).reshape(-1)
    cents, kc = _cents_dev(v_vector_codebook)
    d = np.asarray(v_vector_codebook).shape[1]
    return _value_output_dev(wd, _u8(v_indices).reshape(-1, 1), cents, kc, 1, d).cpu().numpy()


def full_vector_vq_attention(q, k_indices, k_codebook, v_indices, v_codebook, scale):
    """Path B: K-side scores -> softmax -> V-side output (compressed_attention.py:136-160)."""
    L.require_device()
    s = _vq_scores_dev(q, k_indices, k_codebook, scale)
    w = _softmax_dev(s)
    cents, kc = _cents_dev(v_codebook)
    d = np.asarray(v_codebook).shape[1]
    out = _value_output_dev(w, _u8(v_indices).reshape(-1, 1), cents, kc, 1, d)
    return s.cpu().numpy(), out.cpu().numpy()


# -- Path D: product quantization --

def _pq_scores_dev(q, k_pq_indices, cb, scale):
    from .product_codebook import tables_for, gather_scores
    cents, kd = cb.centroids_device
    if not cb.finalized:
        raise RuntimeError("ProductCodebook not finalized")
    qq = np.asarray(q, dtype=np.float32).ravel()
    if qq.shape[0] != cb.head_dim:
        raise ValueError(f"Expected query of dim {cb.head_dim}, got {qq.shape[0]}")
    T = tables_for(_f32(qq), cents, kd, cb.n_subspaces, int(cb._k_host.max()))
    return gather_scores(T, _u8(k_pq_indices), np.float32(scale))


def pq_attention_scores(q, k_pq_indices, k_product_codebook, scale):
    """PQ tables + gather, times f32(scale) (compressed_attention.py:165-184)."""
    L.require_device()
    s = _pq_scores_dev(q, k_pq_indices, k_product_codebook, scale)
    L.device_status()
    return s.cpu().numpy()


def pq_value_output(attn_weights, v_pq_indices, v_product_codebook):
    """Per-subspace binned V output (compressed_attention.py:187-227)."""
    L.require_device()
    w = np.asarray(attn_weights)
    wd = L.to_dev(w, torch.float64 if w.dtype == np.float64 else torch.float32).reshape(-1)
    cents, kd = v_product_codebook.centroids_device
    return _value_output_dev(wd, _u8(v_pq_indices), cents, kd, v_product_codebook.n_subspaces,
                             v_product_codebook.sub_dim).cpu().numpy()


def full_pq_attention(q, k_pq_indices, k_pq_cb, v_pq_indices, v_pq_cb, scale):
    """Path D: PQ scores -> softmax -> PQ V output (compressed_attention.py:230-254)."""
    L.require_device()
    s = _pq_scores_dev(q, k_pq_indices, k_pq_cb, scale)
    w = _softmax_dev(s)
    cents, kd = v_pq_cb.centroids_device
    out = _value_output_dev(w, _u8(v_pq_indices), cents, kd, v_pq_cb.n_subspaces, v_pq_cb.sub_dim)
    return s.cpu().numpy(), out.cpu().numpy()


# -- Path F: prefiltered attention --

def prefiltered_attention(q, K, V, k_indices, k_codebook, scale, top_p: int = 32):
    """Top-p clusters by q . centroid, exact attention on their tokens, -1e9
    elsewhere (compressed_attention.py:259-310)."""
    L.require_device()
    from .product_codebook import tables_for
    cb = np.asarray(k_codebook, dtype=np.float32)
    n_clusters = cb.shape[0]
    cents, kc = _cents_dev(cb)
    coarse = tables_for(_f32(q).reshape(-1), cents, kc, 1, n_clusters).reshape(-1)
    idx = _u8(k_indices).reshape(-1)
    mask = torch.empty(idx.numel(), dtype=torch.uint8, device=idx.device)
    L.check(L.lib().hokv_prefilter_mask(L.ptr(coarse), n_clusters, L.ptr(idx), idx.numel(),
                                        min(int(top_p), n_clusters), L.ptr(mask), L.stream()), "prefilter_mask")
    return _dense(q, K, V, scale, mask=mask, scores_f32=True, out_f32=True)


# -- Path G: hybrid PQ + prefilter (CDC-03) --

def hybrid_pq_attention(q, K, V, k_pq_indices, k_pq_cb, scale, top_k: int = 256, sink_tokens: int = 4):
    """CDC-03: PQ scores rank all tokens, exact softmax attention over the
    sinks plus the top (top_k - sinks) tokens (compressed_attention.py:315-412).

    Returns (scores [seq_len] with -inf where unselected, output [head_dim], meta).
    """
    L.require_device()
    from .cdc03 import cdc03_single
    Kn = np.asarray(K, dtype=np.float32)
    seq_len = Kn.shape[0]
    codes = np.asarray(k_pq_indices)
    if codes.size and int(codes.max()) >= int(k_pq_cb._k_host.max()):
        raise IndexError("PQ code beyond the codebook size")
    approx = _pq_scores_dev(q, codes, k_pq_cb, scale)
    amin, amax = torch.aminmax(approx)
    cents, kd = k_pq_cb.centroids_device
    out, sel, ex = cdc03_single(_f32(q).reshape(-1), _f32(Kn), _f32(V), _u8(codes), cents, kd, float(scale),
                                int(top_k), int(sink_tokens), 0, k_pq_cb.sub_dim)
    scores = torch.full((seq_len,), float("-inf"), dtype=torch.float32, device=out.device)
    scores[sel.long()] = ex
    n_sel = int(sel.numel())
    meta = {
        "selected_count": n_sel,
        "coverage": float(n_sel) / seq_len,
        "pq_score_range": float(np.float32(amax.item()) - np.float32(amin.item())),
        "sink_count": min(sink_tokens, seq_len),
    }
    return scores.cpu().numpy(), out.cpu().numpy().astype(np.float32), meta
