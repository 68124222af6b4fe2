"""CPU oracle for the helix-online-kv compressed-KV hot path.

TEST INFRASTRUCTURE ONLY.  This module restates, in NumPy, the algorithm of the
reference package ``helix_online_kv`` (echo313unfolding/helix-online-kv) for the
hot path: codebook calibration, nearest-centroid assignment, PQ lookup tables,
ADC scoring and CDC-03 hybrid attention.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and its
``--impl reference`` arm) may import it, and only as the checker or the timed
CPU baseline.  The shipped package never imports it; the product path runs the
CUDA library and fails loudly without it.

Parity pin: every function below was checked against the reference itself run
in the build container (NumPy 2.3.5, SciPy 1.18.1, OpenBLAS 0.3.30), through
the golden fixtures in ``tests/golden/`` written by
``tests/golden/make_golden.py``; ``tests/test_oracle_golden.py`` re-checks the
pin.  Where NumPy delegates to BLAS (``@``), the result depends on the BLAS
build and CPU; the fixtures record the values of the build container.

Each function cites the reference ``file:line`` it restates.
"""

from __future__ import annotations

import numpy as np
from scipy.special import softmax as _softmax

F32 = np.float32

# ---------------------------------------------------------------------------
# Seeded synthetic inputs (stand-ins for the reference's WikiText-2 KV dumps).
# The order of RNG draws is frozen: changing it changes every fixture.
# ---------------------------------------------------------------------------


def gen_kv(seed: int, B: int, H_kv: int, S: int, D: int, n_outliers: int = 4):
    """K, V float32 ``[B, H_kv, S, D]``.

    Per (sequence, head): channel scales ``U(0.5, 2)``, values ``N(0,1)*scale``,
    then ``n_outliers`` channels overwritten by ``Student-t(3) * 5``.  K is drawn
    before V for each (b, h); (b, h) run in row-major order.
    """
    rng = np.random.default_rng(seed)
    K = np.empty((B, H_kv, S, D), F32)
    V = np.empty((B, H_kv, S, D), F32)
    for b in range(B):
        for h in range(H_kv):
            for dst in (K, V):
                scale = rng.uniform(0.5, 2.0, D)
                vals = rng.standard_normal((S, D)) * scale
                cols = rng.choice(D, n_outliers, replace=False)
                vals[:, cols] = rng.standard_t(3, (S, n_outliers)) * 5.0
                dst[b, h] = vals.astype(F32)
    return K, V


def gen_queries(seed: int, B: int, H_q: int, D: int):
    """Queries float32 ``[B, H_q, D]`` drawn ``N(0, 1)``."""
    rng = np.random.default_rng(seed + 7919)
    return rng.standard_normal((B, H_q, D)).astype(F32)


def to_fp16_values(x):
    """Round to fp16 and back: the values the device store holds."""
    return np.asarray(x, F32).astype(np.float16).astype(F32)


# ---------------------------------------------------------------------------
# Scalar codebook  (helix_online_kv/codebook.py)
# ---------------------------------------------------------------------------


def scalar_assign(values, centroids):
    """argmin_j |x - c_j| (first minimum) as uint8.  codebook.py:86-99."""
    flat = np.asarray(values).ravel().astype(F32)
    return np.argmin(np.abs(flat[:, None] - centroids), axis=1).astype(np.uint8)


def scalar_fit(data, n_clusters: int = 256, max_iters: int = 10, rtol: float = 1e-3):
    """1-D k-means with percentile init.  codebook.py:178-221.

    Returns ``(centroids f32 [k], assignments u8 [N], n_iters)``; the
    assignments are those of the last assignment step, as in the reference.
    """
    data = np.asarray(data, F32).ravel()
    k = min(n_clusters, len(np.unique(data)))
    cents = np.percentile(data, np.linspace(0, 100, k)).astype(F32)
    span = float(cents[-1] - cents[0])
    tol = rtol * (span if span >= 1e-30 else 1.0)
    assign = np.zeros(len(data), np.uint8)
    it = 0
    for it in range(1, max_iters + 1):
        assign = np.argmin(np.abs(data[:, None] - cents), axis=1).astype(np.uint8)
        nxt = np.zeros_like(cents)
        for j in range(k):
            members = data[assign == j]
            nxt[j] = np.mean(members) if members.size else cents[j]
        shift = float(np.max(np.abs(nxt - cents)))
        cents = nxt
        if shift < tol:
            break
    return cents, assign, it


def scalar_finalize_stats(data, cents, assign, n_iters):
    """Stats dict of OnlineCodebook.finalize_calibration (codebook.py:57-84)."""
    data = np.asarray(data, F32).ravel()
    mse = float(np.mean((data - cents[assign]) ** 2))
    return {"n_samples": len(data), "n_clusters": len(cents), "n_iters": n_iters,
            "calibration_mse": mse}


def scalar_ema_update(values, centroids, alpha: float):
    """EMA drift correction of codebook.py:146-176 (caller checks the threshold)."""
    flat = np.asarray(values).ravel().astype(F32)
    idx = scalar_assign(flat, centroids)
    out = centroids.copy()
    for i in range(len(centroids)):
        m = idx == i
        if np.any(m):
            out[i] = (1 - alpha) * centroids[i] + alpha * np.mean(flat[m])
    return out


# ---------------------------------------------------------------------------
# Vector codebook  (helix_online_kv/vector_codebook.py)
# ---------------------------------------------------------------------------


def _l2_dists(x, cents):
    # ||x||^2 - 2 x.c + ||c||^2 evaluated as ((x2 - 2*dot) + c2), f32.
    x2 = np.sum(x ** 2, axis=1, keepdims=True)
    c2 = np.sum(cents ** 2, axis=1)
    return x2 - 2 * (x @ cents.T) + c2


def vq_assign(vectors, cents):
    """Nearest centroid under the L2 expansion.  vector_codebook.py:113-119."""
    x = np.asarray(vectors, F32)
    return np.argmin(_l2_dists(x, cents), axis=1).astype(np.uint8)


def vq_fit(data, n_clusters: int = 256, max_iters: int = 30, rtol: float = 1e-4):
    """Vector k-means, norm-sorted init.  vector_codebook.py:185-242."""
    data = np.asarray(data, F32)
    n = len(data)
    k = min(n_clusters, len(np.unique(data, axis=0)))
    norms = np.linalg.norm(data, axis=1)
    order = np.argsort(norms)
    picks = np.linspace(0, n - 1, k).astype(int)
    cents = data[order[picks]].copy().astype(F32)
    span = float(np.max(norms) - np.min(norms))
    tol = rtol * (span if span >= 1e-30 else 1.0)
    assign = np.zeros(n, np.uint8)
    it = 0
    for it in range(1, max_iters + 1):
        assign = np.argmin(_l2_dists(data, cents), axis=1).astype(np.uint8)
        nxt = np.zeros_like(cents)
        for j in range(k):
            m = assign == j
            nxt[j] = np.mean(data[m], axis=0) if np.any(m) else cents[j]
        shift = float(np.max(np.linalg.norm(nxt - cents, axis=1)))
        cents = nxt
        if shift < tol:
            break
    return cents, assign, it


def vq_finalize_stats(data, cents, assign, n_iters, head_dim):
    """Stats dict of VectorCodebook.finalize_calibration (vector_codebook.py:79-93)."""
    data = np.asarray(data, F32)
    mse = float(np.mean((data - cents[assign]) ** 2))
    return {"n_samples": len(data), "n_clusters": len(cents), "head_dim": head_dim,
            "n_iters": n_iters, "calibration_mse": mse}


# ---------------------------------------------------------------------------
# Product codebook  (helix_online_kv/product_codebook.py)
# ---------------------------------------------------------------------------


def pq_split(vectors, M):
    x = np.asarray(vectors, F32)
    sd = x.shape[1] // M
    return [x[:, s * sd:(s + 1) * sd] for s in range(M)]


def pq_fit(vectors, M: int = 8, sub_clusters: int = 256, max_iters: int = 30,
           rtol: float = 1e-4):
    """One vector k-means per contiguous subspace.  product_codebook.py:65-116."""
    fits = [vq_fit(part, sub_clusters, max_iters, rtol) for part in pq_split(vectors, M)]
    return [f[0] for f in fits], fits


def pq_assign(vectors, cents_list):
    """[N, M] uint8 codes.  product_codebook.py:118-145."""
    parts = pq_split(vectors, len(cents_list))
    out = np.zeros((parts[0].shape[0], len(cents_list)), np.uint8)
    for s, (p, c) in enumerate(zip(parts, cents_list)):
        out[:, s] = vq_assign(p, c)
    return out


def pq_decode(codes, cents_list):
    """Concatenated sub-centroids.  product_codebook.py:147-168."""
    return np.concatenate([c[codes[:, s]] for s, c in enumerate(cents_list)], axis=1).astype(F32)


def pq_tables(q, cents_list):
    """LUT T[s, j] = q_s . C_s[j], zero-padded to max k.  product_codebook.py:172-205."""
    q = np.asarray(q, F32).ravel()
    M = len(cents_list)
    sd = q.shape[0] // M
    kmax = max(len(c) for c in cents_list)
    T = np.zeros((M, kmax), F32)
    for s, c in enumerate(cents_list):
        T[s, :len(c)] = q[s * sd:(s + 1) * sd] @ c.T
    return T


def pq_gather(tables, codes):
    """ADC score: sum over subspaces in ascending order, f32.  product_codebook.py:207-227."""
    out = np.zeros(codes.shape[0], F32)
    for s in range(tables.shape[0]):
        out += tables[s][codes[:, s]]
    return out


# ---------------------------------------------------------------------------
# Attention paths  (helix_online_kv/compressed_attention.py)
# ---------------------------------------------------------------------------


def standard_attention(q, K, V, scale):
    """compressed_attention.py:38-55."""
    s = (q @ K.T) * scale
    return s, _softmax(s) @ V


def scalar_vq_attention(q, k_idx, k_cb, V, scale):
    """Path A, compressed_attention.py:60-80."""
    return standard_attention(q, k_cb[k_idx], V, scale)


def vector_vq_attention_scores(q, k_idx, k_cb, scale):
    """Path B K side, compressed_attention.py:85-107."""
    return (q @ k_cb.T)[k_idx] * scale


def vector_vq_value_output(w, v_idx, v_cb):
    """Path B V side: f64 bins then weighted centroid sum.  compressed_attention.py:110-133."""
    bins = np.zeros(len(v_cb), np.float64)
    np.add.at(bins, v_idx, w)
    return (bins @ v_cb).astype(F32)


def pq_attention_scores(q, codes, cents_list, scale):
    """Path D K side, compressed_attention.py:165-184."""
    return pq_gather(pq_tables(q, cents_list), codes) * np.float32(scale)


def pq_value_output(w, codes, cents_list):
    """Path D V side, compressed_attention.py:187-227."""
    sd = cents_list[0].shape[1]
    out = np.zeros(len(cents_list) * sd, F32)
    for s, c in enumerate(cents_list):
        bins = np.zeros(len(c), np.float64)
        np.add.at(bins, codes[:, s], w)
        out[s * sd:(s + 1) * sd] = (bins @ c).astype(F32)
    return out


def prefiltered_attention(q, K, V, k_idx, k_cb, scale, top_p=32):
    """Path F, compressed_attention.py:259-310."""
    p = min(top_p, len(k_cb))
    keep = np.argsort(q @ k_cb.T)[-p:]
    mask = np.isin(k_idx, keep)
    s = np.full(K.shape[0], -1e9, dtype=F32)
    if np.any(mask):
        s[mask] = (q @ K[mask].T) * scale
    return s, (_softmax(s) @ V).astype(F32)


def cdc03_select(approx, top_k, sink_tokens):
    """Selected token set of CDC-03 (compressed_attention.py:366-388), sorted.

    Uses ``np.argpartition`` like the reference, so ties at the boundary are
    broken the way NumPy breaks them.
    """
    n = approx.shape[0]
    k = min(top_k, n)
    sink = min(sink_tokens, n)
    if k >= n:
        return np.arange(n)
    chosen = set(range(sink))
    budget = k - sink
    if budget > 0:
        masked = approx.copy()
        masked[:sink] = -np.inf
        chosen |= set(np.argpartition(masked, -budget)[-budget:].tolist())
    return np.array(sorted(chosen), dtype=np.intp)


def cdc03_select_canonical(approx, top_k, sink_tokens):
    """Same rule, ties broken toward the lower token index (the device rule)."""
    n = approx.shape[0]
    k = min(top_k, n)
    sink = min(sink_tokens, n)
    if k >= n:
        return np.arange(n)
    budget = k - sink
    chosen = list(range(sink))
    if budget > 0:
        cand = np.arange(sink, n)
        order = np.lexsort((cand, -approx[sink:].astype(np.float64)))
        chosen += cand[order[:budget]].tolist()
    return np.array(sorted(chosen), dtype=np.intp)


def hybrid_pq_attention(q, K, V, codes, cents_list, scale, top_k=256, sink_tokens=4,
                        select=cdc03_select):
    """CDC-03 (Path G), compressed_attention.py:315-412."""
    n = K.shape[0]
    approx = pq_gather(pq_tables(q, cents_list), codes) * np.float32(scale)
    sel = select(approx, top_k, sink_tokens)
    exact = (q @ K[sel].T) * scale
    out = (_softmax(exact) @ V[sel]).astype(F32)
    scores = np.full(n, -np.inf, dtype=F32)
    scores[sel] = exact
    meta = {"selected_count": len(sel), "coverage": float(len(sel)) / n,
            "pq_score_range": float(np.max(approx) - np.min(approx)),
            "sink_count": min(sink_tokens, n)}
    return scores, out, meta


def cdc03_hot_attention(q, K, V, codes, cents_list, scale, top_k=128, sink_tokens=4,
                        hot_window=256, select=cdc03_select_canonical):
    """CDC-03 with an exact hot window, composed only of the steps above.

    Tokens ``[0, S_c)`` with ``S_c = max(0, S - hot_window)`` are cold: they are
    ranked by the PQ score and selected by the CDC-03 rule on that range.  Hot
    tokens ``[S_c, S)`` are always attended.  Exact f32 softmax over the union.
    With ``hot_window=0`` this is :func:`hybrid_pq_attention`.

    Returns ``(selected cold indices, exact scores of the union, out [D] f32)``.
    """
    S = K.shape[0]
    Sc = max(0, S - hot_window)
    if Sc > 0:
        approx = pq_gather(pq_tables(q, cents_list), codes[:Sc]) * np.float32(scale)
        sel = select(approx, top_k, sink_tokens)
    else:
        sel = np.zeros(0, np.intp)
    union = np.concatenate([sel, np.arange(Sc, S)]).astype(np.intp)
    exact = (q @ K[union].T) * scale
    out = (_softmax(exact) @ V[union]).astype(F32)
    return sel, exact, out


def fused_scalar_vq_qkt_numpy(q, k_idx, codebook, scale):
    """triton_attention.py:123-141."""
    return ((codebook[k_idx] @ q) * scale).astype(F32)


# ---------------------------------------------------------------------------
# Layer state and aging  (layer_state.py, aging_policy.py) -- host logic.
# ---------------------------------------------------------------------------


def tier_boundary(total_tokens: int, hot_window: int, min_age=None):
    """aging_policy.py:42-56."""
    age = hot_window if min_age is None else min_age
    return 0 if total_tokens <= age else total_tokens - age


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    return 0.0 if na < 1e-30 or nb < 1e-30 else float(a @ b / (na * nb))
