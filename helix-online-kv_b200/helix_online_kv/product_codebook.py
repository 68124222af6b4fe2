"""ProductCodebook: product quantization over M contiguous subspaces.

Drop-in for the reference class (helix_online_kv/product_codebook.py).  The
per-subspace k-means fits run as one batched kernel launch, assignment is one
launch over all subspaces, and the compressed-domain primitives (sub-tables,
ADC gather) are the same kernels the CDC-03 decode path uses.
"""

from __future__ import annotations

import numpy as np

from . import _lib as L
from .vector_codebook import VectorCodebook

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None

SLOTS = 256


def _is_tensor(x) -> bool:
    return torch is not None and isinstance(x, torch.Tensor)


def fit_subspaces(data, M: int, n_clusters: int, max_iters: int, rtol: float):
    """Batched vector k-means over ``M`` subspaces of ``data`` [sets, n, M*sd].

    Returns device tensors cents [sets, M, 256, sd], k [sets, M] (int32) and
    host arrays iters, mse of shape [sets, M].
    """
    L.require_device()
    data = data.float().contiguous()
    n_sets, n, D = data.shape
    sd = D // M
    dev = data.device
    cents = torch.zeros((n_sets, M, SLOTS, sd), dtype=torch.float32, device=dev)
    k = torch.zeros((n_sets, M), dtype=torch.int32, device=dev)
    it = torch.zeros((n_sets, M), dtype=torch.int32, device=dev)
    mse = torch.zeros((n_sets, M), dtype=torch.float64, device=dev)
    # set (b, s) reads columns [s*sd, (s+1)*sd) of rows of length D
    ws = L.workspace(L.lib().hokv_vq_kmeans_workspace_size(n, sd, M))
    for b in range(n_sets):
        base = data[b]
        L.check(L.lib().hokv_vq_kmeans(L.ptr(base), n, sd, D, sd, M, n_clusters, max_iters, float(rtol),
                                       L.ptr(cents[b]), SLOTS, L.ptr(k[b]), L.ptr(it[b]), L.ptr(mse[b]),
                                       L.ptr(ws), ws.numel(), L.stream()), "vq_kmeans")
    return cents, k, it.cpu().numpy(), mse.cpu().numpy()


def assign_subspaces(x, cents, k, M: int, order: int | None = None):
    """Codes [N, M] uint8 of vectors ``x`` [N, M*sd] (CUDA) against one codebook."""
    N = x.shape[0]
    sd = cents.shape[-1]
    out = torch.empty((N, M), dtype=torch.uint8, device=x.device)
    if N == 0:
        return out
    if order is None:
        order = L.dot_order_for(N, sd)
    L.check(L.lib().hokv_pq_assign(L.ptr(x), L.dtype_code(x), N, x.shape[1], 0, M, sd, L.ptr(cents), SLOTS, 0,
                                   L.ptr(k), 0, L.ptr(out), M, 0, 1, order, L.stream()), "pq_assign")
    return out


def tables_for(q, cents, k, M: int, t_cols: int):
    """Sub-tables T[M, t_cols] of one query (CUDA f32)."""
    sd = cents.shape[-1]
    T = torch.empty((M, t_cols), dtype=torch.float32, device=q.device)
    L.check(L.lib().hokv_pq_tables(L.ptr(q), 1, M, sd, L.ptr(cents), SLOTS, 0, L.ptr(k), 0, None, L.ptr(T), t_cols,
                                   L.stream()), "pq_tables")
    return T


def gather_scores(T, codes, scale: float | None = None):
    """((0 + T[0][c0]) + T[1][c1]) + ... [* f32 scale] for codes [S, M] (CUDA)."""
    S, M = codes.shape
    out = torch.empty(S, dtype=torch.float32, device=codes.device)
    if S == 0:
        return out
    L.check(L.lib().hokv_pq_gather(L.ptr(T), T.shape[0], T.shape[1], L.ptr(codes), S, codes.stride(0),
                                   int(scale is not None), float(np.float32(scale if scale is not None else 1.0)),
                                   L.ptr(out), L.stream()), "pq_gather")
    return out


class ProductCodebook:
    """Product quantization: M independent sub-codebooks over head_dim
    (product_codebook.py:28-250)."""

    def __init__(self, n_subspaces: int = 8, sub_clusters: int = 256, head_dim: int = 64,
                 max_iters: int = 30, rtol: float = 1e-4):
        if head_dim % n_subspaces != 0:
            raise ValueError(
                f"head_dim ({head_dim}) must be divisible by n_subspaces ({n_subspaces})")
        self.n_subspaces = n_subspaces
        self.sub_clusters = sub_clusters
        self.head_dim = head_dim
        self.sub_dim = head_dim // n_subspaces
        self.max_iters = max_iters
        self.rtol = rtol
        self._codebooks: list[VectorCodebook] = [
            VectorCodebook(n_clusters=sub_clusters, head_dim=self.sub_dim, max_iters=max_iters, rtol=rtol)
            for _ in range(n_subspaces)
        ]
        self._buffer: list = []
        self._cents_dev = None   # [M, 256, sd]
        self._k_dev = None       # [M] int32
        self._k_host = None
        self._finalized = False

    @property
    def finalized(self) -> bool:
        return self._finalized

    @property
    def centroids_device(self):
        """(centroids [M, 256, sub_dim] f32, counts [M] int32) on the device."""
        return self._cents_dev, self._k_dev

    def _check_shape(self, v):
        if v.ndim != 2 or v.shape[1] != self.head_dim:
            raise ValueError(f"Expected shape [N, {self.head_dim}], got {tuple(v.shape)}")

    def feed_calibration(self, vectors) -> None:
        """Accumulate [N, head_dim] calibration vectors (product_codebook.py:65-84)."""
        if self._finalized:
            raise RuntimeError("ProductCodebook already finalized")
        v = vectors.detach().float() if _is_tensor(vectors) else np.asarray(vectors, dtype=np.float32)
        self._check_shape(v)
        self._buffer.append(v)
        for cb in self._codebooks:   # keeps the reference's per-subspace buffer visible
            cb._calibration_buffer.append(None)

    def finalize_calibration(self) -> dict:
        """Fit all subspaces in one batched launch (product_codebook.py:86-116)."""
        if self._finalized:
            raise RuntimeError("ProductCodebook already finalized")
        if not self._buffer:
            raise RuntimeError("No calibration data fed")
        L.require_device()
        parts = [p.to(L.device()) if _is_tensor(p) else torch.from_numpy(p).to(L.device()) for p in self._buffer]
        data = torch.cat(parts, 0).contiguous()
        self._buffer.clear()
        cents, k, iters, mse = fit_subspaces(data[None], self.n_subspaces, self.sub_clusters, self.max_iters,
                                             self.rtol)
        self._cents_dev, self._k_dev = cents[0].contiguous(), k[0].contiguous()
        self._k_host = self._k_dev.cpu().numpy()
        host_c = self._cents_dev.cpu().numpy()
        n = data.shape[0]
        for s, cb in enumerate(self._codebooks):
            cb._calibration_buffer.clear()
            cb._adopt(self._cents_dev[s:s + 1], self._k_dev[s:s + 1], host_c[s, :self._k_host[s]],
                      {"n_samples": n, "n_clusters": int(self._k_host[s]), "head_dim": self.sub_dim,
                       "n_iters": int(iters[0, s]), "calibration_mse": float(mse[0, s])})
        self._finalized = True
        per = [float(x) for x in mse[0]]
        return {
            "n_subspaces": self.n_subspaces,
            "sub_dim": self.sub_dim,
            "head_dim": self.head_dim,
            "sub_clusters": [int(x) for x in self._k_host],
            "calibration_mse_per_sub": per,
            "calibration_mse_total": float(np.mean(per)),
            "n_iters_per_sub": [int(x) for x in iters[0]],
        }

    def _require(self, msg):
        if not self._finalized:
            raise RuntimeError(msg)

    # ---- checkpoint / resume (the reference has no serialization) ------------
    _PARAMS = ("n_subspaces", "sub_clusters", "head_dim", "max_iters", "rtol")

    def state_dict(self) -> dict:
        """Parameters, phase, the M sub-codebooks (slots and counts) and pending
        calibration vectors, as CPU tensors."""
        buf = [p.float().cpu() if _is_tensor(p) else torch.from_numpy(np.asarray(p, np.float32)) for p in self._buffer]
        return {"params": {k: getattr(self, k) for k in self._PARAMS}, "finalized": self._finalized,
                "centroids": None if self._cents_dev is None else self._cents_dev.detach().cpu(),
                "counts": None if self._k_dev is None else self._k_dev.detach().cpu(),
                "calibration": torch.cat(buf, 0) if buf else None}

    def load_state_dict(self, state: dict) -> None:
        mine = {k: getattr(self, k) for k in self._PARAMS}
        if state["params"] != mine:
            raise ValueError(f"Expected parameters {mine}, got {state['params']}")
        self._buffer = [] if state["calibration"] is None else [state["calibration"].clone()]
        for cb in self._codebooks:
            cb._calibration_buffer = [None] * len(self._buffer)
        self._finalized = bool(state["finalized"])
        if state["centroids"] is None:
            self._cents_dev = self._k_dev = self._k_host = None
            return
        self._cents_dev = L.to_dev(state["centroids"])
        self._k_dev = L.to_dev(state["counts"], torch.int32)
        self._k_host = state["counts"].numpy().astype(np.int32)
        host_c = state["centroids"].numpy()
        for s, cb in enumerate(self._codebooks):
            cb._calibration_buffer = []
            cb._adopt(self._cents_dev[s:s + 1], self._k_dev[s:s + 1], host_c[s, :self._k_host[s]].copy(), None)

    def assign(self, vectors):
        """[N, M] uint8 codes (product_codebook.py:118-145)."""
        self._require("ProductCodebook not finalized -- call finalize_calibration() first")
        x = vectors.detach() if _is_tensor(vectors) else np.asarray(vectors, dtype=np.float32)
        self._check_shape(x)
        xd = L.to_dev(x) if not _is_tensor(x) else x.to(L.device()).contiguous()
        if xd.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            xd = xd.float()
        out = assign_subspaces(xd, self._cents_dev, self._k_dev, self.n_subspaces)
        return out if _is_tensor(vectors) else out.cpu().numpy()

    def decode(self, indices):
        """[N, head_dim] reconstruction (product_codebook.py:147-168)."""
        self._require("ProductCodebook not finalized")
        idx = indices if _is_tensor(indices) else L.to_dev(np.asarray(indices), torch.uint8)
        idx = idx.to(torch.uint8).contiguous()
        N = idx.shape[0]
        out = torch.empty((N, self.head_dim), dtype=torch.float32, device=idx.device)
        if N:
            L.check(L.lib().hokv_pq_decode(L.ptr(idx), N, idx.stride(0), self.n_subspaces, self.sub_dim,
                                           L.ptr(self._cents_dev), SLOTS, L.ptr(out), L.stream()), "pq_decode")
        return out if _is_tensor(indices) else out.cpu().numpy()

    # -- compressed-domain primitives --

    def precompute_distance_tables(self, q):
        """T[s, j] = q_s . C_s[j], zero-padded to the largest k (product_codebook.py:172-205)."""
        self._require("ProductCodebook not finalized")
        qq = q.detach().float().reshape(-1) if _is_tensor(q) else np.asarray(q, dtype=np.float32).ravel()
        if qq.shape[0] != self.head_dim:
            raise ValueError(f"Expected query of dim {self.head_dim}, got {qq.shape[0]}")
        qd = qq.to(L.device()).contiguous() if _is_tensor(qq) else L.to_dev(qq)
        T = tables_for(qd, self._cents_dev, self._k_dev, self.n_subspaces, int(self._k_host.max()))
        return T if _is_tensor(q) else T.cpu().numpy()

    def gather_pq_scores(self, tables, indices):
        """score_t = sum_s tables[s, indices[t, s]] in ascending s (product_codebook.py:207-227)."""
        T = tables if _is_tensor(tables) else L.to_dev(np.asarray(tables, dtype=np.float32))
        idx = indices if _is_tensor(indices) else L.to_dev(np.asarray(indices), torch.uint8)
        out = gather_scores(T.float().contiguous(), idx.to(torch.uint8).contiguous())
        L.device_status()
        return out if _is_tensor(indices) else out.cpu().numpy()

    # -- quality metrics --

    def cosine_similarity(self, vectors, indices) -> float:
        from .codebook import recon_stats
        x = L.to_dev(np.asarray(vectors, dtype=np.float32)).reshape(-1)
        r = L.to_dev(self.decode(indices)).reshape(-1)
        s = recon_stats(x, r)
        na, nb = np.sqrt(s["xx"]), np.sqrt(s["rr"])
        if na < 1e-30 or nb < 1e-30:
            return 0.0
        return float(s["xr"] / (na * nb))

    def quantization_error(self, vectors, indices) -> float:
        from .codebook import recon_stats
        x = L.to_dev(np.asarray(vectors, dtype=np.float32)).reshape(-1)
        r = L.to_dev(self.decode(indices)).reshape(-1)
        s = recon_stats(x, r)
        return float(np.float32(s["sse"] / s["n"]))
