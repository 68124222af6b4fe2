"""VectorCodebook: one uint8 index per [head_dim] vector.

Drop-in for the reference class (helix_online_kv/vector_codebook.py).  It is
the M = 1 case of the product-quantization kernels: the same k-means,
assignment, sub-table and gather launches.
"""

from __future__ import annotations

import numpy as np

from . import _lib as L

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None


def _is_tensor(x) -> bool:
    return torch is not None and isinstance(x, torch.Tensor)


class VectorCodebook:
    """Vector codebook over [head_dim]-dimensional space (vector_codebook.py:23-242)."""

    def __init__(self, n_clusters: int = 256, head_dim: int = 64, max_iters: int = 30, rtol: float = 1e-4):
        self.n_clusters = n_clusters
        self.head_dim = head_dim
        self.max_iters = max_iters
        self.rtol = rtol
        self._calibration_buffer: list = []
        self._centroids: np.ndarray | None = None
        self._cents_dev = None  # [1, 256, head_dim]
        self._k_dev = None      # [1] int32
        self._finalized = False

    @property
    def finalized(self) -> bool:
        return self._finalized

    @property
    def centroids(self) -> np.ndarray | None:
        return self._centroids

    def _adopt(self, cents_dev, k_dev, host, stats):
        self._cents_dev, self._k_dev, self._centroids = cents_dev, k_dev, host
        self._finalized = True
        return stats

    # ---- checkpoint / resume (the reference has no serialization) ------------
    _PARAMS = ("n_clusters", "head_dim", "max_iters", "rtol")

    def state_dict(self) -> dict:
        """Parameters, phase, centroid slots and counts, pending calibration vectors (CPU tensors)."""
        buf = [p.float().cpu() if _is_tensor(p) else torch.from_numpy(np.asarray(p, np.float32))
               for p in self._calibration_buffer if p is not None]
        return {"params": {k: getattr(self, k) for k in self._PARAMS}, "finalized": self._finalized,
                "centroids": None if self._cents_dev is None else self._cents_dev.detach().cpu(),
                "counts": None if self._k_dev is None else self._k_dev.detach().cpu(),
                "calibration": torch.cat(buf, 0) if buf else None}

    def load_state_dict(self, state: dict) -> None:
        mine = {k: getattr(self, k) for k in self._PARAMS}
        if state["params"] != mine:
            raise ValueError(f"Expected parameters {mine}, got {state['params']}")
        self._calibration_buffer = [] if state["calibration"] is None else [state["calibration"].clone()]
        self._finalized = bool(state["finalized"])
        if state["centroids"] is None:
            self._cents_dev = self._k_dev = self._centroids = None
        else:
            self._cents_dev = L.to_dev(state["centroids"])
            self._k_dev = L.to_dev(state["counts"], torch.int32)
            kk = int(state["counts"].reshape(-1)[0])
            self._centroids = state["centroids"].reshape(-1, state["centroids"].shape[-2],
                                                         self.head_dim)[0, :kk].numpy().copy()

    def _check_shape(self, v):
        if v.ndim != 2 or v.shape[1] != self.head_dim:
            raise ValueError(f"Expected shape [N, {self.head_dim}], got {tuple(v.shape)}")

    def feed_calibration(self, vectors) -> None:
        """Accumulate [N, head_dim] vectors (vector_codebook.py:50-63)."""
        if self._finalized:
            raise RuntimeError("Codebook already finalized")
        v = vectors.detach().float() if _is_tensor(vectors) else np.asarray(vectors, dtype=np.float32)
        self._check_shape(v)
        self._calibration_buffer.append(v)

    def finalize_calibration(self) -> dict:
        """Vector k-means on the device (vector_codebook.py:65-93, 185-242)."""
        if self._finalized:
            raise RuntimeError("Codebook already finalized")
        if not self._calibration_buffer:
            raise RuntimeError("No calibration data fed")
        from .product_codebook import fit_subspaces
        L.require_device()
        parts = [p.to(L.device()) if _is_tensor(p) else torch.from_numpy(p).to(L.device())
                 for p in self._calibration_buffer]
        data = torch.cat(parts, 0).contiguous()
        self._calibration_buffer.clear()
        cents, k, iters, mse = fit_subspaces(data[None], 1, self.n_clusters, self.max_iters, self.rtol)
        kk = int(k[0, 0].item())
        return self._adopt(cents[0].contiguous(), k[0].contiguous(), cents[0, 0, :kk].cpu().numpy(),
                           {"n_samples": int(data.shape[0]), "n_clusters": kk, "head_dim": self.head_dim,
                            "n_iters": int(iters[0, 0]), "calibration_mse": float(mse[0, 0])})

    def assign(self, vectors):
        """Nearest centroid under ((|v|^2 - 2 v.c) + |c|^2) (vector_codebook.py:95-119)."""
        if not self._finalized:
            raise RuntimeError("Codebook not finalized -- call finalize_calibration() first")
        from .product_codebook import assign_subspaces
        x = vectors.detach() if _is_tensor(vectors) else np.asarray(vectors, dtype=np.float32)
        self._check_shape(x)
        xd = x.to(L.device()).contiguous() if _is_tensor(x) else L.to_dev(x)
        if xd.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            xd = xd.float()
        out = assign_subspaces(xd, self._cents_dev, self._k_dev, 1)[:, 0]
        return out if _is_tensor(vectors) else out.cpu().numpy()

    def decode(self, indices):
        """[N, head_dim] reconstruction (vector_codebook.py:121-132)."""
        if not self._finalized:
            raise RuntimeError("Codebook not finalized")
        idx = indices if _is_tensor(indices) else L.to_dev(np.asarray(indices), torch.uint8)
        shape = tuple(idx.shape)
        flat = idx.reshape(-1, 1).to(torch.uint8).contiguous()
        out = torch.empty((flat.shape[0], self.head_dim), dtype=torch.float32, device=flat.device)
        if flat.shape[0]:
            L.check(L.lib().hokv_pq_decode(L.ptr(flat), flat.shape[0], 1, 1, self.head_dim, L.ptr(self._cents_dev),
                                           256, L.ptr(out), L.stream()), "pq_decode")
        out = out.reshape(shape + (self.head_dim,))
        return out if _is_tensor(indices) else out.cpu().numpy()

    def precompute_query_scores(self, q):
        """q . centroid_j for every centroid (vector_codebook.py:136-148)."""
        if not self._finalized:
            raise RuntimeError("Codebook not finalized")
        from .product_codebook import tables_for
        qd = q.detach().float().reshape(-1).to(L.device()).contiguous() if _is_tensor(q) \
            else L.to_dev(np.asarray(q, dtype=np.float32).ravel())
        T = tables_for(qd, self._cents_dev, self._k_dev, 1, int(self._k_dev[0].item()))[0]
        return T if _is_tensor(q) else T.cpu().numpy()

    def gather_scores(self, precomputed, indices):
        """precomputed[indices] (vector_codebook.py:150-162)."""
        from .product_codebook import gather_scores
        T = precomputed if _is_tensor(precomputed) else L.to_dev(np.asarray(precomputed, dtype=np.float32))
        idx = indices if _is_tensor(indices) else L.to_dev(np.asarray(indices), torch.uint8)
        out = gather_scores(T.float().reshape(1, -1).contiguous(), idx.to(torch.uint8).reshape(-1, 1).contiguous())
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
