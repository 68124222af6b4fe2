"""OnlineCodebook: scalar codebook, calibrated on the first tokens, then streamed.

Drop-in for the reference class (helix_online_kv/codebook.py).  Calibration
(percentile-init 1-D k-means), assignment, decoding, drift correction and the
quality metrics all run as CUDA kernels of libhokv; NumPy inputs give NumPy
outputs, CUDA tensors give CUDA tensors.
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


def _flat_dev(values):
    """Flat float32-or-half CUDA view of ``values`` (numpy or tensor)."""
    if _is_tensor(values):
        t = values.detach().reshape(-1)
        if t.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            t = t.float()
        return t.to(L.device()).contiguous()
    return L.to_dev(np.asarray(values).ravel().astype(np.float32))


class OnlineCodebook:
    """Scalar codebook: ``feed_calibration`` -> ``finalize_calibration`` -> ``assign``.

    Lifecycle and errors as in codebook.py:47-176.
    """

    def __init__(self, n_clusters: int = 256, max_iters: int = 10, rtol: float = 0.001,
                 drift_threshold: float = 0.01, drift_ema_alpha: float = 0.05):
        self.n_clusters = n_clusters
        self.max_iters = max_iters
        self.rtol = rtol
        self.drift_threshold = drift_threshold
        self.drift_ema_alpha = drift_ema_alpha
        self._calibration_buffer: list = []
        self._centroids: np.ndarray | None = None
        self._cent_dev = None
        self._finalized = False

    @property
    def finalized(self) -> bool:
        return self._finalized

    @property
    def centroids(self) -> np.ndarray | None:
        return self._centroids

    @property
    def centroids_device(self):
        """The centroids as a CUDA float32 tensor (None before calibration)."""
        return self._cent_dev

    def _set_centroids_dev(self, dev):
        self._cent_dev = dev
        self._centroids = dev.cpu().numpy()

    # ---- checkpoint / resume (the reference has no serialization) ------------
    _PARAMS = ("n_clusters", "max_iters", "rtol", "drift_threshold", "drift_ema_alpha")

    def state_dict(self) -> dict:
        """Parameters, phase, centroids and pending calibration values, as CPU tensors."""
        buf = [p.reshape(-1).float().cpu() if _is_tensor(p) else torch.from_numpy(np.asarray(p, np.float32).ravel())
               for p in self._calibration_buffer]
        return {"params": {k: getattr(self, k) for k in self._PARAMS}, "finalized": self._finalized,
                "centroids": None if self._cent_dev is None else self._cent_dev.detach().cpu(),
                "calibration": torch.cat(buf) if buf else None}

    def load_state_dict(self, state: dict) -> None:
        mine = {k: getattr(self, k) for k in self._PARAMS}
        if state["params"] != mine:
            raise ValueError(f"Expected parameters {mine}, got {state['params']}")
        self._calibration_buffer = [] if state["calibration"] is None else [state["calibration"].clone()]
        self._finalized = bool(state["finalized"])
        if state["centroids"] is None:
            self._cent_dev, self._centroids = None, None
        else:
            self._set_centroids_dev(L.to_dev(state["centroids"]))

    def feed_calibration(self, values) -> None:
        """Accumulate calibration values (codebook.py:47-55)."""
        if self._finalized:
            raise RuntimeError("Codebook already finalized")
        if _is_tensor(values):
            self._calibration_buffer.append(values.detach().reshape(-1).float())
        else:
            self._calibration_buffer.append(np.asarray(values).ravel().astype(np.float32))

    def finalize_calibration(self) -> dict:
        """Fit the codebook on the device (codebook.py:57-84, 178-221)."""
        if self._finalized:
            raise RuntimeError("Codebook already finalized")
        if not self._calibration_buffer:
            raise RuntimeError("No calibration data fed")
        L.require_device()
        parts = [p if _is_tensor(p) else torch.from_numpy(p) for p in self._calibration_buffer]
        data = torch.cat([p.to(L.device()) for p in parts]).contiguous()
        self._calibration_buffer.clear()
        stats = fit_scalar(data[None, :], self.n_clusters, self.max_iters, self.rtol)
        self._set_centroids_dev(stats["centroids"][0, :stats["k"][0]].contiguous())
        self._finalized = True
        return {"n_samples": int(data.numel()), "n_clusters": int(stats["k"][0]),
                "n_iters": int(stats["iters"][0]), "calibration_mse": float(stats["mse"][0])}

    def assign(self, values):
        """Nearest centroid (first minimum) as uint8 (codebook.py:86-99)."""
        if not self._finalized:
            raise RuntimeError("Codebook not finalized — call finalize_calibration() first")
        x = _flat_dev(values)
        out = torch.empty(x.numel(), dtype=torch.uint8, device=x.device)
        if x.numel():
            L.check(L.lib().hokv_scalar_assign(L.ptr(x), L.dtype_code(x), x.numel(), 0, L.ptr(self._cent_dev),
                                               self._cent_dev.numel(), 0, L.ptr(out), 0, 1, L.stream()),
                    "scalar_assign")
        return out if _is_tensor(values) else out.cpu().numpy()

    def decode(self, indices):
        """centroids[indices] (codebook.py:101-112)."""
        if not self._finalized:
            raise RuntimeError("Codebook not finalized")
        idx = indices if _is_tensor(indices) else L.to_dev(np.asarray(indices), torch.uint8)
        flat = idx.reshape(-1).to(torch.uint8).contiguous()
        out = torch.empty(flat.numel(), dtype=torch.float32, device=flat.device)
        if flat.numel():
            L.check(L.lib().hokv_scalar_decode(L.ptr(flat), flat.numel(), L.ptr(self._cent_dev),
                                               self._cent_dev.numel(), L.ptr(out), L.stream()), "scalar_decode")
        out = out.reshape(tuple(idx.shape))
        return out if _is_tensor(indices) else out.cpu().numpy()

    def _stats(self, values, indices):
        x = _flat_dev(values).float().contiguous()
        r = self.decode(indices if _is_tensor(indices) else L.to_dev(np.asarray(indices), torch.uint8))
        return recon_stats(x, r.reshape(-1).contiguous())

    def quantization_error(self, values, indices) -> float:
        """MSE of the reconstruction in NumPy's float32 order (codebook.py:114-125)."""
        s = self._stats(values, indices)
        return float(np.float32(s["sse"] / s["n"]))

    def cosine_similarity(self, values, indices) -> float:
        """Cosine between values and reconstruction (codebook.py:127-144)."""
        s = self._stats(values, indices)
        na, nb = np.sqrt(s["xx"]), np.sqrt(s["rr"])
        if na < 1e-30 or nb < 1e-30:
            return 0.0
        return float(s["xr"] / (na * nb))

    def maybe_update_centroids(self, values, error: float) -> bool:
        """EMA drift correction when error exceeds the threshold (codebook.py:146-176)."""
        if not self._finalized:
            return False
        if error <= self.drift_threshold:
            return False
        x = _flat_dev(values).float().contiguous()
        cents = self._cent_dev.clone()
        ws = L.workspace(L.lib().hokv_scalar_ema_workspace_size(x.numel()))
        L.check(L.lib().hokv_scalar_ema(L.ptr(x), x.numel(), L.ptr(cents), cents.numel(),
                                        float(self.drift_ema_alpha), L.ptr(ws), ws.numel(), L.stream()),
                "scalar_ema")
        self._set_centroids_dev(cents)
        return True


def fit_scalar(data, n_clusters: int, max_iters: int, rtol: float):
    """Batched 1-D k-means: ``data`` is a [sets, n] float32 CUDA tensor."""
    L.require_device()
    data = data.float().contiguous()
    n_sets, n = data.shape
    dev = data.device
    cents = torch.zeros((n_sets, n_clusters), dtype=torch.float32, device=dev)
    k = torch.zeros(n_sets, dtype=torch.int32, device=dev)
    it = torch.zeros(n_sets, dtype=torch.int32, device=dev)
    mse = torch.zeros(n_sets, dtype=torch.float64, device=dev)
    ws = L.workspace(L.lib().hokv_scalar_kmeans_workspace_size(n, n_sets))
    L.check(L.lib().hokv_scalar_kmeans(L.ptr(data), n, n, n_sets, n_clusters, max_iters, float(rtol), L.ptr(cents),
                                       L.ptr(k), L.ptr(it), L.ptr(mse), None, L.ptr(ws), ws.numel(), L.stream()),
            "scalar_kmeans")
    return {"centroids": cents, "k": k.cpu().numpy(), "iters": it.cpu().numpy(), "mse": mse.cpu().numpy()}


def recon_stats(x, r) -> dict:
    """sum((x - r)^2) in NumPy's order, x.r, |x|^2, |r|^2 for two flat f32 CUDA tensors."""
    out = torch.zeros(4, dtype=torch.float64, device=x.device)
    ws = L.workspace(4 * x.numel())
    L.check(L.lib().hokv_recon_stats(L.ptr(x), L.ptr(r), x.numel(), L.ptr(out), L.ptr(ws), ws.numel(), L.stream()),
            "recon_stats")
    o = out.cpu().numpy()
    return {"sse": o[0], "xr": o[1], "xx": o[2], "rr": o[3], "n": x.numel()}
