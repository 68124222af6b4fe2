"""Batched CDC-03 decode attention on device-resident tiers.

``CDC03Store`` holds, for B sequences x L layers x H_kv KV heads, the exact
K/V store (fp16/bf16), the uint8 PQ codes of every token, the per-(sequence,
layer, head) PQ codebooks and the per-sequence lengths, all in HBM:

    k, v      [L, B, H_kv, capacity, D]           fp16 / bf16
    codes     [L, B, H_kv, capacity, code_bytes]  uint8 (bytes >= M unused)
    codebook  [L, B, H_kv, M, 256, D / M]         float32
    cb_k      [L, B, H_kv, M]                     int32 (centroids per subspace)
    seq_len   [B]                                 int32 (device)

``decode`` runs one layer of CDC-03 attention (libhokv ``hokv_cdc03_decode``)
for queries [B, H_q, D] on the current stream, with no host synchronisation,
so a decode step over all layers can be captured in a CUDA graph.  The
per-call selection rule is the reference's (compressed_attention.py:366-388)
applied to the cold range [0, seq_len - hot_window); the hot window is always
attended.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib as L
from .product_codebook import SLOTS


def code_bytes_for(M: int) -> int:
    for c in (4, 8, 16, 32):
        if M <= c:
            return c
    raise ValueError(f"at most 32 PQ subspaces are supported, got {M}")


class CDC03Store:
    def __init__(self, batch: int, n_layers: int, kv_heads: int, head_dim: int, capacity: int,
                 n_subspaces: int = 8, dtype=torch.float16, device=None):
        L.require_device()
        if head_dim % n_subspaces:
            raise ValueError(f"head_dim ({head_dim}) must be divisible by n_subspaces ({n_subspaces})")
        self.B, self.L, self.H, self.D = batch, n_layers, kv_heads, head_dim
        self.M = n_subspaces
        self.sd = head_dim // n_subspaces
        self.CS = code_bytes_for(n_subspaces)
        self.cap = int(-(-capacity // 16) * 16)
        dev = device or L.device()
        self.k = torch.zeros((n_layers, batch, kv_heads, self.cap, head_dim), dtype=dtype, device=dev)
        self.v = torch.zeros_like(self.k)
        self.codes = torch.zeros((n_layers, batch, kv_heads, self.cap, self.CS), dtype=torch.uint8, device=dev)
        self.codebook = torch.zeros((n_layers, batch, kv_heads, n_subspaces, SLOTS, self.sd), dtype=torch.float32,
                                    device=dev)
        self.cb_k = torch.zeros((n_layers, batch, kv_heads, n_subspaces), dtype=torch.int32, device=dev)
        self.seq_len = torch.zeros(batch, dtype=torch.int32, device=dev)
        self._ws = None
        self._args_cache = {}   # decode arguments by (layer, tensors, budgets): no per-call rebuild
        self._ws_need = {}      # workspace bytes by (group, budgets)

    # ---- calibration and assignment -----------------------------------------
    def calibrate(self, layer: int, n_tokens: int = 128, sub_clusters: int = 256, max_iters: int = 30,
                  rtol: float = 1e-4):
        """Fit the PQ codebooks of one layer on tokens [0, n_tokens) of every (b, h)
        (ProductCodebook.finalize_calibration, product_codebook.py:86-116)."""
        n = int(n_tokens)
        U = self.B * self.H
        # one launch for every (sequence, head, subspace) fit: sets [U * M][n][sd]
        data = (self.k[layer, :, :, :n, :self.M * self.sd].float().reshape(U, n, self.M, self.sd)
                .permute(0, 2, 1, 3).contiguous())
        n_sets = U * self.M
        ws = L.workspace(L.lib().hokv_vq_kmeans_workspace_size(n, self.sd, n_sets))
        it = torch.zeros(n_sets, dtype=torch.int32, device=data.device)
        mse = torch.zeros(n_sets, dtype=torch.float64, device=data.device)
        cb = self.codebook[layer].reshape(n_sets, SLOTS, self.sd)
        kk = self.cb_k[layer].reshape(n_sets)
        L.check(L.lib().hokv_vq_kmeans(L.ptr(data), n, self.sd, self.sd, n * self.sd, n_sets, sub_clusters,
                                       max_iters, float(rtol), L.ptr(cb), SLOTS, L.ptr(kk), L.ptr(it),
                                       L.ptr(mse), L.ptr(ws), ws.numel(), L.stream()), "vq_kmeans")

    def assign(self, layer: int, start: int, end: int, order: int | None = None):
        """PQ codes of tokens [start, end) of every (b, h) of one layer
        (ProductCodebook.assign, product_codebook.py:118-145)."""
        n = int(end) - int(start)
        if n <= 0:
            return
        if order is None:
            order = L.dot_order_for(n, self.sd)
        # one launch over every (sequence, head): sets are B * H_kv equally strided tiers
        x = self.k[layer, :, :, start:end, :]
        out = self.codes[layer, :, :, start:end, :]
        L.check(L.lib().hokv_pq_assign(L.ptr(x), L.dtype_code(x), n, self.D, self.cap * self.D, self.M, self.sd,
                                       L.ptr(self.codebook[layer]), SLOTS, self.M * SLOTS * self.sd,
                                       L.ptr(self.cb_k[layer]), self.M, L.ptr(out), self.CS,
                                       self.cap * self.CS, self.B * self.H, order, L.stream()), "pq_assign")

    # ---- checkpoint / resume ---------------------------------------------------
    _STATE = ("k", "v", "codes", "codebook", "cb_k", "seq_len")

    def state_dict(self) -> dict:
        """The store's tensors (exact tiers, codes, codebooks, lengths) and geometry;
        the reference has no serialization of its codebooks or indices."""
        state = {name: getattr(self, name) for name in self._STATE}
        state["geometry"] = dict(batch=self.B, n_layers=self.L, kv_heads=self.H, head_dim=self.D,
                                 capacity=self.cap, n_subspaces=self.M)
        return state

    def load_state_dict(self, state: dict) -> None:
        geo = state["geometry"]
        mine = dict(batch=self.B, n_layers=self.L, kv_heads=self.H, head_dim=self.D, capacity=self.cap,
                    n_subspaces=self.M)
        if geo != mine:
            raise ValueError(f"Expected shape {mine}, got {geo}")
        for name in self._STATE:
            getattr(self, name).copy_(state[name])

    # ---- tier aging ----------------------------------------------------------
    def _store_args(self, layer: int) -> L.Cdc03Args:
        a = L.Cdc03Args()
        a.batch, a.kv_heads, a.q_per_kv, a.head_dim = self.B, self.H, 1, self.D
        a.n_subspaces, a.sub_dim, a.code_bytes, a.cb_slots = self.M, self.sd, self.CS, SLOTS
        kl = self.k[layer]
        a.k, a.v, a.kv_dtype = kl.data_ptr(), self.v[layer].data_ptr(), L.dtype_code(kl)
        a.kv_stride_b, a.kv_stride_h = kl.stride(0), kl.stride(1)
        a.capacity = self.cap
        cl = self.codes[layer]
        a.codes, a.code_stride_b, a.code_stride_h = cl.data_ptr(), cl.stride(0), cl.stride(1)
        cb, ck = self.codebook[layer], self.cb_k[layer]
        a.codebook, a.cb_stride_b, a.cb_stride_h = cb.data_ptr(), cb.stride(0), cb.stride(1)
        a.cb_k, a.cbk_stride_b, a.cbk_stride_h = ck.data_ptr(), ck.stride(0), ck.stride(1)
        a.seq_len = self.seq_len.data_ptr()
        return a

    def age(self, layer: int, cold_from, cold_to, order: int | None = None):
        """PQ codes, in place, for tokens [cold_from[b], cold_to[b]) of every
        sequence b (device int32 tensors [B]); the tokens leaving the hot window
        (AgingPolicy.tier_boundary, aging_policy.py:42-56)."""
        cf = cold_from.to(device=self.k.device, dtype=torch.int32).contiguous()
        ct = cold_to.to(device=self.k.device, dtype=torch.int32).contiguous()
        if order is None:
            order = L.dot_order_for(1, self.sd)
        a = self._store_args(layer)
        L.check(L.lib().hokv_age_tokens(ctypes.byref(a), L.ptr(cf), L.ptr(ct), order, L.stream()), "age_tokens")

    def append(self, k_new, v_new, hot_window: int = 256, order: int | None = None):
        """One decode step's new token for every layer and sequence:
        k_new/v_new [L, B, H_kv, D] go to position seq_len[b]; the token that
        leaves the hot window (position seq_len[b] - hot_window) gets its PQ
        codes; seq_len grows by one.  Device-side only (no host sync)."""
        if k_new.shape != (self.L, self.B, self.H, self.D) or v_new.shape != k_new.shape:
            raise ValueError(f"Expected shape {(self.L, self.B, self.H, self.D)}, got {tuple(k_new.shape)}")
        # a full sequence keeps its rows; its length still grows, so the next
        # decode reports HOKV_ERR_DEVICE_INPUT through the device status
        full = (self.seq_len >= self.cap)[:, None, None, None]
        pos = torch.clamp(self.seq_len.long(), max=self.cap - 1)
        ar = torch.arange(self.B, device=pos.device)
        for store, new in ((self.k, k_new), (self.v, v_new)):
            store[:, ar, :, pos] = torch.where(full, store[:, ar, :, pos], new.to(store.dtype).permute(1, 0, 2, 3))
        cold_from = torch.clamp(self.seq_len - hot_window, min=0)
        cold_to = torch.clamp(self.seq_len + 1 - hot_window, min=0)
        for layer in range(self.L):
            self.age(layer, cold_from, cold_to, order)
        self.seq_len += 1

    # ---- decode ---------------------------------------------------------------
    def args(self, layer: int, q, out, scale: float, top_k: int = 128, sink_tokens: int = 4,
             hot_window: int = 256, sel_idx=None, sel_score=None, sel_count=None) -> L.Cdc03Args:
        """The C-ABI arguments of one layer's decode.  Built once per (layer,
        tensors, budgets) and kept: a decode step repeats the same calls, and the
        structure holds only device addresses and sizes."""
        ptr = lambda t: None if t is None else t.data_ptr()   # noqa: E731
        key = (layer, q.data_ptr(), q.dtype, tuple(q.shape), tuple(q.stride()), out.data_ptr(), out.dtype,
               tuple(out.stride()), float(scale), int(top_k), int(sink_tokens), int(hot_window), ptr(sel_idx),
               ptr(sel_score), ptr(sel_count))
        a = self._args_cache.get(key)
        if a is not None and self._ws is not None and a.workspace == self._ws.data_ptr():
            return a
        if len(self._args_cache) > 1024:
            self._args_cache.clear()
        a = self._build_args(layer, q, out, scale, top_k, sink_tokens, hot_window, sel_idx, sel_score, sel_count)
        self._args_cache[key] = a
        return a

    def _build_args(self, layer, q, out, scale, top_k, sink_tokens, hot_window, sel_idx, sel_score, sel_count):
        B, Hq, D = q.shape
        if B != self.B or D != self.D or Hq % self.H:
            raise ValueError(f"queries {tuple(q.shape)} do not match the store (B={self.B}, H_kv={self.H}, D={self.D})")
        if q.stride(2) != 1 or q.stride(1) != D or out.shape != q.shape or out.stride(2) != 1 or out.stride(1) != D:
            raise ValueError("queries and outputs must be [B, H_q, D] with contiguous heads")
        if not 0 <= layer < self.L:
            raise ValueError(f"layer {layer} outside 0..{self.L - 1}")
        a = L.Cdc03Args()
        a.batch, a.kv_heads, a.q_per_kv, a.head_dim = self.B, self.H, Hq // self.H, self.D
        a.n_subspaces, a.sub_dim, a.code_bytes, a.cb_slots = self.M, self.sd, self.CS, SLOTS
        a.top_k, a.sink_tokens, a.hot_window = int(top_k), int(sink_tokens), int(hot_window)
        a.scale = float(np.float32(scale))
        a.lut_order = L.DOT_GEMV
        a.q, a.q_dtype, a.q_stride_b = q.data_ptr(), L.dtype_code(q), q.stride(0)
        a.out, a.out_dtype, a.out_stride_b = out.data_ptr(), L.dtype_code(out), out.stride(0)
        kl, vl = self.k[layer], self.v[layer]
        a.k, a.v, a.kv_dtype = kl.data_ptr(), vl.data_ptr(), L.dtype_code(kl)
        a.kv_stride_b, a.kv_stride_h = kl.stride(0), kl.stride(1)
        a.capacity = self.cap
        cl = self.codes[layer]
        a.codes, a.code_stride_b, a.code_stride_h = cl.data_ptr(), cl.stride(0), cl.stride(1)
        cb, ck = self.codebook[layer], self.cb_k[layer]
        a.codebook, a.cb_stride_b, a.cb_stride_h = cb.data_ptr(), cb.stride(0), cb.stride(1)
        a.cb_k, a.cbk_stride_b, a.cbk_stride_h = ck.data_ptr(), ck.stride(0), ck.stride(1)
        a.seq_len = self.seq_len.data_ptr()
        a.sel_idx = sel_idx.data_ptr() if sel_idx is not None else None
        a.sel_score = sel_score.data_ptr() if sel_score is not None else None
        a.sel_count = sel_count.data_ptr() if sel_count is not None else None
        wkey = (a.q_per_kv, a.top_k, a.sink_tokens, a.hot_window)
        need = self._ws_need.get(wkey)
        if need is None:
            n = ctypes.c_size_t(0)
            L.check(L.lib().hokv_cdc03_workspace_size(ctypes.byref(a), ctypes.byref(n)), "cdc03_workspace_size")
            need = self._ws_need[wkey] = n.value
        if self._ws is None or self._ws.numel() < need:
            self._ws = L.workspace(need)
            self._args_cache.clear()   # earlier arguments point at the old workspace
        a.workspace, a.workspace_bytes = self._ws.data_ptr(), self._ws.numel()
        return a

    def decode(self, layer: int, q, scale: float, top_k: int = 128, sink_tokens: int = 4, hot_window: int = 256,
               out=None, out_dtype=None, return_selection: bool = False):
        """CDC-03 attention of queries q [B, H_q, D] against one layer."""
        q = q.contiguous()
        if out is None:
            out = torch.empty(q.shape, dtype=out_dtype or q.dtype, device=q.device)
        sel = None
        if return_selection:
            B, Hq, _ = q.shape
            cap = max(top_k, sink_tokens, 1)
            sel = (torch.empty((B, Hq, cap), dtype=torch.int32, device=q.device),
                   torch.empty((B, Hq, cap), dtype=torch.float32, device=q.device),
                   torch.empty((B, Hq), dtype=torch.int32, device=q.device))
        a = self.args(layer, q, out, scale, top_k, sink_tokens, hot_window, *(sel or (None, None, None)))
        L.check(L.lib().hokv_cdc03_decode(ctypes.byref(a), L.stream()), "cdc03_decode")
        return (out, sel) if return_selection else out


def cdc03_single(q, K, V, codes, cents, k_counts, scale: float, top_k: int, sink_tokens: int, hot_window: int = 0,
                 sub_dim: int | None = None):
    """One query head against one key sequence, float32 K/V (the NumPy API path).

    q [D], K/V [S, D] f32 CUDA; codes [S, M] uint8; cents [M, 256, sd]; k_counts [M].
    Returns (out [D] f32, selected token indices, exact scores of those tokens).
    """
    S, D = K.shape
    M = codes.shape[1]
    sd = sub_dim or cents.shape[-1]
    Dp = next(d for d in (32, 64, 128, 256, 1 << 30) if d >= D)
    if Dp > 256:
        raise ValueError(f"head_dim {D} > 256 is not supported by the CDC-03 kernels")
    CS = code_bytes_for(M)
    cap = int(-(-max(S, 1) // 16) * 16)
    dev = K.device
    Kp = torch.zeros((cap, Dp), dtype=torch.float32, device=dev)
    Vp = torch.zeros_like(Kp)
    Kp[:S, :D] = K
    Vp[:S, :D] = V
    qp = torch.zeros((1, 1, Dp), dtype=torch.float32, device=dev)
    qp[0, 0, :D] = q
    cp = torch.zeros((cap, CS), dtype=torch.uint8, device=dev)
    cp[:S, :M] = codes
    seq = torch.tensor([S], dtype=torch.int32, device=dev)
    out = torch.empty((1, 1, Dp), dtype=torch.float32, device=dev)
    kk = max(int(top_k), int(sink_tokens), 1)
    sel_idx = torch.empty((1, 1, kk), dtype=torch.int32, device=dev)
    sel_score = torch.empty((1, 1, kk), dtype=torch.float32, device=dev)
    sel_count = torch.empty((1, 1), dtype=torch.int32, device=dev)
    a = L.Cdc03Args()
    a.batch = a.kv_heads = a.q_per_kv = 1
    a.head_dim, a.n_subspaces, a.sub_dim, a.code_bytes, a.cb_slots = Dp, M, sd, CS, SLOTS
    a.top_k, a.sink_tokens, a.hot_window = int(top_k), int(sink_tokens), int(hot_window)
    a.scale = float(np.float32(scale))
    a.lut_order = L.DOT_GEMV
    a.q, a.q_dtype, a.q_stride_b = qp.data_ptr(), L.F32, Dp
    a.out, a.out_dtype, a.out_stride_b = out.data_ptr(), L.F32, Dp
    a.k, a.v, a.kv_dtype, a.kv_stride_b, a.kv_stride_h = Kp.data_ptr(), Vp.data_ptr(), L.F32, cap * Dp, cap * Dp
    a.capacity = cap
    a.codes, a.code_stride_b, a.code_stride_h = cp.data_ptr(), cap * CS, cap * CS
    cents = cents.contiguous()
    a.codebook, a.cb_stride_b, a.cb_stride_h = cents.data_ptr(), 0, 0
    kc = k_counts.to(torch.int32).contiguous()
    a.cb_k, a.cbk_stride_b, a.cbk_stride_h = kc.data_ptr(), 0, 0
    a.seq_len = seq.data_ptr()
    a.sel_idx, a.sel_score, a.sel_count = sel_idx.data_ptr(), sel_score.data_ptr(), sel_count.data_ptr()
    need = ctypes.c_size_t(0)
    L.check(L.lib().hokv_cdc03_workspace_size(ctypes.byref(a), ctypes.byref(need)), "cdc03_workspace_size")
    ws = L.workspace(need.value)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    L.check(L.lib().hokv_cdc03_decode(ctypes.byref(a), L.stream()), "cdc03_decode")
    L.device_status()
    n = int(sel_count[0, 0].item())
    return out[0, 0, :D], sel_idx[0, 0, :n], sel_score[0, 0, :n]
