"""hokv_cdc03_decode_noalloc: CDC-03 decode without any device allocation.

Some callers cannot allocate device memory: a plugin inside a serving runtime
that has reserved nearly all HBM for its own KV pool and offers no allocator.
For them the library keeps one fixed scratch array per device and this entry
point uses it instead of a caller workspace.  These tests call it through the
C ABI and compare it with hokv_cdc03_decode (caller workspace) on the same
inputs, on two calls in a row with different shapes, so the second call runs
on scratch that still holds the first call's contents.

The file is named to be collected last.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import hokv_oracle as O

pytestmark = pytest.mark.gpu

ATOL = 1e-2   # output tolerance of the other CDC-03 tests


def _store(B, Hkv, G, D, S, M, seq_lens, seed):
    from helix_online_kv.cdc03 import CDC03Store
    K, V = O.gen_kv(seed, B, Hkv, S, D)
    Q = O.gen_queries(seed, B, Hkv * G, D)
    st = CDC03Store(B, 1, Hkv, D, S, n_subspaces=M, dtype=torch.bfloat16)
    st.k[0, :, :, :S] = torch.from_numpy(K).to(torch.bfloat16).cuda()
    st.v[0, :, :, :S] = torch.from_numpy(V).to(torch.bfloat16).cuda()
    st.seq_len.copy_(torch.tensor(seq_lens, dtype=torch.int32))
    st.calibrate(0, 128)
    st.assign(0, 0, S)
    return st, torch.from_numpy(Q).to(torch.bfloat16).cuda()


def _run(st, q, entry, top_k=128, sink=4, hot=256):
    from helix_online_kv import _lib as L
    B, Hq, _ = q.shape
    cap = max(top_k, sink, 1)
    out = torch.full(q.shape, float("nan"), dtype=torch.float32, device=q.device)
    sel = torch.full((B, Hq, cap), -7, dtype=torch.int32, device=q.device)
    cnt = torch.full((B, Hq), -7, dtype=torch.int32, device=q.device)
    a = st.args(0, q, out, 1 / np.sqrt(q.shape[-1]), top_k, sink, hot, sel_idx=sel, sel_count=cnt)
    L.check(getattr(L.lib(), entry)(ctypes.byref(a), L.stream()), entry)
    torch.cuda.synchronize()
    L.device_status()
    return out, sel, cnt


def _compare(ref, got, label):
    out_r, sel_r, cnt_r = ref
    out_g, sel_g, cnt_g = got
    assert torch.equal(cnt_g, cnt_r), f"{label}: selected counts differ"
    for b in range(cnt_r.shape[0]):
        for hq in range(cnt_r.shape[1]):
            n = int(cnt_r[b, hq])
            a = np.sort(sel_r[b, hq, :n].cpu().numpy())
            g = np.sort(sel_g[b, hq, :n].cpu().numpy())
            assert np.array_equal(a, g), f"{label}: selection of b{b} hq{hq} differs"
    assert torch.isfinite(out_g).all(), f"{label}: non-finite output"
    assert torch.allclose(out_g, out_r, atol=ATOL, rtol=0), f"{label}: max diff {(out_g - out_r).abs().max()}"


def test_noalloc_matches_workspace_entry_point_twice():
    from helix_online_kv import _lib as L
    L.require_device()
    # call 1: 2 sequences x 2 KV heads x 4 query heads, 5000 / 3333 tokens
    st1, q1 = _store(2, 2, 4, 128, 5000, 16, [5000, 3333], seed=21)
    ref1 = _run(st1, q1, "hokv_cdc03_decode")
    got1 = _run(st1, q1, "hokv_cdc03_decode_noalloc")
    _compare(ref1, got1, "call 1")
    # call 2, straight after: another geometry (16K tokens, 8 query heads per
    # KV head), so the shared scratch still holds call 1's candidates
    st2, q2 = _store(1, 2, 8, 64, 16384, 8, [16384], seed=22)
    got2 = _run(st2, q2, "hokv_cdc03_decode_noalloc")
    ref2 = _run(st2, q2, "hokv_cdc03_decode")
    _compare(ref2, got2, "call 2")


def test_noalloc_rejects_configurations_beyond_its_scratch():
    from helix_online_kv import _lib as L
    L.require_device()
    st, q = _store(2, 2, 4, 128, 5000, 16, [5000, 5000], seed=23)
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    a = st.args(0, q, out, 0.088, 128, 4, 256)
    a.batch = 64   # 128 (sequence, KV head) units: more scratch than the library holds (never launched)
    need = ctypes.c_size_t(0)
    assert L.lib().hokv_cdc03_workspace_size(ctypes.byref(a), ctypes.byref(need)) == 0
    assert need.value > 16 << 20
    st_code = L.lib().hokv_cdc03_decode_noalloc(ctypes.byref(a), L.stream())
    assert st_code == 6, st_code   # HOKV_ERR_WORKSPACE
    msg = L.lib().hokv_last_error().decode()
    assert "scratch" in msg and str(need.value) in msg, msg
