"""Pin the CPU oracle to the reference: every golden fixture is reproduced.

The fixtures were written by running the reference package itself
(``tests/golden/make_golden.py``).  Where the reference result passes through
BLAS, equality holds on the BLAS build recorded in ``versions.json``; on other
hosts a last-ulp difference is allowed and counted.
"""

import json
import os

import numpy as np
import pytest

from oracle import hokv_oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
with open(os.path.join(HERE, "golden", "versions.json")) as _f:
    _V = json.load(_f)
SAME_BLAS = (np.__version__ == _V["numpy"])


def _cfg0():
    B, Hkv, Hq, D, S = 1, 4, 32, 64, 1024
    K, V = O.gen_kv(0, B, Hkv, S, D)
    Q = O.gen_queries(0, B, Hq, D)
    return O.to_fp16_values(K), O.to_fp16_values(V), O.to_fp16_values(Q)


def test_input_generator_frozen(golden):
    import hashlib
    K, V, Q = _cfg0()
    m = hashlib.sha256()
    for a in (K, V, Q):
        m.update(np.ascontiguousarray(a).tobytes())
    assert m.hexdigest()[:16] == str(golden["c0_input_hash"])


@pytest.mark.parametrize("M", [8, 16])
def test_pq_calibration_and_cdc03(golden, M):
    K, V, Q = _cfg0()
    scale = 1.0 / np.sqrt(64)
    heads = range(4) if M == 8 else range(2)
    for h in heads:
        cents, fits = O.pq_fit(K[0, h, :128], M=M, sub_clusters=256)
        k = golden[f"c0m{M}_h{h}_k"]
        gc = golden[f"c0m{M}_h{h}_cents"]
        for s in range(M):
            assert len(cents[s]) == k[s]
            np.testing.assert_array_equal(cents[s], gc[s, :k[s]])
        assert [f[2] for f in fits] == list(golden[f"c0m{M}_h{h}_iters"])
        codes = O.pq_assign(K[0, h], cents)
        np.testing.assert_array_equal(codes, golden[f"c0m{M}_h{h}_codes"])
        for qi in range(8):
            hq = h * 8 + qi
            q = Q[0, hq]
            pre = f"c0m{M}_q{hq}"
            T = O.pq_tables(q, cents)
            if qi < 2:
                np.testing.assert_array_equal(T, golden[pre + "_T"])
            approx = O.pq_gather(T, codes) * np.float32(scale)
            np.testing.assert_array_equal(approx, golden[pre + "_approx"])
            sc, out, meta = O.hybrid_pq_attention(q, K[0, h], V[0, h], codes, cents, scale,
                                                  top_k=128, sink_tokens=4)
            np.testing.assert_array_equal(np.flatnonzero(np.isfinite(sc)), golden[pre + "_sel"])
            np.testing.assert_array_equal(out, golden[pre + "_out"])
            gm = golden[pre + "_meta"]
            assert meta["selected_count"] == gm[0] and meta["pq_score_range"] == gm[2]
            # canonical (lowest-index) tie rule agrees with argpartition here
            np.testing.assert_array_equal(
                O.cdc03_select_canonical(approx, 128, 4), O.cdc03_select(approx, 128, 4))
            if M == 8:
                sel, _, o_hot = O.cdc03_hot_attention(q, K[0, h], V[0, h], codes, cents, scale,
                                                      top_k=128, sink_tokens=4, hot_window=256)
                np.testing.assert_array_equal(sel, golden[pre + "_hot_sel"])
                np.testing.assert_allclose(o_hot, golden[pre + "_hot_out"], rtol=1e-5, atol=1e-6)


def test_hot_window_zero_is_hybrid(golden):
    K, V, Q = _cfg0()
    scale = 1.0 / np.sqrt(64)
    cents, _ = O.pq_fit(K[0, 0, :128], M=8)
    codes = O.pq_assign(K[0, 0], cents)
    for hq in range(4):
        sel, _, out = O.cdc03_hot_attention(Q[0, hq], K[0, 0], V[0, 0], codes, cents, scale,
                                            top_k=128, sink_tokens=4, hot_window=0,
                                            select=O.cdc03_select)
        np.testing.assert_array_equal(sel, golden[f"c0m8_q{hq}_sel"])
        np.testing.assert_array_equal(out, golden[f"c0m8_q{hq}_out"])


def test_scalar_codebook(golden):
    K, _, _ = _cfg0()
    flat = K[0].transpose(1, 0, 2).reshape(1024, 256)
    cents, assign, it = O.scalar_fit(flat[:128].ravel(), 256, 10, 1e-3)
    np.testing.assert_array_equal(cents, golden["sc_cents"])
    st = O.scalar_finalize_stats(flat[:128].ravel(), cents, assign, it)
    gs = golden["sc_stats"]
    assert [st["n_samples"], st["n_clusters"], st["n_iters"]] == list(gs[:3].astype(int))
    assert st["calibration_mse"] == gs[3]
    np.testing.assert_array_equal(O.scalar_assign(flat[128:144], cents), golden["sc_assign"])
    drift = flat[144:160].ravel() + 0.75
    np.testing.assert_array_equal(O.scalar_ema_update(drift, cents, 0.05), golden["sc_ema"])
    for seed, (n, kk) in enumerate([(10000, 256), (2000, 16), (777, 64), (5000, 200)]):
        rng = np.random.default_rng(100 + seed)
        d = rng.standard_normal(n).astype(np.float32)
        if seed == 3:
            d = np.round(d * 8).astype(np.float32) / 8
        c, a, it = O.scalar_fit(d, kk)
        np.testing.assert_array_equal(c, golden[f"sc{seed}_cents"])
        assert it == int(golden[f"sc{seed}_stats"][2])
        test = rng.standard_normal(3000).astype(np.float32) * 1.5
        np.testing.assert_array_equal(O.scalar_assign(test, c), golden[f"sc{seed}_assign"])


def test_vector_codebook(golden):
    rng = np.random.default_rng(11)
    for tag, (n, dd, kk) in {"vq0": (128, 64, 256), "vq1": (1024, 64, 64),
                             "vq2": (300, 8, 32), "vq3": (200, 64, 16)}.items():
        data = (rng.standard_normal((n, dd)) * rng.uniform(0.5, 2, dd)).astype(np.float32)
        c, a, it = O.vq_fit(data, kk)
        np.testing.assert_array_equal(c, golden[f"{tag}_cents"])
        assert it == int(golden[f"{tag}_stats"][2])
        for N in (1, 3, 16, 1000):
            x = (rng.standard_normal((N, dd)) * 1.3).astype(np.float32)
            np.testing.assert_array_equal(O.vq_assign(x, c), golden[f"{tag}_assign{N}"])
        qv = rng.standard_normal(dd).astype(np.float32)
        np.testing.assert_array_equal(qv @ c.T, golden[f"{tag}_qscores"])


def test_product_codebook(golden):
    rng = np.random.default_rng(12)
    for tag, (n, M, kk) in {"pq0": (512, 8, 64), "pq1": (256, 16, 64), "pq2": (256, 4, 64)}.items():
        data = rng.standard_normal((n, 64)).astype(np.float32)
        cents, fits = O.pq_fit(data, M, kk)
        np.testing.assert_array_equal(np.stack(cents), golden[f"{tag}_cents"])
        assert [f[2] for f in fits] == list(golden[f"{tag}_iters"])
        for N in (1, 3, 200):
            x = rng.standard_normal((N, 64)).astype(np.float32)
            np.testing.assert_array_equal(O.pq_assign(x, cents), golden[f"{tag}_assign{N}"])
        qv = rng.standard_normal(64).astype(np.float32)
        np.testing.assert_array_equal(O.pq_tables(qv, cents), golden[f"{tag}_T"])


def test_attention_paths(golden):
    rng = np.random.default_rng(42)
    q = rng.standard_normal(64).astype(np.float32)
    Ks = rng.standard_normal((200, 64)).astype(np.float32)
    Vs = rng.standard_normal((200, 64)).astype(np.float32)
    sc = 1.0 / np.sqrt(64)
    ck, _, _ = O.vq_fit(Ks, 64)
    kidx = O.vq_assign(Ks, ck)
    cv, _, _ = O.vq_fit(Vs, 64)
    vidx = O.vq_assign(Vs, cv)
    np.testing.assert_array_equal(kidx, golden["pathB_kidx"])
    s = O.vector_vq_attention_scores(q, kidx, ck, sc)
    from scipy.special import softmax
    o = O.vector_vq_value_output(softmax(s), vidx, cv)
    np.testing.assert_array_equal(s, golden["pathB_scores"])
    np.testing.assert_array_equal(o, golden["pathB_out"])
    pk, _ = O.pq_fit(Ks, 8, 64)
    pv, _ = O.pq_fit(Vs, 8, 64)
    s = O.pq_attention_scores(q, O.pq_assign(Ks, pk), pk, sc)
    o = O.pq_value_output(softmax(s), O.pq_assign(Vs, pv), pv)
    np.testing.assert_array_equal(s, golden["pathD_scores"])
    np.testing.assert_array_equal(o, golden["pathD_out"])
    s, o = O.prefiltered_attention(q, Ks, Vs, kidx, ck, sc, top_p=16)
    np.testing.assert_array_equal(s, golden["pathF_scores"])
    np.testing.assert_array_equal(o, golden["pathF_out"])
    c, _, _ = O.scalar_fit(Ks.ravel(), 256)
    ki = O.scalar_assign(Ks.ravel(), c).reshape(Ks.shape)
    np.testing.assert_array_equal(O.fused_scalar_vq_qkt_numpy(q, ki, c, sc), golden["pathA_qkt"])
    s, o = O.scalar_vq_attention(q, ki, c, Vs, sc)
    np.testing.assert_array_equal(s, golden["pathA_scores"])
    s, o = O.standard_attention(q, Ks, Vs, sc)
    np.testing.assert_array_equal(o, golden["std_out"])


def test_tier_boundary():
    assert O.tier_boundary(100, 256) == 0
    assert O.tier_boundary(256, 256) == 0
    assert O.tier_boundary(257, 256) == 1
    assert O.tier_boundary(1024, 128) == 896
    assert O.tier_boundary(1000, 256, min_age=128) == 872
