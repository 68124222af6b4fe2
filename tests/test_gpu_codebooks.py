"""Codebook kernels on the GPU against the reference fixtures: calibration
(scalar, vector and product k-means), assignment, decoding, drift correction
and the layer-state phase machine.  Integer and index results are bit-exact;
centroids are compared bit for bit as well (the kernels follow NumPy's
reduction orders)."""

import numpy as np
import pytest
import torch

from oracle import hokv_oracle as O

pytestmark = pytest.mark.gpu


def _cfg0():
    K, V = O.gen_kv(0, 1, 4, 1024, 64)
    return O.to_fp16_values(K), O.to_fp16_values(V), O.to_fp16_values(O.gen_queries(0, 1, 32, 64))


def test_scalar_codebook_matches_reference(golden):
    from helix_online_kv.codebook import OnlineCodebook
    K, _, _ = _cfg0()
    flat = K[0].transpose(1, 0, 2).reshape(1024, 256)
    cb = OnlineCodebook(n_clusters=256, max_iters=10, rtol=1e-3)
    for t in range(128):
        cb.feed_calibration(flat[t])
    st = cb.finalize_calibration()
    np.testing.assert_array_equal(cb.centroids, golden["sc_cents"])
    gs = golden["sc_stats"]
    assert [st["n_samples"], st["n_clusters"], st["n_iters"]] == [int(x) for x in gs[:3]]
    assert st["calibration_mse"] == gs[3]
    np.testing.assert_array_equal(cb.assign(flat[128:144].ravel()), golden["sc_assign"])
    drift = flat[144:160].ravel() + 0.75
    err = cb.quantization_error(drift, cb.assign(drift))
    cb2 = OnlineCodebook(n_clusters=256, drift_threshold=0.0001)
    cb2.feed_calibration(flat[:128].ravel())
    cb2.finalize_calibration()
    assert cb2.maybe_update_centroids(drift, err)
    np.testing.assert_array_equal(cb2.centroids, golden["sc_ema"])


@pytest.mark.parametrize("seed,n,kk", [(0, 10000, 256), (1, 2000, 16), (2, 777, 64), (3, 5000, 200)])
def test_scalar_fits(golden, seed, n, kk):
    from helix_online_kv.codebook import OnlineCodebook
    rng = np.random.default_rng(100 + seed)
    d = rng.standard_normal(n).astype(np.float32)
    if seed == 3:
        d = np.round(d * 8).astype(np.float32) / 8
    c = OnlineCodebook(n_clusters=kk)
    c.feed_calibration(d)
    st = c.finalize_calibration()
    np.testing.assert_array_equal(c.centroids, golden[f"sc{seed}_cents"])
    g = golden[f"sc{seed}_stats"]
    assert st["n_clusters"] == int(g[1]) and st["n_iters"] == int(g[2]) and st["calibration_mse"] == g[3]
    test = rng.standard_normal(3000).astype(np.float32) * 1.5
    np.testing.assert_array_equal(c.assign(test), golden[f"sc{seed}_assign"])


def test_vector_codebooks(golden):
    from helix_online_kv.vector_codebook import VectorCodebook
    rng = np.random.default_rng(11)
    for tag, (n, dd, kk) in {"vq0": (128, 64, 256), "vq1": (1024, 64, 64),
                             "vq2": (300, 8, 32), "vq3": (200, 64, 16)}.items():
        data = (rng.standard_normal((n, dd)) * rng.uniform(0.5, 2, dd)).astype(np.float32)
        vq = VectorCodebook(n_clusters=kk, head_dim=dd)
        vq.feed_calibration(data)
        st = vq.finalize_calibration()
        np.testing.assert_array_equal(vq.centroids, golden[f"{tag}_cents"], err_msg=tag)
        g = golden[f"{tag}_stats"]
        assert st["n_clusters"] == int(g[1]) and st["n_iters"] == int(g[2]), tag
        assert st["calibration_mse"] == g[3], tag
        for N in (1, 3, 16, 1000):
            x = (rng.standard_normal((N, dd)) * 1.3).astype(np.float32)
            np.testing.assert_array_equal(vq.assign(x), golden[f"{tag}_assign{N}"], err_msg=f"{tag} N={N}")
        qv = rng.standard_normal(dd).astype(np.float32)
        pre = vq.precompute_query_scores(qv)
        np.testing.assert_array_equal(pre, golden[f"{tag}_qscores"])
        idx = vq.assign(data)
        np.testing.assert_array_equal(vq.gather_scores(pre, idx), pre[idx])
        np.testing.assert_allclose(vq.decode(idx), vq.centroids[idx])


def test_product_codebooks(golden):
    from helix_online_kv.product_codebook import ProductCodebook
    rng = np.random.default_rng(12)
    for tag, (n, M, kk) in {"pq0": (512, 8, 64), "pq1": (256, 16, 64), "pq2": (256, 4, 64)}.items():
        data = rng.standard_normal((n, 64)).astype(np.float32)
        pq = ProductCodebook(n_subspaces=M, sub_clusters=kk, head_dim=64)
        pq.feed_calibration(data)
        st = pq.finalize_calibration()
        np.testing.assert_array_equal(np.stack([c.centroids for c in pq._codebooks]), golden[f"{tag}_cents"])
        assert st["n_iters_per_sub"] == list(golden[f"{tag}_iters"]), tag
        assert st["calibration_mse_per_sub"] == list(golden[f"{tag}_mse"]), tag
        for N in (1, 3, 200):
            x = rng.standard_normal((N, 64)).astype(np.float32)
            np.testing.assert_array_equal(pq.assign(x), golden[f"{tag}_assign{N}"], err_msg=f"{tag} N={N}")
        qv = rng.standard_normal(64).astype(np.float32)
        T = pq.precompute_distance_tables(qv)
        np.testing.assert_array_equal(T, golden[f"{tag}_T"])
        codes = pq.assign(data)
        np.testing.assert_array_equal(pq.gather_pq_scores(T, codes), O.pq_gather(T, codes))
        np.testing.assert_array_equal(pq.decode(codes), O.pq_decode(codes, [c.centroids for c in pq._codebooks]))


@pytest.mark.parametrize("M", [8, 16])
def test_cdc03_calibration_codes(golden, M):
    """The config-0 per-head PQ fits on 128 tokens (degenerate: k = 128) and the codes of all 1024 tokens."""
    from helix_online_kv.product_codebook import ProductCodebook
    K, _, _ = _cfg0()
    for h in (range(4) if M == 8 else range(2)):
        pq = ProductCodebook(n_subspaces=M, sub_clusters=256, head_dim=64)
        pq.feed_calibration(K[0, h, :128])
        st = pq.finalize_calibration()
        assert st["sub_clusters"] == list(golden[f"c0m{M}_h{h}_k"])
        gc = golden[f"c0m{M}_h{h}_cents"]
        for s, cb in enumerate(pq._codebooks):
            np.testing.assert_array_equal(cb.centroids, gc[s, :len(cb.centroids)])
        np.testing.assert_array_equal(pq.assign(K[0, h]), golden[f"c0m{M}_h{h}_codes"])


def test_layer_state_matches_reference(golden):
    from helix_online_kv.config import OnlineKVConfig
    from helix_online_kv.layer_state import KVLayerState
    cfg = OnlineKVConfig(calibration_tokens=16, n_clusters=64, exact_layers=[])
    rng = np.random.default_rng(5)
    toks = rng.standard_normal((40, 2, 256)).astype(np.float32)
    ls = KVLayerState(1, cfg)
    res = [ls.feed_token(toks[t, 0], toks[t, 1]) for t in range(40)]
    assert [r is not None for r in res].index(True) == 15
    np.testing.assert_array_equal(ls.k_codebook.centroids, golden["ls_k_cents"])
    np.testing.assert_array_equal(ls.v_codebook.centroids, golden["ls_v_cents"])
    np.testing.assert_array_equal(np.stack(ls._k_indices), golden["ls_k_idx"])
    np.testing.assert_array_equal(np.stack(ls._v_indices), golden["ls_v_idx"])
    assert ls.compressed_token_count == 24
    mem = ls.memory_bytes()
    assert [mem[k] for k in ("codebook_bytes", "index_bytes", "total_bytes")] == list(golden["ls_mem"])
    # the batched device form gives the same indices
    ls2 = KVLayerState(1, cfg)
    kd = torch.from_numpy(toks[:, 0]).cuda()
    vd = torch.from_numpy(toks[:, 1]).cuda()
    out = ls2.feed_tokens(kd[:10], vd[:10]) + ls2.feed_tokens(kd[10:], vd[10:])
    assert len(out) == 1 and ls2.is_streaming
    np.testing.assert_array_equal(ls2.get_all_compressed_k().cpu().numpy(),
                                  ls.k_codebook.centroids[golden["ls_k_idx"]])


def test_codebook_quality_properties():
    """Reference test semantics: roundtrip cosine, generalization, MSE monotone in k."""
    from helix_online_kv.codebook import OnlineCodebook
    from helix_online_kv.vector_codebook import VectorCodebook
    rng = np.random.default_rng(42)
    data = rng.standard_normal(10000).astype(np.float32)
    cb = OnlineCodebook(n_clusters=256)
    cb.feed_calibration(data[:2000])
    cb.finalize_calibration()
    idx = cb.assign(data[2000:])
    assert cb.cosine_similarity(data[2000:], idx) > 0.998
    errs = []
    for k in (16, 64, 256):
        c = OnlineCodebook(n_clusters=k)
        c.feed_calibration(data[:2000])
        c.finalize_calibration()
        errs.append(c.quantization_error(data[2000:5000], c.assign(data[2000:5000])))
    assert errs[0] > errs[1] > errs[2]
    vq = VectorCodebook(n_clusters=256, head_dim=64)
    vq.feed_calibration(rng.standard_normal((50, 64)).astype(np.float32))
    assert vq.finalize_calibration()["n_clusters"] <= 50
    with pytest.raises(RuntimeError, match="already finalized"):
        vq.feed_calibration(rng.standard_normal((5, 64)).astype(np.float32))


def test_vector_gather_scores_equal_decode_dot():
    """VectorCodebook: precomputed query scores gathered by index equal the dot
    products with the decoded vectors (the reference's rtol 1e-5 identity)."""
    from helix_online_kv.vector_codebook import VectorCodebook
    rng = np.random.default_rng(7)
    x = rng.standard_normal((600, 64)).astype(np.float32)
    vq = VectorCodebook(n_clusters=64, head_dim=64)
    vq.feed_calibration(x[:300])
    vq.finalize_calibration()
    idx = vq.assign(x[300:])
    assert idx.shape == (300,) and idx.dtype == np.uint8
    q = rng.standard_normal(64).astype(np.float32)
    got = vq.gather_scores(vq.precompute_query_scores(q), idx)
    np.testing.assert_allclose(got, vq.decode(idx) @ q, rtol=1e-5, atol=1e-6)
    with pytest.raises(ValueError, match="Expected shape"):
        vq.assign(rng.standard_normal((4, 32)).astype(np.float32))


@pytest.mark.parametrize("M", [4, 8, 16])
def test_product_adc_equals_decode_dot(M):
    """ProductCodebook: [N, M] uint8 codes; ADC scores from the distance tables
    match the dot with the decoded vectors (rtol 1e-4, atol 1e-5)."""
    from helix_online_kv.product_codebook import ProductCodebook
    rng = np.random.default_rng(11 + M)
    x = rng.standard_normal((800, 64)).astype(np.float32)
    pq = ProductCodebook(n_subspaces=M, sub_clusters=64, head_dim=64)
    pq.feed_calibration(x[:400])
    pq.finalize_calibration()
    codes = pq.assign(x[400:])
    assert codes.shape == (400, M) and codes.dtype == np.uint8
    q = rng.standard_normal(64).astype(np.float32)
    adc = pq.gather_pq_scores(pq.precompute_distance_tables(q), codes)
    np.testing.assert_allclose(adc, pq.decode(codes) @ q, rtol=1e-4, atol=1e-5)
    with pytest.raises(ValueError, match="divisible"):
        ProductCodebook(n_subspaces=7, head_dim=64)


def test_product_beats_vector_quantisation():
    """At the same codes per subspace, PQ reconstructs better than one VQ codebook."""
    from helix_online_kv.product_codebook import ProductCodebook
    from helix_online_kv.vector_codebook import VectorCodebook
    rng = np.random.default_rng(3)
    x = rng.standard_normal((1500, 64)).astype(np.float32)
    vq = VectorCodebook(n_clusters=64, head_dim=64)
    vq.feed_calibration(x[:1000])
    vq.finalize_calibration()
    pq = ProductCodebook(n_subspaces=8, sub_clusters=64, head_dim=64)
    pq.feed_calibration(x[:1000])
    pq.finalize_calibration()
    test = x[1000:]
    assert pq.quantization_error(test, pq.assign(test)) < vq.quantization_error(test, vq.assign(test))


def test_scalar_drift_update():
    """EMA drift correction runs only above the threshold and moves the centroids."""
    from helix_online_kv.codebook import OnlineCodebook
    rng = np.random.default_rng(5)
    cb = OnlineCodebook(n_clusters=16)
    cb.feed_calibration(rng.standard_normal(4000).astype(np.float32))
    cb.finalize_calibration()
    before = cb.centroids.copy()
    assert not cb.maybe_update_centroids(rng.standard_normal(100).astype(np.float32), error=0.0)
    np.testing.assert_array_equal(cb.centroids, before)
    shifted = (rng.standard_normal(4000) + 3.0).astype(np.float32)
    assert cb.maybe_update_centroids(shifted, error=1.0)
    assert not np.array_equal(cb.centroids, before)
    assert cb.centroids.mean() > before.mean()


def test_layer_state_lifecycle():
    """KVLayerState: phase change at exactly calibration_tokens, compressed
    count, decoded tokens close to the originals, memory accounting."""
    from helix_online_kv.config import OnlineKVConfig
    from helix_online_kv.layer_state import KVLayerState
    rng = np.random.default_rng(17)
    cfg = OnlineKVConfig(calibration_tokens=32, exact_layers=[0])
    ls = KVLayerState(1, cfg)
    dim = 2 * 64
    toks = rng.standard_normal((80, 2, dim)).astype(np.float32)
    for i in range(32):
        assert ls.is_calibrating
        ls.feed_token(toks[i, 0], toks[i, 1])
    assert ls.is_streaming and ls.compressed_token_count == 0
    for i in range(32, 80):
        ls.feed_token(toks[i, 0], toks[i, 1])
    assert ls.compressed_token_count == 48 and ls.tokens_seen == 80
    k, v = ls.get_compressed_kv(10)
    kt = np.asarray(k.cpu() if hasattr(k, "cpu") else k, dtype=np.float32)
    cos = float(kt @ toks[42, 0] / (np.linalg.norm(kt) * np.linalg.norm(toks[42, 0])))
    assert cos > 0.99
    mem = ls.memory_bytes()
    assert mem["index_bytes"] == 48 * 2 * dim and mem["total_bytes"] == mem["codebook_bytes"] + mem["index_bytes"]
    assert KVLayerState(0, cfg).memory_bytes()["total_bytes"] == 0


def test_store_calibration_matches_product_codebook():
    """CDC03Store.calibrate fits every (sequence, head, subspace) in one launch;
    each fit equals ProductCodebook's on the same calibration tokens."""
    from helix_online_kv.cdc03 import CDC03Store
    from helix_online_kv.product_codebook import ProductCodebook
    K, V = O.gen_kv(29, 2, 3, 300, 64)
    st = CDC03Store(2, 1, 3, 64, 300, n_subspaces=8, dtype=torch.float16)
    st.k[0, :, :, :300] = torch.from_numpy(K).half().cuda()
    st.calibrate(0, 128)
    for b in range(2):
        for h in range(3):
            pq = ProductCodebook(n_subspaces=8, sub_clusters=256, head_dim=64)
            pq.feed_calibration(st.k[0, b, h, :128].float().cpu().numpy())
            info = pq.finalize_calibration()
            kk = st.cb_k[0, b, h].cpu().numpy()
            assert list(kk) == list(info["sub_clusters"])
            for s, cb in enumerate(pq._codebooks):
                np.testing.assert_array_equal(st.codebook[0, b, h, s, :kk[s]].cpu().numpy(), cb.centroids)
