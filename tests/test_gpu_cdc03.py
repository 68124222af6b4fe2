"""CDC-03 decode attention on the GPU against the reference and the oracle.

Selection parity: the selected token set equals the reference's
(compressed_attention.py:366-388) bit for bit; where the host's BLAS gives a
sub-table entry one ulp away from the device's, a differing token must be a
near-tie (its reference score within 8 ulp of the boundary score) and such
tokens are counted.  Output parity: max-abs <= 1e-2 and cosine >= 0.9999
against the oracle's exact attention over the same fp16/bf16 values.
"""

import numpy as np
import pytest
import torch

from oracle import hokv_oracle as O

pytestmark = pytest.mark.gpu

ATOL, COS = 1e-2, 0.9999


def _assert_selection(got, approx, top_k, sink, label=""):
    """got: selected cold indices from the device; approx: reference f32 PQ scores."""
    ref = O.cdc03_select_canonical(approx, top_k, sink)
    got = np.sort(np.asarray(got))
    if np.array_equal(got, ref):
        return 0
    n = approx.shape[0]
    k = min(top_k, n)
    sink_n = min(sink, n)
    diff = np.setxor1d(got, ref)
    if k >= n or k - sink_n <= 0:
        raise AssertionError(f"{label}: selection differs in a no-ranking case: {diff}")
    masked = approx.astype(np.float64).copy()
    masked[:sink_n] = -np.inf
    boundary = np.sort(masked)[-(k - sink_n)]
    tol = 8 * np.spacing(np.float32(abs(boundary)))
    bad = [t for t in diff if abs(float(approx[t]) - boundary) > tol]
    assert not bad and len(diff) <= 4, f"{label}: non-tie selection differences {bad} (diff {diff})"
    return len(diff)


def _out_ok(o, ref, label=""):
    assert np.max(np.abs(o - ref)) <= ATOL, f"{label}: max-abs {np.max(np.abs(o - ref))}"
    assert O.cosine(o, ref) >= COS, f"{label}: cosine {O.cosine(o, ref)}"


def test_hybrid_pq_attention_matches_reference(golden):
    """The NumPy-facing Path G on config 0 (M = 8 and 16) against the reference run."""
    from helix_online_kv.compressed_attention import hybrid_pq_attention
    from helix_online_kv.product_codebook import ProductCodebook
    K, V = O.gen_kv(0, 1, 4, 1024, 64)
    K, V = O.to_fp16_values(K), O.to_fp16_values(V)
    Q = O.to_fp16_values(O.gen_queries(0, 1, 32, 64))
    scale = 1.0 / np.sqrt(64)
    ties = 0
    for M in (8, 16):
        for h in (range(4) if M == 8 else range(2)):
            pq = ProductCodebook(n_subspaces=M, sub_clusters=256, head_dim=64)
            pq.feed_calibration(K[0, h, :128])
            pq.finalize_calibration()
            codes = pq.assign(K[0, h])
            for qi in range(8):
                hq = h * 8 + qi
                pre = f"c0m{M}_q{hq}"
                sc, out, meta = hybrid_pq_attention(Q[0, hq], K[0, h], V[0, h], codes, pq, scale,
                                                    top_k=128, sink_tokens=4)
                sel = np.flatnonzero(np.isfinite(sc))
                ties += _assert_selection(sel, golden[pre + "_approx"], 128, 4, pre)
                np.testing.assert_allclose(out, golden[pre + "_out"], atol=1e-5, rtol=1e-4)
                gm = golden[pre + "_meta"]
                assert meta["selected_count"] == int(gm[0]) and meta["sink_count"] == int(gm[3])
                assert meta["pq_score_range"] == pytest.approx(gm[2], rel=1e-6)
                # exact scores at the selected positions
                ref_s, _ = O.standard_attention(Q[0, hq], K[0, h, sel], V[0, h, sel], scale)
                np.testing.assert_allclose(sc[sel], ref_s, rtol=1e-5, atol=1e-6)
    assert ties <= 4


def test_hybrid_reference_semantics():
    """Reference test semantics: shapes, selected_count, full coverage == standard,
    monotone in top_k, single token."""
    from helix_online_kv.compressed_attention import hybrid_pq_attention, standard_attention
    from helix_online_kv.product_codebook import ProductCodebook
    rng = np.random.default_rng(42)
    q = rng.standard_normal(64).astype(np.float32)
    K = rng.standard_normal((200, 64)).astype(np.float32)
    V = rng.standard_normal((200, 64)).astype(np.float32)
    scale = 1.0 / np.sqrt(64)
    pq = ProductCodebook(n_subspaces=8, sub_clusters=64, head_dim=64)
    pq.feed_calibration(K)
    pq.finalize_calibration()
    idx = pq.assign(K)
    scores, out, meta = hybrid_pq_attention(q, K, V, idx, pq, scale, top_k=64)
    assert scores.shape == (200,) and out.shape == (64,) and meta["selected_count"] == 64
    _, ref = standard_attention(q, K, V, scale)
    _, full, _ = hybrid_pq_attention(q, K, V, idx, pq, scale, top_k=200)
    assert O.cosine(full, ref) > 0.9999
    pq16 = ProductCodebook(n_subspaces=16, sub_clusters=64, head_dim=64)
    pq16.feed_calibration(K)
    pq16.finalize_calibration()
    idx16 = pq16.assign(K)
    cos = [O.cosine(hybrid_pq_attention(q, K, V, idx16, pq16, scale, top_k=tk)[1], ref) for tk in (32, 64, 128, 200)]
    assert all(cos[i] <= cos[i + 1] + 1e-6 for i in range(3)), cos
    # top_k below the sink count keeps the sinks, top_k = 0 as well
    s0, _, m0 = hybrid_pq_attention(q, K, V, idx, pq, scale, top_k=0, sink_tokens=4)
    assert m0["selected_count"] == 4 and np.isfinite(s0[:4]).all() and not np.isfinite(s0[4:]).any()


def _store(B, Hkv, G, D, S, M, dtype, seed=0, seq_lens=None, hot=256, cal=128):
    from helix_online_kv.cdc03 import CDC03Store
    K, V = O.gen_kv(seed, B, Hkv, S, D)
    Q = O.gen_queries(seed, B, Hkv * G, D)
    st = CDC03Store(B, 1, Hkv, D, S, n_subspaces=M, dtype=dtype)
    st.k[0, :, :, :S] = torch.from_numpy(K).to(dtype).cuda()
    st.v[0, :, :, :S] = torch.from_numpy(V).to(dtype).cuda()
    lens = seq_lens if seq_lens is not None else [S] * B
    st.seq_len.copy_(torch.tensor(lens, dtype=torch.int32))
    st.calibrate(0, cal)
    st.assign(0, 0, S)
    return st, torch.from_numpy(Q).to(dtype).cuda(), lens


def _check_store(st, q, lens, scale, top_k, sink, hot, label, exclude_rows=None):
    out, (sel, ssc, cnt) = st.decode(0, q, scale, top_k, sink, hot, out_dtype=torch.float32, return_selection=True)
    torch.cuda.synchronize()
    from helix_online_kv import _lib
    _lib.device_status()
    B, Hq, D = q.shape
    G = Hq // st.H
    ties = 0
    for b in range(B):
        S = lens[b]
        for h in range(st.H):
            Kh = st.k[0, b, h, :S].float().cpu().numpy()
            Vh = st.v[0, b, h, :S].float().cpu().numpy()
            kk = st.cb_k[0, b, h].cpu().numpy()
            cbk = st.codebook[0, b, h].cpu().numpy()
            cents = [cbk[s, :kk[s]] for s in range(st.M)]
            codes = st.codes[0, b, h, :S, :st.M].cpu().numpy()
            # the codes the decode reads: the cold range (rows aged one at a
            # time are checked against a one-token assign by their own test)
            Sc = max(0, S - hot)
            rows = [t for t in range(Sc) if t not in (exclude_rows or {}).get(b, ())]
            np.testing.assert_array_equal(codes[rows], O.pq_assign(Kh, cents)[rows], err_msg=f"{label} codes b{b} h{h}")
            for g in range(G):
                hq = h * G + g
                qv = q[b, hq].float().cpu().numpy()
                Sc = max(0, S - hot)
                n = int(cnt[b, hq])
                got = sel[b, hq, :n].cpu().numpy()
                if Sc > 0:
                    approx = O.pq_gather(O.pq_tables(qv, cents), codes[:Sc]) * np.float32(scale)
                    ties += _assert_selection(got, approx, top_k, sink, f"{label} b{b} hq{hq}")
                else:
                    assert n == 0
                union = np.concatenate([np.sort(got), np.arange(Sc, S)]).astype(int)
                ex = (qv @ Kh[union].T) * scale
                w = np.exp(ex - ex.max())
                ref = (w / w.sum()) @ Vh[union]
                _out_ok(out[b, hq].cpu().numpy(), ref, f"{label} b{b} hq{hq}")
                np.testing.assert_allclose(ssc[b, hq, :n].cpu().numpy(), (qv @ Kh[got].T) * scale,
                                           rtol=1e-4, atol=1e-5)
    return ties


def test_store_config0_gqa():
    """Config 0 (B=1, 4 KV heads, 32 query heads, D=64, S=1024, M=8, top-128, hot 256), fp16."""
    st, q, lens = _store(1, 4, 8, 64, 1024, 8, torch.float16)
    assert _check_store(st, q, lens, 1 / 8, 128, 4, 256, "cfg0") <= 4


def test_store_llama3_geometry_bf16():
    """Llama-3 geometry: 8 KV heads -> here 2, G=4, D=128, M=16, bf16, ragged lengths."""
    st, q, lens = _store(2, 2, 4, 128, 5000, 16, torch.bfloat16, seed=3, seq_lens=[5000, 3333])
    assert _check_store(st, q, lens, 1 / np.sqrt(128), 128, 4, 256, "llama3") <= 4


def test_store_long_context_16k():
    """16K-token context at the north-star geometry (one sequence, one KV head pair)."""
    st, q, lens = _store(1, 2, 4, 128, 16384, 16, torch.bfloat16, seed=5)
    assert _check_store(st, q, lens, 1 / np.sqrt(128), 128, 4, 256, "16k") <= 4


def test_store_long_context_20k_two_pass_chunks():
    """20K tokens: 10 chunks over a cluster of 8 CTAs, so two CTAs score two
    chunks each, once for the histogram and again for the candidate list."""
    st, q, lens = _store(1, 1, 4, 128, 20000, 16, torch.bfloat16, seed=11)
    assert _check_store(st, q, lens, 1 / np.sqrt(128), 128, 4, 256, "20k") <= 4


def test_store_long_context_64k():
    """64K tokens: 32 chunks, four per CTA of the cluster, one unit-wide threshold."""
    st, q, lens = _store(1, 1, 2, 64, 65536, 8, torch.float16, seed=19)
    assert _check_store(st, q, lens, 0.125, 128, 4, 256, "64k") <= 4


@pytest.mark.parametrize("top_k", [300, 600])
def test_store_16k_list_sizes(top_k):
    """16K tokens, 8 chunks: top-300 leaves 33 to 64 candidates per chunk (the
    attention stage reads each chunk's count with its first 64 keys, two per
    lane); top-600 leaves more than 64 (counts first, then the keys)."""
    st, q, lens = _store(1, 1, 2, 64, 16384, 8, torch.float16, seed=23)
    assert _check_store(st, q, lens, 0.125, top_k, 4, 256, f"16k top{top_k}") <= 4


@pytest.mark.parametrize("top_k", [128, 500])
def test_store_30k_two_chunks_per_warp(top_k):
    """30K tokens, 15 chunks: the attention stage reads two chunks per warp
    with 32 list slots each; top-500 leaves more than 32 candidates in some
    chunks, which then take the counts-first path."""
    st, q, lens = _store(1, 1, 2, 64, 30000, 8, torch.float16, seed=37)
    assert _check_store(st, q, lens, 0.125, top_k, 4, 256, f"30k top{top_k}") <= 4


def test_store_more_than_128_live_centroids():
    """Codebooks calibrated on 300 tokens keep up to 256 live centroids per
    subspace: the candidate stage reads the rows past the first 128 in a
    second copy, once it has the live counts."""
    st, q, lens = _store(1, 2, 4, 128, 5000, 16, torch.bfloat16, seed=29, cal=300)
    assert int(st.cb_k[0].max()) > 128
    assert _check_store(st, q, lens, 1 / np.sqrt(128), 128, 4, 256, "cal300") <= 4


@pytest.mark.parametrize("D,M,dtype", [
    (256, 16, torch.float16),    # 8 dims per lane, a whole warp per row
    (32, 8, torch.bfloat16),     # 8 dims per lane, 4 lanes per row, 8 rows per warp step
    (128, 16, torch.float32),    # fp32 K/V: 4 dims (16 bytes) per lane
    (256, 32, torch.float32),    # fp32 K/V, 32-byte row slices, 32-byte code rows
])
def test_store_head_dims_and_kv_dtypes(D, M, dtype):
    """Head dims 32 and 256 and fp32 K/V stores: the attention loop's per-lane
    row slices and the code widths that the 16K workload does not reach."""
    st, q, lens = _store(1, 2, 4, D, 3000, M, dtype, seed=D + M, seq_lens=[2900])
    assert _check_store(st, q, lens, 1 / np.sqrt(D), 128, 4, 256, f"D{D} M{M} {dtype}") <= 4


def test_store_group_of_three_uneven_cluster():
    """G = 3 query heads per KV head (one padded score lane) and 3 chunks per
    unit, so the cluster splits 4 subspace groups unevenly over 3 CTAs."""
    st, q, lens = _store(2, 2, 3, 64, 5000, 8, torch.float16, seed=13, seq_lens=[5000, 4100])
    assert _check_store(st, q, lens, 0.125, 128, 4, 256, "g3") <= 4


@pytest.mark.parametrize("S,top_k,sink,hot", [
    (100, 128, 4, 256),    # shorter than the hot window: no cold tokens
    (300, 128, 4, 256),    # cold range shorter than top_k: all cold selected
    (1000, 2, 4, 256),     # top_k below the sink count: sinks only
    (1000, 0, 4, 256),     # top_k = 0: sinks only
    (1, 128, 4, 0),        # a single token, no hot window
    (2000, 700, 4, 64),    # large top_k
    (3000, 128, 0, 0),     # no sinks, no hot window (plain hybrid_pq_attention)
])
def test_store_edge_cases(S, top_k, sink, hot):
    st, q, lens = _store(1, 1, 2, 64, S, 8, torch.float16, seed=S % 97, cal=min(128, S))
    _check_store(st, q, lens, 0.125, top_k, sink, hot, f"edge S={S} k={top_k}")


def test_ties_and_candidate_overflow():
    """Keys drawn from 8 distinct rows: exact score ties everywhere.  The lower
    token index wins; the tied band around the k'-th score overflows the
    candidate lists, and those chunks are rescanned exactly."""
    from helix_online_kv.cdc03 import CDC03Store
    B, H, S, D, M = 2, 40, 6000, 64, 8
    st = CDC03Store(B, 1, H, D, S, n_subspaces=M, dtype=torch.float16)
    rng = np.random.default_rng(9)
    for b in range(B):
        for h in range(H):
            base = rng.standard_normal((8, D)).astype(np.float32)
            st.k[0, b, h, :S] = torch.from_numpy(base[rng.integers(0, 8, S)]).half().cuda()
    st.v[0, :, :, :S] = torch.from_numpy(rng.standard_normal((B, H, S, D)).astype(np.float32)).half().cuda()
    st.seq_len.fill_(S)
    st.calibrate(0, 128)
    st.assign(0, 0, S)
    q = torch.from_numpy(rng.standard_normal((B, 2 * H, D)).astype(np.float32)).half().cuda()
    _check_store(st, q, [S, S], 0.125, 128, 4, 256, "ties")


def test_one_bin_holding_more_than_65535_tokens():
    """80K identical keys: every score falls in one histogram bin, whose count
    over the whole cluster passes the 16-bit counters of one CTA.  The
    cluster's count is summed in 32 bits, every chunk's list overflows and is
    rescanned exactly, and the selection is the lowest token indices."""
    from helix_online_kv.cdc03 import CDC03Store
    B, H, S, D, M = 1, 1, 80000, 64, 8
    st = CDC03Store(B, 1, H, D, S, n_subspaces=M, dtype=torch.float16)
    rng = np.random.default_rng(17)
    row = rng.standard_normal(D).astype(np.float32)
    st.k[0, 0, 0, :S] = torch.from_numpy(np.tile(row, (S, 1))).half().cuda()
    st.v[0, 0, 0, :S] = torch.from_numpy(rng.standard_normal((S, D)).astype(np.float32)).half().cuda()
    st.seq_len.fill_(S)
    st.calibrate(0, 128)
    st.assign(0, 0, S)
    q = torch.from_numpy(rng.standard_normal((B, 2 * H, D)).astype(np.float32)).half().cuda()
    assert _check_store(st, q, [S], 0.125, 128, 4, 256, "one bin") == 0


def test_hot_window_zero_equals_hybrid(golden):
    """hot_window = 0 on the batched store is the reference hybrid_pq_attention."""
    K, V = O.gen_kv(0, 1, 4, 1024, 64)
    Q = O.gen_queries(0, 1, 32, 64)
    from helix_online_kv.cdc03 import CDC03Store
    st = CDC03Store(1, 1, 4, 64, 1024, n_subspaces=8, dtype=torch.float16)
    st.k[0, 0, :, :1024] = torch.from_numpy(K[0]).half().cuda()
    st.v[0, 0, :, :1024] = torch.from_numpy(V[0]).half().cuda()
    st.seq_len.fill_(1024)
    st.calibrate(0, 128)
    st.assign(0, 0, 1024)
    q = torch.from_numpy(O.to_fp16_values(Q)).half().cuda()
    out, (sel, _, cnt) = st.decode(0, q, 1 / 8, 128, 4, 0, out_dtype=torch.float32, return_selection=True)
    for hq in range(32):
        got = sel[0, hq, :int(cnt[0, hq])].cpu().numpy()
        _assert_selection(got, golden[f"c0m8_q{hq}_approx"], 128, 4, f"hq{hq}")
        np.testing.assert_allclose(out[0, hq].cpu().numpy(), golden[f"c0m8_q{hq}_out"], atol=2e-3)


def test_age_tokens_and_append():
    """Tier aging in place: tokens leaving the hot window get the PQ codes a
    one-token assign gives (GEMV order), ragged per sequence; append() writes
    the new rows, ages the boundary token and grows the lengths; a decode after
    it matches the oracle at the new length."""
    from helix_online_kv.cdc03 import CDC03Store
    from helix_online_kv import _lib
    B, H, G, D, S, M, hot = 2, 2, 4, 64, 1600, 8, 256
    lens = [1500, 1200]
    K, V = O.gen_kv(31, B, H, S, D)
    st = CDC03Store(B, 2, H, D, S, n_subspaces=M, dtype=torch.float16)
    for layer in range(2):
        st.k[layer, :, :, :S] = torch.from_numpy(K).half().cuda()
        st.v[layer, :, :, :S] = torch.from_numpy(V).half().cuda()
        st.calibrate(layer, 128)
    st.seq_len.copy_(torch.tensor(lens, dtype=torch.int32))
    # ragged aging ranges on layer 1, codes zeroed first
    st.codes[1].zero_()
    cf = torch.tensor([100, 700], dtype=torch.int32)
    ct = torch.tensor([140, 705], dtype=torch.int32)
    st.age(1, cf, ct)
    torch.cuda.synchronize()
    _lib.device_status()
    for b in range(B):
        for h in range(H):
            kk = st.cb_k[1, b, h].cpu().numpy()
            cbk = st.codebook[1, b, h].cpu().numpy()
            cents = [cbk[s, :kk[s]] for s in range(M)]
            Kh = st.k[1, b, h].float().cpu().numpy()
            got = st.codes[1, b, h, :, :M].cpu().numpy()
            for t in range(int(cf[b]), int(ct[b])):
                np.testing.assert_array_equal(got[t], O.pq_assign(Kh[t:t + 1], cents)[0], err_msg=f"b{b} h{h} t{t}")
            assert not got[:int(cf[b])].any() and not got[int(ct[b]):].any(), "codes outside the range changed"
    # append one token to every layer; the boundary token is aged on every layer
    for layer in range(2):
        st.assign(layer, 0, max(lens))
    rng = np.random.default_rng(5)
    kn = torch.from_numpy(rng.standard_normal((2, B, H, D)).astype(np.float32)).half().cuda()
    vn = torch.from_numpy(rng.standard_normal((2, B, H, D)).astype(np.float32)).half().cuda()
    before = st.codes.clone()
    st.append(kn, vn, hot_window=hot)
    torch.cuda.synchronize()
    _lib.device_status()
    assert st.seq_len.cpu().tolist() == [n + 1 for n in lens]
    for layer in range(2):
        for b in range(B):
            assert torch.equal(st.k[layer, b, :, lens[b]], kn[layer, b]) and torch.equal(st.v[layer, b, :, lens[b]], vn[layer, b])
            t = lens[b] - hot
            for h in range(H):
                kk = st.cb_k[layer, b, h].cpu().numpy()
                cbk = st.codebook[layer, b, h].cpu().numpy()
                cents = [cbk[s, :kk[s]] for s in range(M)]
                Kh = st.k[layer, b, h].float().cpu().numpy()
                np.testing.assert_array_equal(st.codes[layer, b, h, t, :M].cpu().numpy(),
                                              O.pq_assign(Kh[t:t + 1], cents)[0])
            mask = torch.ones(st.cap, dtype=torch.bool)
            mask[t] = False
            assert torch.equal(st.codes[layer, b][:, mask], before[layer, b][:, mask])
    # the decode at the new length agrees with the oracle
    Q = O.gen_queries(31, B, H * G, D)
    q = torch.from_numpy(Q).half().cuda()
    _check_store(st, q, [n + 1 for n in lens], 0.125, 128, 4, hot, "after append",
                 exclude_rows={b: {lens[b] - hot} for b in range(B)})


def test_store_checkpoint_resume(tmp_path):
    """state_dict / load_state_dict through torch.save: the restored store
    decodes bit-identically; a store of another geometry is refused."""
    from helix_online_kv.cdc03 import CDC03Store
    st, q, lens = _store(2, 2, 4, 64, 1500, 8, torch.float16, seed=41, seq_lens=[1500, 1100])
    out1 = st.decode(0, q, 0.125, 64, 4, 128, out_dtype=torch.float32)
    path = tmp_path / "store.pt"
    torch.save(st.state_dict(), path)
    st2 = CDC03Store(2, 1, 2, 64, 1500, n_subspaces=8, dtype=torch.float16)
    st2.load_state_dict(torch.load(path))
    out2 = st2.decode(0, q, 0.125, 64, 4, 128, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(out1, out2)
    with pytest.raises(ValueError, match="Expected shape"):
        CDC03Store(2, 1, 2, 64, 1024, n_subspaces=8, dtype=torch.float16).load_state_dict(torch.load(path))


def test_store_128k_tinyllama_geometry():
    """128K-token contexts at the TinyLlama KV geometry (G = 8 query heads per
    KV head, D = 64, M = 8): 63 chunks of 2048 tokens per unit, eight per CTA of
    the cluster, ragged lengths (131072 and 100000)."""
    st, q, lens = _store(2, 1, 8, 64, 131072, 8, torch.float16, seed=43, seq_lens=[131072, 100000])
    assert _check_store(st, q, lens, 0.125, 128, 4, 256, "128k") <= 4
