"""Write the golden fixtures by running the reference implementation.

Run in the build container, where the reference checkout is mounted:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py /root/reference

The reference package (echo313unfolding/helix-online-kv, pure NumPy/SciPy) is
imported from the given checkout.  Inputs come from the seeded generators in
``oracle/hokv_oracle.py``; the fixtures hold the reference's outputs plus a
checksum of the inputs so a changed generator is caught.  Versions of NumPy,
SciPy and the BLAS build are recorded in ``versions.json``.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _h(*arrays):
    m = hashlib.sha256()
    for a in arrays:
        m.update(np.ascontiguousarray(a).tobytes())
    return m.hexdigest()[:16]


def main(ref_root: str):
    sys.path.insert(0, ref_root)
    sys.path.insert(1, REPO)
    import helix_online_kv as ref  # noqa: F401  (the reference package)
    from helix_online_kv.codebook import OnlineCodebook
    from helix_online_kv.vector_codebook import VectorCodebook
    from helix_online_kv.product_codebook import ProductCodebook
    from helix_online_kv import compressed_attention as ca
    from helix_online_kv.triton_attention import fused_scalar_vq_qkt_numpy
    from helix_online_kv.config import OnlineKVConfig
    from helix_online_kv.layer_state import KVLayerState
    assert os.path.realpath(ref.__file__).startswith(os.path.realpath(ref_root))
    from oracle import hokv_oracle as O

    out = {}

    # ---- config 0: B=1, H_kv=4, H_q=32, D=64, S=1024, fp16 store -------------
    B, Hkv, Hq, D, S = 1, 4, 32, 64, 1024
    K, V = O.gen_kv(0, B, Hkv, S, D)
    Q = O.gen_queries(0, B, Hq, D)
    K, V, Q = O.to_fp16_values(K), O.to_fp16_values(V), O.to_fp16_values(Q)
    out["c0_input_hash"] = np.array(_h(K, V, Q))
    scale = 1.0 / np.sqrt(D)
    g = Hq // Hkv
    for M in (8, 16):
        tag = f"c0m{M}"
        heads = range(Hkv) if M == 8 else range(2)
        for h in heads:
            pq = ProductCodebook(n_subspaces=M, sub_clusters=256, head_dim=D)
            pq.feed_calibration(K[0, h, :128])
            st = pq.finalize_calibration()
            cents = np.stack([np.pad(c.centroids, ((0, 256 - len(c.centroids)), (0, 0)))
                              for c in pq._codebooks])
            out[f"{tag}_h{h}_cents"] = cents.astype(np.float32)
            out[f"{tag}_h{h}_k"] = np.array(st["sub_clusters"], np.int32)
            out[f"{tag}_h{h}_iters"] = np.array(st["n_iters_per_sub"], np.int32)
            codes = pq.assign(K[0, h])
            out[f"{tag}_h{h}_codes"] = codes
            for qi in range(g):
                hq = h * g + qi
                q = Q[0, hq]
                T = pq.precompute_distance_tables(q)
                approx = pq.gather_pq_scores(T, codes) * np.float32(scale)
                sc, o, meta = ca.hybrid_pq_attention(q, K[0, h], V[0, h], codes, pq, scale,
                                                    top_k=128, sink_tokens=4)
                pre = f"{tag}_q{hq}"
                if qi < 2:
                    out[pre + "_T"] = T
                out[pre + "_approx"] = approx
                out[pre + "_sel"] = np.flatnonzero(np.isfinite(sc)).astype(np.int32)
                out[pre + "_out"] = o
                out[pre + "_meta"] = np.array([meta["selected_count"], meta["coverage"],
                                               meta["pq_score_range"], meta["sink_count"]])
                if M == 8:
                    # composed hot-window oracle from reference calls only: CDC-03 on
                    # the cold range, then exact softmax over (selected cold) U hot.
                    Sc = S - 256
                    sc_c, _, _ = ca.hybrid_pq_attention(q, K[0, h, :Sc], V[0, h, :Sc], codes[:Sc],
                                                        pq, scale, top_k=128, sink_tokens=4)
                    selc = np.flatnonzero(np.isfinite(sc_c))
                    union = np.concatenate([selc, np.arange(Sc, S)])
                    _, o_hot = ca.standard_attention(q, K[0, h, union], V[0, h, union], scale)
                    out[pre + "_hot_sel"] = selc.astype(np.int32)
                    out[pre + "_hot_out"] = np.asarray(o_hot, np.float32)

    # ---- scalar codebook (layer-state style: 128 tokens x H_kv*D values) ------
    flat_k = K[0].transpose(1, 0, 2).reshape(S, Hkv * D)
    cb = OnlineCodebook(n_clusters=256, max_iters=10, rtol=1e-3)
    for t in range(128):
        cb.feed_calibration(flat_k[t])
    st = cb.finalize_calibration()
    out["sc_cents"] = cb.centroids
    out["sc_stats"] = np.array([st["n_samples"], st["n_clusters"], st["n_iters"],
                                st["calibration_mse"]])
    out["sc_assign"] = cb.assign(flat_k[128:144])
    drift_vals = flat_k[144:160].ravel() + 0.75
    err = cb.quantization_error(drift_vals, cb.assign(drift_vals))
    cb2 = OnlineCodebook(n_clusters=256, drift_threshold=0.0001)
    cb2._centroids = cb.centroids.copy()
    cb2._finalized = True
    upd = cb2.maybe_update_centroids(drift_vals, err)
    out["sc_ema"] = cb2.centroids
    out["sc_ema_flag"] = np.array(int(upd))
    for seed, (n, kk) in enumerate([(10000, 256), (2000, 16), (777, 64), (5000, 200)]):
        rng = np.random.default_rng(100 + seed)
        d = rng.standard_normal(n).astype(np.float32)
        if seed == 3:
            d = np.round(d * 8).astype(np.float32) / 8  # many ties
        c = OnlineCodebook(n_clusters=kk)
        c.feed_calibration(d)
        s2 = c.finalize_calibration()
        out[f"sc{seed}_cents"] = c.centroids
        out[f"sc{seed}_stats"] = np.array([s2["n_samples"], s2["n_clusters"], s2["n_iters"],
                                           s2["calibration_mse"]])
        test = rng.standard_normal(3000).astype(np.float32) * 1.5
        out[f"sc{seed}_assign"] = c.assign(test)

    # ---- vector codebook: degenerate and converging fits, several N ----------
    rng = np.random.default_rng(11)
    for tag, (n, dd, kk) in {"vq0": (128, 64, 256), "vq1": (1024, 64, 64),
                             "vq2": (300, 8, 32), "vq3": (200, 64, 16)}.items():
        data = (rng.standard_normal((n, dd)) * rng.uniform(0.5, 2, dd)).astype(np.float32)
        vq = VectorCodebook(n_clusters=kk, head_dim=dd)
        vq.feed_calibration(data)
        st = vq.finalize_calibration()
        out[f"{tag}_data_hash"] = np.array(_h(data))
        out[f"{tag}_cents"] = vq.centroids
        out[f"{tag}_stats"] = np.array([st["n_samples"], st["n_clusters"], st["n_iters"],
                                        st["calibration_mse"]])
        for N in (1, 3, 16, 1000):
            x = (rng.standard_normal((N, dd)) * 1.3).astype(np.float32)
            out[f"{tag}_x{N}_hash"] = np.array(_h(x))
            out[f"{tag}_assign{N}"] = vq.assign(x)
        qv = rng.standard_normal(dd).astype(np.float32)
        out[f"{tag}_qscores"] = vq.precompute_query_scores(qv)

    # ---- product codebook, converging fit (sub_clusters 64 on 512 vectors) ---
    rng = np.random.default_rng(12)
    for tag, (n, M, kk) in {"pq0": (512, 8, 64), "pq1": (256, 16, 64), "pq2": (256, 4, 64)}.items():
        data = rng.standard_normal((n, 64)).astype(np.float32)
        pq = ProductCodebook(n_subspaces=M, sub_clusters=kk, head_dim=64)
        pq.feed_calibration(data)
        st = pq.finalize_calibration()
        out[f"{tag}_cents"] = np.stack([c.centroids for c in pq._codebooks])
        out[f"{tag}_iters"] = np.array(st["n_iters_per_sub"], np.int32)
        out[f"{tag}_mse"] = np.array(st["calibration_mse_per_sub"])
        for N in (1, 3, 200):
            x = rng.standard_normal((N, 64)).astype(np.float32)
            out[f"{tag}_assign{N}"] = pq.assign(x)
        qv = rng.standard_normal(64).astype(np.float32)
        out[f"{tag}_T"] = pq.precompute_distance_tables(qv)

    # ---- attention paths A/B/D/F on the reference test shapes ----------------
    rng = np.random.default_rng(42)
    q = rng.standard_normal(64).astype(np.float32)
    Ks = rng.standard_normal((200, 64)).astype(np.float32)
    Vs = rng.standard_normal((200, 64)).astype(np.float32)
    sc_scale = 1.0 / np.sqrt(64)
    cbk = VectorCodebook(n_clusters=64, head_dim=64)
    cbk.feed_calibration(Ks)
    cbk.finalize_calibration()
    kidx = cbk.assign(Ks)
    cbv = VectorCodebook(n_clusters=64, head_dim=64)
    cbv.feed_calibration(Vs)
    cbv.finalize_calibration()
    vidx = cbv.assign(Vs)
    s_b, o_b = ca.full_vector_vq_attention(q, kidx, cbk.centroids, vidx, cbv.centroids, sc_scale)
    out["pathB_scores"], out["pathB_out"] = s_b, o_b
    out["pathB_kidx"], out["pathB_vidx"] = kidx, vidx
    pk = ProductCodebook(n_subspaces=8, sub_clusters=64, head_dim=64)
    pk.feed_calibration(Ks)
    pk.finalize_calibration()
    pv = ProductCodebook(n_subspaces=8, sub_clusters=64, head_dim=64)
    pv.feed_calibration(Vs)
    pv.finalize_calibration()
    s_d, o_d = ca.full_pq_attention(q, pk.assign(Ks), pk, pv.assign(Vs), pv, sc_scale)
    out["pathD_scores"], out["pathD_out"] = s_d, o_d
    s_f, o_f = ca.prefiltered_attention(q, Ks, Vs, kidx, cbk.centroids, sc_scale, top_p=16)
    out["pathF_scores"], out["pathF_out"] = s_f, o_f
    scb = OnlineCodebook(n_clusters=256)
    scb.feed_calibration(Ks.ravel())
    scb.finalize_calibration()
    ki = scb.assign(Ks.ravel()).reshape(Ks.shape)
    s_a, o_a = ca.scalar_vq_attention(q, ki, scb.centroids, Vs, sc_scale)
    out["pathA_scores"], out["pathA_out"], out["pathA_cents"] = s_a, o_a, scb.centroids
    out["pathA_qkt"] = fused_scalar_vq_qkt_numpy(q, ki, scb.centroids, sc_scale)
    s_s, o_s = ca.standard_attention(q, Ks, Vs, sc_scale)
    out["std_scores"], out["std_out"] = s_s, o_s

    # ---- layer state (scalar codebooks, calibration_tokens=16) ---------------
    cfg = OnlineKVConfig(calibration_tokens=16, n_clusters=64, exact_layers=[])
    ls = KVLayerState(1, cfg)
    rng = np.random.default_rng(5)
    toks = rng.standard_normal((40, 2, 256)).astype(np.float32)
    stats = None
    for t in range(40):
        r = ls.feed_token(toks[t, 0], toks[t, 1])
        stats = stats or r
    out["ls_k_cents"] = ls.k_codebook.centroids
    out["ls_v_cents"] = ls.v_codebook.centroids
    out["ls_k_idx"] = np.stack(ls._k_indices)
    out["ls_v_idx"] = np.stack(ls._v_indices)
    out["ls_mem"] = np.array([ls.memory_bytes()[k] for k in ("codebook_bytes", "index_bytes", "total_bytes")])

    np.savez_compressed(os.path.join(HERE, "reference_golden.npz"), **out)
    import scipy
    cfg_blas = np.show_config(mode="dicts")["Build Dependencies"]["blas"]
    with open(os.path.join(HERE, "versions.json"), "w") as f:
        json.dump({"numpy": np.__version__, "scipy": scipy.__version__,
                   "blas": f"{cfg_blas.get('name')} {cfg_blas.get('version')}",
                   "python": sys.version.split()[0], "n_arrays": len(out)}, f, indent=1)
    print("wrote", len(out), "arrays")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
