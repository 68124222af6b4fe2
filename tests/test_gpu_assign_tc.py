"""Batched nearest-centroid assignment on the tensor cores (k_pq_assign_tc,
hokv_pq_assign for N >= 256 rows in the (N x d) @ (d x k) order) against the
oracle: codes bit-exact for f16, bf16 and f32 inputs, product and vector
codebooks, ragged tiles, several sets, live counts below the slot count,
exact ties (duplicated centroids: the lowest index wins) and heavy outliers.

Reference: vector_codebook.py:95-119, product_codebook.py:118-145.
"""

import numpy as np
import pytest
import torch

from oracle import hokv_oracle as O

pytestmark = pytest.mark.gpu

SLOTS = 256


def _codebooks(rng, xs, M, sd, k, n_sets, dup=False):
    """[n_sets, M, SLOTS, sd] f32 centroids drawn near data rows (slots past k
    hold garbage that must be ignored), counts [n_sets, M]."""
    cb = rng.standard_normal((n_sets, M, SLOTS, sd)).astype(np.float32) * 50.0
    for t in range(n_sets):
        for s in range(M):
            rows = xs[t][rng.integers(0, xs[t].shape[0], k), s * sd:(s + 1) * sd]
            cb[t, s, :k] = rows + rng.standard_normal((k, sd)).astype(np.float32) * 0.05
            if dup:
                cb[t, s, 10] = cb[t, s, 3]
                cb[t, s, k - 1] = cb[t, s, 0]
    return cb, np.full((n_sets, M), k, np.int32)


def _assign(x, cb, counts, M, sd):
    from helix_online_kv import _lib as L
    n_sets, N, D = x.shape
    cbd = torch.from_numpy(cb).cuda()
    kd = torch.from_numpy(counts).cuda()
    out = torch.zeros((n_sets, N, M), dtype=torch.uint8, device="cuda")
    L.check(L.lib().hokv_pq_assign(L.ptr(x), L.dtype_code(x), N, D, N * D, M, sd, L.ptr(cbd), SLOTS, M * SLOTS * sd,
                                   L.ptr(kd), M, L.ptr(out), M, N * M, n_sets, L.DOT_SEQ_FMA, L.stream()),
            "pq_assign")
    torch.cuda.synchronize()
    L.device_status()
    return out.cpu().numpy()


@pytest.mark.parametrize("N,M,sd,k,dtype,n_sets", [
    (4096, 8, 8, 128, torch.float16, 1),      # TinyLlama geometry, 128-token calibration
    (32768, 8, 8, 128, torch.bfloat16, 1),    # the encoder sweep's largest batch
    (5000, 16, 8, 256, torch.bfloat16, 2),    # Llama-3 geometry, full codebooks, ragged last tile, two sets
    (4096, 16, 4, 200, torch.float16, 1),     # 4-dim subspaces (one K slice, half used)
    (4096, 1, 64, 256, torch.float16, 1),     # vector codebook over the whole head
    (3000, 4, 16, 100, torch.float32, 1),     # fp32 inputs: x split into two tf32 parts
    (300, 2, 32, 256, torch.float32, 3),      # the smallest batch on this path, 32-dim subspaces
])
def test_tensor_core_assign_bit_exact(N, M, sd, k, dtype, n_sets):
    rng = np.random.default_rng(N + M * 7 + sd)
    D = M * sd
    K, _ = O.gen_kv(N % 97, n_sets, 1, N, D)
    x = torch.from_numpy(K[:, 0]).to(dtype).cuda().contiguous()
    xs = [x[t].float().cpu().numpy() for t in range(n_sets)]
    cb, counts = _codebooks(rng, xs, M, sd, k, n_sets)
    got = _assign(x, cb, counts, M, sd)
    for t in range(n_sets):
        ref = O.pq_assign(xs[t], [cb[t, s, :k] for s in range(M)])
        np.testing.assert_array_equal(got[t], ref, err_msg=f"set {t}")


def test_tensor_core_assign_ties_and_outliers():
    """Duplicated centroids give exactly equal distances (the first wins);
    rows equal to a centroid; a few rows 1000x the rest."""
    rng = np.random.default_rng(5)
    N, M, sd, k = 2048, 8, 8, 64
    K, _ = O.gen_kv(3, 1, 1, N, M * sd)
    base = K[0, 0]
    cb, counts = _codebooks(rng, [base], M, sd, k, 1, dup=True)
    for s in range(M):   # some rows sit exactly on duplicated centroids
        base[:50, s * sd:(s + 1) * sd] = cb[0, s, 3]
        base[50:60, s * sd:(s + 1) * sd] = cb[0, s, 0]
    base[100:110] *= 1000.0
    x = torch.from_numpy(base).half().cuda()[None]
    xf = x[0].float().cpu().numpy()
    got = _assign(x, cb, counts, M, sd)
    ref = O.pq_assign(xf, [cb[0, s, :k] for s in range(M)])
    np.testing.assert_array_equal(got[0], ref)
    assert (got[0, :50] == 3).all()


def test_store_assign_on_tensor_cores_matches_oracle():
    """CDC03Store.assign (the decode path's batched encoder) at a prefill-sized
    block runs the tensor-core kernel and matches the oracle."""
    from helix_online_kv.cdc03 import CDC03Store
    B, H, S, D, M = 2, 2, 3000, 128, 16
    K, V = O.gen_kv(8, B, H, S, D)
    st = CDC03Store(B, 1, H, D, S, n_subspaces=M, dtype=torch.bfloat16)
    st.k[0, :, :, :S] = torch.from_numpy(K).to(torch.bfloat16).cuda()
    st.calibrate(0, 128)
    st.assign(0, 0, S)
    torch.cuda.synchronize()
    for b in range(B):
        for h in range(H):
            kk = st.cb_k[0, b, h].cpu().numpy()
            cbh = st.codebook[0, b, h].cpu().numpy()
            ref = O.pq_assign(st.k[0, b, h, :S].float().cpu().numpy(), [cbh[s, :kk[s]] for s in range(M)])
            np.testing.assert_array_equal(st.codes[0, b, h, :S, :M].cpu().numpy(), ref)
