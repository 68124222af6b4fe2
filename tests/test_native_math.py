"""The library's exact-order fp32 arithmetic (hokv_math.cuh), built for the host
with g++, reproduces the reference fixtures: sub-tables, L2 assignment,
pairwise sums, percentile init and norm-order picks.  CPU only."""

import ctypes
import os
import subprocess

import numpy as np
import pytest

from oracle import hokv_oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(REPO, "helix-online-kv_b200", "csrc")
OUT = os.path.join(HERE, "native", "_build", "libhokv_math_host.so")


@pytest.fixture(scope="module")
def lib():
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    src = os.path.join(HERE, "native", "hokv_math_host.cpp")
    if not os.path.exists(OUT) or os.path.getmtime(OUT) < max(
            os.path.getmtime(src), os.path.getmtime(os.path.join(CSRC, "hokv_math.cuh"))):
        subprocess.check_call(["g++", "-O2", "-ffp-contract=off", "-fno-fast-math", "-std=c++17", "-shared",
                               "-fPIC", "-I", CSRC, "-o", OUT, src])
    L = ctypes.CDLL(OUT)
    L.host_pw_sum.restype = ctypes.c_float
    L.host_adc_score.restype = ctypes.c_float
    L.host_linspace_pick.restype = ctypes.c_int64
    L.host_pw_sum.argtypes = [ctypes.c_void_p, ctypes.c_int64]
    L.host_linspace_pick.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_int]
    L.host_dot_order_for.argtypes = [ctypes.c_int64, ctypes.c_int]
    L.host_l2_argmin.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                 ctypes.c_int, ctypes.c_void_p]
    L.host_percentiles.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p]
    L.host_pq_tables.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                 ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
    L.host_adc_score.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_float]
    return L


def _p(a):
    return a.ctypes.data


def _tables(lib, q, cents_list, t_cols):
    M = len(cents_list)
    sd = cents_list[0].shape[1]
    slots = max(len(c) for c in cents_list)
    cb = np.zeros((M, slots, sd), np.float32)
    k = np.array([len(c) for c in cents_list], np.int32)
    for s, c in enumerate(cents_list):
        cb[s, :len(c)] = c
    T = np.zeros((M, t_cols), np.float32)
    q = np.ascontiguousarray(q, np.float32)
    lib.host_pq_tables(_p(q), M, sd, _p(cb), slots, _p(k), _p(T), t_cols, 1)
    return T


def test_pq_tables_match_reference(lib, golden):
    K, V = O.gen_kv(0, 1, 4, 1024, 64)
    Q = O.to_fp16_values(O.gen_queries(0, 1, 32, 64))
    K = O.to_fp16_values(K)
    for M in (8, 16):
        for h in (range(4) if M == 8 else range(2)):
            kk = golden[f"c0m{M}_h{h}_k"]
            gc = golden[f"c0m{M}_h{h}_cents"]
            cents = [gc[s, :kk[s]] for s in range(M)]
            for qi in range(2):
                hq = h * 8 + qi
                T = _tables(lib, Q[0, hq], cents, int(kk.max()))
                np.testing.assert_array_equal(T, golden[f"c0m{M}_q{hq}_T"])


def test_adc_scores_bit_exact(lib, golden):
    Q = O.to_fp16_values(O.gen_queries(0, 1, 32, 64))
    kk = golden["c0m8_h0_k"]
    gc = golden["c0m8_h0_cents"]
    cents = [gc[s, :kk[s]] for s in range(8)]
    codes = np.ascontiguousarray(golden["c0m8_h0_codes"])
    T = _tables(lib, Q[0, 0], cents, 256)
    sc = np.float32(1.0 / np.sqrt(64))
    got = np.array([lib.host_adc_score(_p(T), 8, 256, _p(codes[t]), sc) for t in range(0, 1024, 7)], np.float32)
    np.testing.assert_array_equal(got, golden["c0m8_q0_approx"][::7])


def test_pq_tables_converging_fits(lib, golden):
    rng = np.random.default_rng(12)
    for tag, (n, M, kk) in {"pq0": (512, 8, 64), "pq1": (256, 16, 64), "pq2": (256, 4, 64)}.items():
        rng.standard_normal((n, 64))
        for N in (1, 3, 200):
            rng.standard_normal((N, 64))
        qv = rng.standard_normal(64).astype(np.float32)
        cents = list(golden[f"{tag}_cents"])
        np.testing.assert_array_equal(_tables(lib, qv, cents, kk), golden[f"{tag}_T"])


@pytest.mark.parametrize("tag,dims", [("vq0", (128, 64, 256)), ("vq1", (1024, 64, 64)),
                                      ("vq2", (300, 8, 32)), ("vq3", (200, 64, 16))])
def test_vq_assign_orders(lib, golden, tag, dims):
    n, dd, kk = dims
    rng = np.random.default_rng(11)
    order_tags = ["vq0", "vq1", "vq2", "vq3"]
    allds = {"vq0": (128, 64, 256), "vq1": (1024, 64, 64), "vq2": (300, 8, 32), "vq3": (200, 64, 16)}
    for t in order_tags:
        nn, d2, _ = allds[t]
        data = (rng.standard_normal((nn, d2)) * rng.uniform(0.5, 2, d2)).astype(np.float32)
        xs = {N: (rng.standard_normal((N, d2)) * 1.3).astype(np.float32) for N in (1, 3, 16, 1000)}
        rng.standard_normal(d2)
        if t == tag:
            break
    cents = np.ascontiguousarray(golden[f"{tag}_cents"])
    for N, x in xs.items():
        out = np.zeros(N, np.uint8)
        order = lib.host_dot_order_for(N, dd)
        lib.host_l2_argmin(_p(x), N, dd, _p(cents), len(cents), order, _p(out))
        np.testing.assert_array_equal(out, golden[f"{tag}_assign{N}"], err_msg=f"N={N}")


def test_pairwise_sum_and_percentile(lib):
    rng = np.random.default_rng(3)
    for n in (1, 5, 8, 127, 128, 129, 1000, 40000):
        a = (rng.standard_normal(n) * 3).astype(np.float32)
        assert np.float32(lib.host_pw_sum(_p(a), n)) == np.sum(a)
    for n, k in ((1000, 256), (32768, 256), (5, 3), (2, 1), (777, 64)):
        a = rng.standard_normal(n).astype(np.float32)
        srt = np.sort(a)
        out = np.zeros(k, np.float32)
        lib.host_percentiles(_p(srt), n, k, _p(out))
        np.testing.assert_array_equal(out, np.percentile(a, np.linspace(0, 100, k)).astype(np.float32))
    for n, k in ((128, 128), (128, 37), (1024, 256), (1, 1), (10, 3)):
        ref = np.linspace(0, n - 1, k).astype(int)
        assert [lib.host_linspace_pick(n, k, i) for i in range(k)] == list(ref)
