"""Host-side API checks that need no GPU: the C ABI library loads and exports
every declared entry point, lifecycle errors and messages match the
reference's, configuration/aging arithmetic, and the package refuses to run
without a CUDA device (there is no CPU fallback)."""

import ctypes
import os
import re

import numpy as np
import pytest

import helix_online_kv as hk
from helix_online_kv import _lib
from helix_online_kv.aging_policy import AgingPolicy
from helix_online_kv.codebook import OnlineCodebook
from helix_online_kv.config import OnlineKVConfig
from helix_online_kv.layer_state import KVLayerState, LayerPhase
from helix_online_kv.product_codebook import ProductCodebook
from helix_online_kv.vector_codebook import VectorCodebook

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    with open(os.path.join(REPO, "include", "hokv.h")) as f:
        return sorted(set(re.findall(r"\b(hokv_\w+)\s*\(", f.read())))


def test_library_exports_every_declared_symbol():
    from helix_online_kv import _build
    _build.build(verbose=False)
    lib = ctypes.CDLL(_lib.LIB_PATH)
    names = _declared()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    lib.hokv_abi_version.restype = ctypes.c_int
    assert lib.hokv_abi_version() == 1


def test_binding_covers_the_header():
    """Every declared entry point has a ctypes signature in the binding."""
    assert set(_declared()) <= set(_lib._SIGS), set(_declared()) - set(_lib._SIGS)


def test_status_strings():
    L = _lib.lib()
    assert L.hokv_status_string(0) == b"ok"
    assert b"workspace" in L.hokv_status_string(6)


def test_argument_validation_without_device():
    """Host-side validation rejects bad shapes before any launch."""
    L = _lib.lib()
    st = L.hokv_scalar_assign(None, 0, 10, 10, None, 300, 0, None, 0, 1, None)
    assert st == _lib.ERR_INVALID
    assert b"k=300" in L.hokv_last_error()
    a = _lib.Cdc03Args()
    a.batch, a.kv_heads, a.q_per_kv, a.head_dim, a.n_subspaces = 1, 1, 1, 96, 8
    need = ctypes.c_size_t(0)
    assert L.hokv_cdc03_workspace_size(ctypes.byref(a), ctypes.byref(need)) == _lib.ERR_INVALID
    assert b"head_dim" in L.hokv_last_error()


def test_exports():
    for name in ("OnlineKVConfig", "OnlineCodebook", "VectorCodebook", "ProductCodebook", "KVLayerState",
                 "AgingPolicy"):
        assert hasattr(hk, name)


def test_config_defaults_match_reference():
    c = OnlineKVConfig()
    assert (c.calibration_tokens, c.hot_window, c.n_clusters, c.max_kmeans_iters) == (128, 256, 256, 10)
    assert (c.rtol, c.drift_threshold, c.drift_ema_alpha, c.exact_layers) == (0.001, 0.01, 0.05, [0])
    with pytest.raises(Exception):
        c.hot_window = 3  # frozen


def test_aging_policy():
    ap = AgingPolicy(hot_window=256)
    assert not ap.should_compress(255) and ap.should_compress(256)
    assert ap.tier_boundary(100) == 0 and ap.tier_boundary(257) == 1 and ap.tier_boundary(512) == 256
    assert AgingPolicy(hot_window=128).tier_boundary(1024) == 896
    ap2 = AgingPolicy(hot_window=256, min_age_tokens=128)
    assert not ap2.should_compress(127) and ap2.should_compress(128)


def test_lifecycle_errors_need_no_device():
    with pytest.raises(RuntimeError, match="not finalized"):
        OnlineCodebook(n_clusters=16).assign(np.zeros(4, np.float32))
    with pytest.raises(RuntimeError, match="No calibration data"):
        OnlineCodebook(n_clusters=16).finalize_calibration()
    with pytest.raises(RuntimeError, match="not finalized"):
        VectorCodebook(n_clusters=16, head_dim=64).assign(np.zeros((2, 64), np.float32))
    with pytest.raises(RuntimeError, match="No calibration data"):
        VectorCodebook(n_clusters=16, head_dim=64).finalize_calibration()
    with pytest.raises(ValueError, match="Expected shape"):
        VectorCodebook(n_clusters=16, head_dim=64).feed_calibration(np.zeros((10, 32), np.float32))
    with pytest.raises(ValueError, match="divisible"):
        ProductCodebook(n_subspaces=7, head_dim=64)
    with pytest.raises(ValueError, match="Expected shape"):
        ProductCodebook(n_subspaces=8, head_dim=64).feed_calibration(np.zeros((10, 32), np.float32))
    with pytest.raises(RuntimeError, match="No calibration data"):
        ProductCodebook(n_subspaces=8, head_dim=64).finalize_calibration()
    with pytest.raises(RuntimeError, match="not finalized"):
        ProductCodebook(n_subspaces=8, head_dim=64).precompute_distance_tables(np.zeros(64, np.float32))


def test_exact_layer_state():
    ls = KVLayerState(0, OnlineKVConfig(exact_layers=[0]))
    assert ls.is_exact and ls.phase == LayerPhase.EXACT
    assert ls.feed_token(np.zeros(256, np.float32), np.zeros(256, np.float32)) is None
    assert ls.memory_bytes() == {"codebook_bytes": 0, "index_bytes": 0, "total_bytes": 0}


@pytest.mark.skipif(_lib.available(), reason="a CUDA device is present")
def test_no_cpu_fallback():
    """Without a CUDA device the compute path raises instead of falling back."""
    cb = OnlineCodebook(n_clusters=4)
    cb.feed_calibration(np.arange(10, dtype=np.float32))
    with pytest.raises(RuntimeError, match="CUDA"):
        cb.finalize_calibration()
    from helix_online_kv.compressed_attention import standard_attention
    with pytest.raises(RuntimeError, match="CUDA"):
        standard_attention(np.zeros(8, np.float32), np.zeros((4, 8), np.float32), np.zeros((4, 8), np.float32),
                           0.3)
    from helix_online_kv.triton_attention import _HAS_TRITON
    assert _HAS_TRITON is False


def test_cdc03_context_limit_is_refused():
    """Contexts needing more than 248 candidate chunks of 2048 tokens per
    (sequence, KV head) are refused by the workspace query, on the host."""
    from helix_online_kv import _build
    _build.build(verbose=False)
    lib = _lib.lib()
    a = _lib.Cdc03Args()
    a.batch, a.kv_heads, a.q_per_kv, a.head_dim = 1, 1, 4, 64
    a.n_subspaces, a.sub_dim, a.code_bytes, a.cb_slots = 8, 8, 8, 256
    a.top_k, a.sink_tokens, a.hot_window, a.scale, a.lut_order = 128, 4, 256, 0.125, _lib.DOT_GEMV
    dummy = 1 << 20   # never dereferenced: the query only validates
    a.q = a.out = a.k = a.v = a.codes = a.codebook = a.cb_k = a.seq_len = dummy
    a.q_dtype = a.out_dtype = a.kv_dtype = _lib.F16
    a.kv_stride_b = a.kv_stride_h = 0
    a.code_stride_b = a.code_stride_h = 0
    need = ctypes.c_size_t(0)
    a.capacity = 248 * 2048 + 256
    assert lib.hokv_cdc03_workspace_size(ctypes.byref(a), ctypes.byref(need)) == 0 and need.value > 0
    a.capacity = 248 * 2048 + 256 + 16
    st = lib.hokv_cdc03_workspace_size(ctypes.byref(a), ctypes.byref(need))
    assert st != 0 and b"chunks" in lib.hokv_last_error()


def test_prefill_host_checks():
    """hokv_prefill_attention validates on the host: unsupported dtypes and head
    dims, causal calls with fewer keys than queries, strides that are not
    multiples of 8 elements; the Python side accepts only nesting strides and
    CUDA tensors (no CPU path)."""
    import torch
    from helix_online_kv.prefill import _nests, supported
    L = _lib.lib()
    args = [None] * 4
    strides = [0] * 12
    st = L.hokv_prefill_attention(*args, _lib.F16, 1, 4, 2, 16, 16, 64, *strides, 0.125, 1, None)
    assert st == _lib.ERR_INVALID and b"null" in L.hokv_last_error()
    p = ctypes.c_void_p(16)   # never dereferenced: validation fails first
    st = L.hokv_prefill_attention(p, p, p, p, _lib.F32, 1, 4, 2, 16, 16, 64, *strides, 0.125, 1, None)
    assert st == _lib.ERR_UNSUPPORTED and b"dtype" in L.hokv_last_error()
    st = L.hokv_prefill_attention(p, p, p, p, _lib.BF16, 1, 4, 2, 16, 16, 96, *strides, 0.125, 1, None)
    assert st == _lib.ERR_UNSUPPORTED and b"head_dim" in L.hokv_last_error()
    st = L.hokv_prefill_attention(p, p, p, p, _lib.BF16, 1, 4, 2, 32, 16, 64, *strides, 0.125, 1, None)
    assert st == _lib.ERR_INVALID and b"kv_len >= q_len" in L.hokv_last_error()
    bad = [8] * 12
    bad[2] = 12
    st = L.hokv_prefill_attention(p, p, p, p, _lib.BF16, 1, 4, 2, 16, 16, 64, *bad, 0.125, 1, None)
    assert st == _lib.ERR_INVALID and b"stride" in L.hokv_last_error()
    # stride nesting (the tensor maps' requirement), checked on CPU tensors
    assert _nests(torch.empty(2, 600, 8, 64).transpose(1, 2))            # a model's transposed projection
    assert _nests(torch.empty(2, 2, 2048, 64)[:, :, :600])               # a store slice
    assert not _nests(torch.as_strided(torch.empty(4096), (1, 2, 16, 64), (4096, 64, 64, 1)))   # aliasing
    q = torch.zeros(1, 2, 16, 64, dtype=torch.float16)
    assert not supported(q, q, q)                                        # CPU tensors: no kernel, no fallback
