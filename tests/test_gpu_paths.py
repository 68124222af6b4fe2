"""Paths A/B/D/F and the dense reference on the GPU against the reference
fixtures, plus the fused scalar-VQ Q.K^T kernel against NumPy (the reference
Triton test's tolerance: rtol 1e-4, atol 1e-5)."""

import numpy as np
import pytest
import torch

from oracle import hokv_oracle as O

pytestmark = pytest.mark.gpu

SCALE = 1.0 / np.sqrt(64)


def _data():
    rng = np.random.default_rng(42)
    q = rng.standard_normal(64).astype(np.float32)
    K = rng.standard_normal((200, 64)).astype(np.float32)
    V = rng.standard_normal((200, 64)).astype(np.float32)
    return q, K, V


def test_standard_attention(golden):
    from helix_online_kv.compressed_attention import standard_attention
    q, K, V = _data()
    s, o = standard_attention(q, K, V, SCALE)
    assert s.dtype == golden["std_scores"].dtype and o.dtype == golden["std_out"].dtype
    np.testing.assert_allclose(s, golden["std_scores"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(o, golden["std_out"], rtol=1e-5, atol=1e-6)
    s32, o32 = standard_attention(q, K, V, float(SCALE))
    assert s32.dtype == np.float32 and o32.dtype == np.float32


def test_path_a(golden):
    from helix_online_kv.codebook import OnlineCodebook
    from helix_online_kv.compressed_attention import scalar_vq_attention
    from helix_online_kv.triton_attention import fused_scalar_vq_qkt_numpy
    q, K, V = _data()
    cb = OnlineCodebook(n_clusters=256)
    cb.feed_calibration(K.ravel())
    cb.finalize_calibration()
    np.testing.assert_array_equal(cb.centroids, golden["pathA_cents"])
    ki = cb.assign(K.ravel()).reshape(K.shape)
    s, o = scalar_vq_attention(q, ki, cb.centroids, V, SCALE)
    np.testing.assert_allclose(s, golden["pathA_scores"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(o, golden["pathA_out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(fused_scalar_vq_qkt_numpy(q, ki, cb.centroids, SCALE), golden["pathA_qkt"],
                               rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("seq_len", [1, 16, 64, 256, 1024, 4097])
def test_fused_scalar_vq_qkt_device(seq_len):
    from helix_online_kv.triton_attention import _HAS_TRITON, fused_scalar_vq_qkt
    assert _HAS_TRITON
    rng = np.random.default_rng(seq_len)
    q = rng.standard_normal(64).astype(np.float32)
    idx = rng.integers(0, 256, size=(seq_len, 64)).astype(np.uint8)
    cb = rng.standard_normal(256).astype(np.float32)
    ref = O.fused_scalar_vq_qkt_numpy(q, idx, cb, SCALE)
    for it in (torch.uint8, torch.int32):
        got = fused_scalar_vq_qkt(torch.from_numpy(q).cuda(), torch.from_numpy(idx).to(it).cuda(),
                                  torch.from_numpy(cb).cuda(), SCALE)
        assert got.is_cuda and got.dtype == torch.float32 and got.shape == (seq_len,)
        np.testing.assert_allclose(got.cpu().numpy(), ref, rtol=1e-4, atol=1e-5)
    with pytest.raises(AssertionError, match="must be on CUDA"):
        fused_scalar_vq_qkt(torch.from_numpy(q), torch.from_numpy(idx).cuda(), torch.from_numpy(cb).cuda(), SCALE)


def test_path_b(golden):
    from helix_online_kv.compressed_attention import full_vector_vq_attention, vector_vq_attention_scores
    from helix_online_kv.vector_codebook import VectorCodebook
    q, K, V = _data()
    ck = VectorCodebook(n_clusters=64, head_dim=64)
    ck.feed_calibration(K)
    ck.finalize_calibration()
    kidx = ck.assign(K)
    np.testing.assert_array_equal(kidx, golden["pathB_kidx"])
    cv = VectorCodebook(n_clusters=64, head_dim=64)
    cv.feed_calibration(V)
    cv.finalize_calibration()
    vidx = cv.assign(V)
    np.testing.assert_array_equal(vidx, golden["pathB_vidx"])
    s = vector_vq_attention_scores(q, kidx, ck.centroids, SCALE)
    np.testing.assert_array_equal(s, golden["pathB_scores"])
    s, o = full_vector_vq_attention(q, kidx, ck.centroids, vidx, cv.centroids, SCALE)
    assert s.dtype == golden["pathB_scores"].dtype
    np.testing.assert_allclose(o, golden["pathB_out"], rtol=1e-5, atol=1e-6)


def test_path_d(golden):
    from helix_online_kv.compressed_attention import full_pq_attention, pq_attention_scores
    from helix_online_kv.product_codebook import ProductCodebook
    q, K, V = _data()
    pk = ProductCodebook(n_subspaces=8, sub_clusters=64, head_dim=64)
    pk.feed_calibration(K)
    pk.finalize_calibration()
    pv = ProductCodebook(n_subspaces=8, sub_clusters=64, head_dim=64)
    pv.feed_calibration(V)
    pv.finalize_calibration()
    ki, vi = pk.assign(K), pv.assign(V)
    s = pq_attention_scores(q, ki, pk, SCALE)
    assert s.dtype == np.float32
    np.testing.assert_array_equal(s, golden["pathD_scores"])
    s, o = full_pq_attention(q, ki, pk, vi, pv, SCALE)
    np.testing.assert_allclose(o, golden["pathD_out"], rtol=1e-5, atol=1e-6)


def test_path_f(golden):
    from helix_online_kv.compressed_attention import prefiltered_attention, standard_attention
    from helix_online_kv.vector_codebook import VectorCodebook
    q, K, V = _data()
    ck = VectorCodebook(n_clusters=64, head_dim=64)
    ck.feed_calibration(K)
    ck.finalize_calibration()
    kidx = ck.assign(K)
    s, o = prefiltered_attention(q, K, V, kidx, ck.centroids, SCALE, top_p=16)
    assert s.dtype == np.float32 and o.dtype == np.float32
    np.testing.assert_array_equal(s == -1e9, golden["pathF_scores"] == -1e9)
    np.testing.assert_allclose(s, golden["pathF_scores"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(o, golden["pathF_out"], rtol=1e-5, atol=1e-6)
    _, full = prefiltered_attention(q, K, V, kidx, ck.centroids, SCALE, top_p=64)
    _, ref = standard_attention(q, K, V, SCALE)
    assert O.cosine(full, ref) > 0.999


def test_compressed_cache_under_generate():
    """CompressedKVCache in HF generate(): calibration, device-side assignment, memory report."""
    transformers = pytest.importorskip("transformers")
    from helix_online_kv import CompressedKVCache
    from helix_online_kv.config import OnlineKVConfig
    cfg = transformers.LlamaConfig(vocab_size=128, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=256)
    torch.manual_seed(0)
    model = transformers.LlamaForCausalLM(cfg).cuda().half().eval()
    cache = CompressedKVCache(OnlineKVConfig(calibration_tokens=16, exact_layers=[0]), n_layers=2)
    ids = torch.randint(0, 128, (1, 24), device="cuda")
    with torch.no_grad():
        model.generate(ids, past_key_values=cache, max_new_tokens=8, do_sample=False)
    assert cache.total_tokens >= 31
    assert cache.calibration_complete
    ls = cache.layer_states[1]
    assert ls.compressed_token_count == cache.total_tokens - 16
    rep = cache.memory_report()
    assert rep["exact_bytes"] > 0 and rep["compressed_bytes"] > 0
    assert rep["total_bytes"] == rep["exact_bytes"] + rep["compressed_bytes"]


def test_cdc03_attention_in_hf_model():
    """CDC-03 as the attention implementation of an HF Llama: with a token budget
    covering the whole cold range a decode step equals exact attention; with
    top-32 it runs the selection, and the tiers follow the cache lifecycle."""
    transformers = pytest.importorskip("transformers")
    from helix_online_kv.cdc03_attention import CDC03Cache
    from helix_online_kv.config import OnlineKVConfig
    cfg = transformers.LlamaConfig(vocab_size=256, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=1024)
    torch.manual_seed(0)
    model = transformers.LlamaForCausalLM(cfg).cuda().half().eval()
    model.config._attn_implementation = "sdpa"
    ids = torch.randint(0, 256, (1, 400), device="cuda")

    def two_steps(cache):
        with torch.no_grad():
            out = model(ids, past_key_values=cache, use_cache=True)
            nxt = out.logits[:, -1:].argmax(-1)
            out2 = model(nxt, past_key_values=cache, use_cache=True)
        return out2.logits[0, -1].float()

    ref = two_steps(transformers.DynamicCache())
    for top_k, exact in ((4096, True), (32, False)):
        kvc = OnlineKVConfig(calibration_tokens=128, hot_window=64, pq_subspaces=8, exact_layers=[0], top_k=top_k)
        cache = CDC03Cache(kvc, n_layers=2, batch=1, kv_heads=2, head_dim=64, capacity=1024, dtype=torch.float16)
        cache.attach(model)
        got = two_steps(cache)
        from helix_online_kv import _lib
        _lib.device_status()
        model.config._attn_implementation = "sdpa"
        assert torch.isfinite(got).all()
        assert cache.ready(1) and not cache.ready(0)
        assert cache._len[1] == 401 and cache._coded[1] == 401 - 64
        cos = torch.nn.functional.cosine_similarity(got, ref, dim=0).item()
        if exact:
            assert cos > 0.9999 and (got - ref).abs().max().item() < 5e-2, (cos, (got - ref).abs().max().item())
        else:
            assert cos > 0.9, cos


def test_cdc03_cache_keeps_one_copy():
    """Compressed layers keep their K/V only in the CDC-03 store (their cache
    layers are views into it): after a 4K-token prefill the cache's device
    bytes are the dense cache's plus the PQ codes and codebooks (under 15 %
    more), where a dense copy beside the store doubled them; memory_report
    counts exactly the allocated tensors; and the decode step with a budget
    covering the cold range equals the dense cache's."""
    transformers = pytest.importorskip("transformers")
    from helix_online_kv.cdc03_attention import CDC03Cache
    from helix_online_kv.config import OnlineKVConfig
    cfg = transformers.LlamaConfig(vocab_size=256, hidden_size=256, intermediate_size=512, num_hidden_layers=4,
                                   num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=8192)
    torch.manual_seed(1)
    model = transformers.LlamaForCausalLM(cfg).cuda().half().eval()
    model.config._attn_implementation = "sdpa"
    S = 4096
    ids = torch.randint(0, 256, (1, S), device="cuda")
    with torch.no_grad():
        dense = transformers.DynamicCache()
        out = model(ids, past_key_values=dense, use_cache=True)
        nxt = out.logits[:, -1:].argmax(-1)
        ref = model(nxt, past_key_values=dense, use_cache=True).logits[0, -1].float()
    dense_bytes = sum(t.element_size() * t.nelement() for layer in dense.layers for t in (layer.keys, layer.values))
    del out
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated()
    kvc = OnlineKVConfig(calibration_tokens=128, hot_window=256, pq_subspaces=8, exact_layers=[0], top_k=S + 16)
    cache = CDC03Cache(kvc, n_layers=4, batch=1, kv_heads=2, head_dim=64, capacity=S + 1, dtype=torch.float16)
    cache.attach(model)
    with torch.no_grad():
        model(ids, past_key_values=cache, use_cache=True)
        torch.cuda.synchronize()
        held = torch.cuda.memory_allocated() - before
        got = model(nxt, past_key_values=cache, use_cache=True).logits[0, -1].float()
    model.config._attn_implementation = "sdpa"
    rep = cache.memory_report()
    st = cache.store
    assert st.k.shape[0] == 3, "the store holds the compressed layers only"
    assert rep["total_bytes"] <= 1.15 * dense_bytes, (rep, dense_bytes)
    assert held <= 1.2 * dense_bytes, (held, dense_bytes)
    assert cache.layers[1].keys.data_ptr() == st.k[0].data_ptr(), "compressed layers are views of the store"
    cos = torch.nn.functional.cosine_similarity(got, ref, dim=0).item()
    assert cos > 0.9999 and (got - ref).abs().max().item() < 5e-2
