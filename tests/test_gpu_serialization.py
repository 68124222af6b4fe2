"""Checkpoint / resume of the codebooks, the layer states and both caches
(state_dict / load_state_dict through torch.save): a restored object gives
bit-identical results; mismatched parameters are refused.  The reference has
no serialization; these are additions."""

import numpy as np
import pytest
import torch

from oracle import hokv_oracle as O

pytestmark = pytest.mark.gpu


def _roundtrip(obj, tmp_path, name):
    path = tmp_path / f"{name}.pt"
    torch.save(obj.state_dict(), path)
    return torch.load(path, weights_only=False)


def test_codebooks_roundtrip(tmp_path):
    from helix_online_kv.codebook import OnlineCodebook
    from helix_online_kv.product_codebook import ProductCodebook
    from helix_online_kv.vector_codebook import VectorCodebook
    K, _ = O.gen_kv(2, 1, 1, 600, 64)
    x = O.to_fp16_values(K[0, 0])
    # scalar: one mid-calibration, one finalized
    a = OnlineCodebook(n_clusters=64)
    a.feed_calibration(x[:128].ravel())
    b = OnlineCodebook(n_clusters=64)
    b.load_state_dict(_roundtrip(a, tmp_path, "sc_cal"))
    a.finalize_calibration()
    b.finalize_calibration()
    np.testing.assert_array_equal(a.centroids, b.centroids)
    c = OnlineCodebook(n_clusters=64)
    c.load_state_dict(_roundtrip(a, tmp_path, "sc"))
    np.testing.assert_array_equal(a.assign(x[128:].ravel()), c.assign(x[128:].ravel()))
    with pytest.raises(ValueError, match="Expected"):
        OnlineCodebook(n_clusters=32).load_state_dict(a.state_dict())
    # vector and product
    for make in (lambda: VectorCodebook(n_clusters=64, head_dim=64),
                 lambda: ProductCodebook(n_subspaces=8, sub_clusters=64, head_dim=64)):
        a = make()
        a.feed_calibration(x[:200])
        a.finalize_calibration()
        b = make()
        b.load_state_dict(_roundtrip(a, tmp_path, "vq"))
        np.testing.assert_array_equal(a.assign(x[200:]), b.assign(x[200:]))
        np.testing.assert_array_equal(a.decode(a.assign(x[200:210])), b.decode(b.assign(x[200:210])))
    with pytest.raises(ValueError, match="Expected"):
        ProductCodebook(n_subspaces=4, sub_clusters=64, head_dim=64).load_state_dict(a.state_dict())


def _tiny_llama():
    transformers = pytest.importorskip("transformers")
    cfg = transformers.LlamaConfig(vocab_size=256, hidden_size=256, intermediate_size=512, num_hidden_layers=3,
                                   num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=2048)
    torch.manual_seed(3)
    return transformers.LlamaForCausalLM(cfg).cuda().half().eval()


def _steps(model, cache, tok, n):
    outs = []
    with torch.no_grad():
        for _ in range(n):
            logits = model(tok, past_key_values=cache, use_cache=True).logits[:, -1:]
            outs.append(logits.float())
            tok = logits.argmax(-1)
    return torch.cat(outs, 1), tok


@pytest.mark.parametrize("kind", ["compressed", "cdc03"])
def test_cache_checkpoint_resume(tmp_path, kind):
    """Prefill and two decode steps, checkpoint, then three more steps from the
    live cache and from a restored one: the logits are bit-identical."""
    from helix_online_kv.cdc03_attention import CDC03Cache
    from helix_online_kv.compressed_cache import CompressedKVCache
    from helix_online_kv.config import OnlineKVConfig
    model = _tiny_llama()
    kvc = OnlineKVConfig(calibration_tokens=128, hot_window=64, pq_subspaces=8, exact_layers=[0], top_k=32)

    def make():
        if kind == "cdc03":
            return CDC03Cache(kvc, n_layers=3, batch=1, kv_heads=2, head_dim=64, capacity=1024).attach(model)
        return CompressedKVCache(kvc, n_layers=3)

    ids = torch.randint(0, 256, (1, 300), device="cuda")
    cache = make()
    with torch.no_grad():
        tok = model(ids, past_key_values=cache, use_cache=True).logits[:, -1:].argmax(-1)
    _, tok = _steps(model, cache, tok, 2)
    state = _roundtrip(cache, tmp_path, kind)
    live, _ = _steps(model, cache, tok, 3)
    restored = make()
    restored.load_state_dict(state)
    again, _ = _steps(model, restored, tok, 3)
    model.config._attn_implementation = "sdpa"
    assert torch.equal(live, again)
    assert restored.total_tokens == cache.total_tokens and restored.calibration_complete
    assert [ls.phase for ls in restored.layer_states] == [ls.phase for ls in cache.layer_states]
    with pytest.raises(ValueError, match="Expected"):
        other = OnlineKVConfig(calibration_tokens=64, hot_window=64, pq_subspaces=8, exact_layers=[0], top_k=32)
        (CDC03Cache(other, n_layers=3, batch=1, kv_heads=2, head_dim=64, capacity=1024) if kind == "cdc03"
         else CompressedKVCache(other, n_layers=3)).load_state_dict(state)
