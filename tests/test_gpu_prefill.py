"""Exact multi-token attention on the tensor cores (hokv_prefill_attention)
against a plain PyTorch fp32 reference of the same op: causal and full,
grouped-query heads, f16 and bf16, head dims 64 and 128, ragged lengths,
queries offset into a longer cache, strided store views, logits that grow
along the sequence (the lazy rescaling of the running maximum) and the
rejection of unsupported inputs.

Tolerance (written per case): the softmax weights are rounded to the input
type before the second product, as FlashAttention does; the error is a few
units in the last place of that type relative to max |V|.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 4e-3, torch.bfloat16: 2.5e-2}


def _ref(q, k, v, scale, causal):
    """fp32 softmax(q k^T scale [causal]) v -> [B, Sq, Hq, D]."""
    B, Hq, Sq, D = q.shape
    G = Hq // k.shape[1]
    kf = k.float().repeat_interleave(G, dim=1)
    vf = v.float().repeat_interleave(G, dim=1)
    s = (q.float() @ kf.transpose(-1, -2)) * scale
    if causal:
        Skv = k.shape[2]
        pos = torch.arange(Sq, device=q.device)[:, None] + (Skv - Sq)
        s = s.masked_fill(torch.arange(Skv, device=q.device)[None, :] > pos, float("-inf"))
    return (torch.softmax(s, dim=-1) @ vf).transpose(1, 2)


def _check(q, k, v, causal=True, scale=None):
    from helix_online_kv import _lib as L
    from helix_online_kv.prefill import prefill_attention
    scale = scale if scale is not None else q.shape[-1] ** -0.5
    out = prefill_attention(q, k, v, scale, is_causal=causal)
    torch.cuda.synchronize()
    L.device_status()
    ref = _ref(q, k, v, scale, causal)
    err = (out.float() - ref).abs().max().item()
    vmax = v.float().abs().max().item()
    assert torch.isfinite(out.float()).all()
    assert err <= TOL[q.dtype] * max(1.0, vmax), (err, vmax)
    return out


def _rand(B, H, S, D, dtype, gen, scale=1.0):
    return (torch.randn((B, H, S, D), generator=gen, device="cuda") * scale).to(dtype)


@pytest.mark.parametrize("B,Hq,Hkv,Sq,Skv,D,dtype,causal", [
    (1, 32, 4, 1024, 1024, 64, torch.float16, True),       # TinyLlama prefill of a 1024-token prompt
    (2, 32, 8, 1000, 1000, 128, torch.bfloat16, True),     # Llama-3-8B geometry, ragged last tiles
    (1, 4, 2, 77, 700, 128, torch.float16, True),          # a chunk of queries at the end of a longer cache
    (2, 6, 3, 130, 257, 64, torch.bfloat16, False),        # full (non-causal) attention
    (1, 8, 8, 1, 300, 64, torch.float16, True),            # one query
    (3, 2, 1, 129, 129, 128, torch.float16, True),         # one row past a tile
])
def test_prefill_matches_fp32_reference(B, Hq, Hkv, Sq, Skv, D, dtype, causal):
    gen = torch.Generator(device="cuda")
    gen.manual_seed(B * 1000 + Sq + D)
    q = _rand(B, Hq, Sq, D, dtype, gen)
    k = _rand(B, Hkv, Skv, D, dtype, gen)
    v = _rand(B, Hkv, Skv, D, dtype, gen)
    _check(q, k, v, causal)


def test_prefill_long_causal():
    """8K tokens, 2 query heads per KV head, bf16."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(8)
    q = _rand(1, 4, 8192, 128, torch.bfloat16, gen)
    k = _rand(1, 2, 8192, 128, torch.bfloat16, gen)
    v = _rand(1, 2, 8192, 128, torch.bfloat16, gen)
    _check(q, k, v, True)


def test_prefill_strided_views_and_hf_query_layout():
    """K/V as views into a larger store ([B, H, capacity, D], first n tokens)
    and the query as the transposed projection HF passes ([B, S, H, D] viewed
    as [B, H, S, D])."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(3)
    B, Hq, Hkv, S, D, cap = 2, 8, 2, 600, 64, 2048
    kbuf = _rand(B, Hkv, cap, D, torch.float16, gen)
    vbuf = _rand(B, Hkv, cap, D, torch.float16, gen)
    q = _rand(B, S, Hq, D, torch.float16, gen).transpose(1, 2)
    _check(q, kbuf[:, :, :S], vbuf[:, :, :S], True)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_prefill_growing_logits_rescale(dtype):
    """Key norms grow along the sequence, so each row's maximum keeps rising by
    more than the lazy-rescaling threshold from tile to tile; plus large
    logits (|s| up to a few hundred)."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(11)
    B, Hq, Hkv, S, D = 1, 4, 4, 1500, 64
    q = _rand(B, Hq, S, D, dtype, gen, 2.0)
    ramp = torch.linspace(0.1, 6.0, S, device="cuda")[None, None, :, None]
    k = (torch.randn((B, Hkv, S, D), generator=gen, device="cuda") * ramp).to(dtype)
    v = _rand(B, Hkv, S, D, dtype, gen)
    _check(q, k, v, True)


def test_prefill_rejects_unsupported():
    from helix_online_kv.prefill import prefill_attention, supported
    q = torch.randn(1, 2, 16, 96, device="cuda", dtype=torch.float16)
    assert not supported(q, q, q)
    with pytest.raises(ValueError, match="Expected"):
        prefill_attention(q, q, q)
    q32 = torch.randn(1, 2, 16, 64, device="cuda")
    assert not supported(q32, q32, q32)
    qh = q32.half()
    with pytest.raises(ValueError, match="kv_len >= q_len"):
        prefill_attention(qh, qh[:, :, :8], qh[:, :, :8])
    # heads aliasing tokens: strides that do not nest
    buf = torch.randn(4096, device="cuda", dtype=torch.float16)
    alias = torch.as_strided(buf, (1, 2, 16, 64), (4096, 64, 64, 1))
    assert not supported(alias, alias, alias)


def test_cdc03_model_prefill_runs_the_kernel():
    """A Hugging Face model under the "cdc03" attention: prefill logits agree
    with the same model under SDPA (every layer's prefill attention runs
    hokv_prefill_attention)."""
    transformers = pytest.importorskip("transformers")
    from helix_online_kv.cdc03_attention import CDC03Cache
    from helix_online_kv.config import OnlineKVConfig
    cfg = transformers.LlamaConfig(vocab_size=256, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=2048)
    import helix_online_kv.cdc03_attention as A
    calls = []
    real = A.prefill_attention

    def counting(*a, **kw):
        calls.append(a[0].shape)
        return real(*a, **kw)

    torch.manual_seed(0)
    model = transformers.LlamaForCausalLM(cfg).cuda().half().eval()
    ids = torch.randint(0, 256, (1, 700), device="cuda")
    A.prefill_attention = counting
    try:
        with torch.no_grad():
            dense = model(ids, past_key_values=transformers.DynamicCache(), use_cache=True).logits.float()
            kvc = OnlineKVConfig(calibration_tokens=128, hot_window=64, pq_subspaces=8, exact_layers=[0], top_k=32)
            cache = CDC03Cache(kvc, n_layers=2, batch=1, kv_heads=2, head_dim=64, capacity=1024).attach(model)
            ours = model(ids, past_key_values=cache, use_cache=True).logits.float()
    finally:
        A.prefill_attention = real
        model.config._attn_implementation = "sdpa"
    assert len(calls) == 2 and all(tuple(c) == (1, 4, 700, 64) for c in calls)
    assert (ours - dense).abs().max().item() < 5e-2
    assert (ours.argmax(-1) == dense.argmax(-1)).float().mean().item() > 0.99
