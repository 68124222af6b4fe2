"""Parity at the benchmarked geometry, run the way bench.py runs it.

8 sequences x 8 KV heads x 4 query heads per KV head, head_dim 128, PQ with
16 subspaces of 8 dims, 16384-token bf16 contexts, 31 layers: one decode step
through the public API (CDC03Store.decode per layer) captured in a CUDA graph
and replayed; then, for two (sequence, KV head) units of every layer, the PQ
codes, the selected sets and the outputs of the replayed step against the
oracle (codes bit-exact, selection exact up to documented near-ties, outputs
within max-abs 1e-2 and cosine 0.9999).
"""

import os
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def test_bench_geometry_31_layer_graph():
    import bench
    from helix_online_kv import _lib as L
    from helix_online_kv.cdc03 import CDC03Store
    w = bench.WORKLOAD
    B, Ls, H, Hq, D, S, M = (w["batch_per_gpu"], w["layers"], w["kv_heads"], w["q_heads"], w["head_dim"],
                             w["context"], w["pq_subspaces"])
    top_k, sink, hot = w["top_k"], w["sink_tokens"], w["hot_window"]
    scale = 1.0 / np.sqrt(D)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(4321)
    store = CDC03Store(B, Ls, H, D, S, n_subspaces=M, dtype=torch.bfloat16)
    for layer in range(Ls):
        bench._fill_layer(store, layer, gen)
        store.calibrate(layer, w["pq_calibration_tokens"])
        store.assign(layer, 0, S)
    store.seq_len.fill_(S)
    q = torch.randn((Ls, B, Hq, D), generator=gen, device="cuda").to(torch.bfloat16)
    out = torch.zeros_like(q)

    def step():
        for l in range(Ls):
            store.decode(l, q[l], scale, top_k, sink, hot, out=out[l])

    step()
    torch.cuda.synchronize()
    eager = out.clone()
    out.zero_()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            step()
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    L.device_status()
    assert torch.equal(out, eager), "graph replay differs from the eager step"
    ties = 0
    for l in range(Ls):
        units = [(l % B, (3 * l) % H), ((l + 5) % B, (3 * l + 4) % H)]
        res = bench._check_against_oracle(store, q, out, [l], units, scale, top_k, sink, hot)
        ties += res["near_tie_tokens"]
    assert ties <= 16
    del g
