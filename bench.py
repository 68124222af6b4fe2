"""CDC-03 decode-attention benchmark (one JSON line on rank 0).

Workload (the per-GPU shard of the Llama-3-8B 16K configuration): per GPU,
8 sequences x 16384 tokens of bf16 K/V for 31 compressed layers (layer 0
exact), 8 KV heads, 32 query heads (GQA 8:1... 4 query heads per KV head),
head_dim 128, PQ with 16 subspaces of 8 dims fitted on the first 128 tokens,
top-128 (4 sinks) plus a 256-token exact hot window.  K/V are seeded synthetic
values with the reference benchmark's distribution (per-channel scales
U(0.5, 2), N(0, 1) values, 4 Student-t(3) x 5 outlier channels per head);
queries are N(0, 1).  A step is one decode step: CDC-03 attention for every
sequence through all 31 layers, launched layer after layer (as a model
would), captured in a CUDA graph.  Sequences are sharded over GPUs with no
collective on the data path (weak scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""

from __future__ import annotations

import os

os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")
os.environ.setdefault("OMP_NUM_THREADS", "1")
os.environ.setdefault("MKL_NUM_THREADS", "1")

import argparse
import ctypes
import json
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "helix-online-kv_b200"))
sys.path.insert(0, REPO)

METRIC = "CDC-03 decode attn tokens/s/GPU @16K ctx; VQ-assign GB/s vs HBM peak"
WORKLOAD = dict(workload="cdc03_decode_llama3_8b_kv_16k", batch_per_gpu=8, context=16384, layers=31, kv_heads=8,
                q_heads=32, head_dim=128, pq_subspaces=16, pq_calibration_tokens=128, top_k=128, sink_tokens=4,
                hot_window=256, kv_dtype="bf16")


def _peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def _profile_field(kernel: str, field: str):
    """The `field:` line of `kernel`'s committed ncu summary (text after the colon), if any."""
    path = os.path.join(REPO, "profiles", f"{kernel}_llama3_16k.md")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith(field + ":"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def _traffic_from_profiles(kernel: str):
    """Per-launch DRAM bytes of `kernel` from the committed ncu summary, if any."""
    v = _profile_field(kernel, "traffic_bytes_per_launch")
    return float(v.split()[0]) if v else None


# ----------------------------------------------------------------------------- reference arm (CPU)
def config_for(w: dict, world: int) -> dict:
    """The workload's `config` object, identical in both arms."""
    step_bytes_note = "inputs larger than L2 (16.6 GB of K/V per GPU, 126 MB L2); no flush needed"
    return dict(w, global_batch=w["batch_per_gpu"] * world, parallelism=f"sequence-sharded x{world}",
                l2=step_bytes_note)


def _ref_unit(seed: int, S: int, D: int, M: int, G: int):
    from oracle import hokv_oracle as O
    K, V = O.gen_kv(seed, 1, 1, S, D)
    K = O.to_fp16_values(K[0, 0])
    V = O.to_fp16_values(V[0, 0])
    cents, _ = O.pq_fit(K[:128], M=M, sub_clusters=256)
    codes = O.pq_assign(K, cents)
    Q = O.gen_queries(seed, 1, G, D)[0]
    return K, V, codes, cents, Q


def _ref_worker(seed, shape, per_step, n_steps, barrier, results):
    """One host core: builds its own (sequence, KV head) unit once, then at every
    step, between two barriers, runs `per_step` CDC-03 head-queries on it."""
    S, D, M, G, top_k, sink, hot = shape
    cpus = sorted(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else []
    if cpus:   # one worker per host core, kept there
        os.sched_setaffinity(0, {cpus[(seed - 1000) % len(cpus)]})
    from oracle import hokv_oracle as O
    K, V, codes, cents, Q = _ref_unit(seed, S, D, M, G)
    scale = 1.0 / np.sqrt(D)
    times = []
    for _ in range(n_steps):
        barrier.wait(timeout=600)
        t0 = time.perf_counter()
        for i in range(per_step):
            O.cdc03_hot_attention(Q[i % G], K, V, codes, cents, scale, top_k, sink, hot)
        times.append(time.perf_counter() - t0)
        barrier.wait(timeout=600)
    results.put(times)


def cpu_rate(n_workers: int, per_step: int, n_steps: int, shape):
    """Wall-clock seconds of each step of `n_workers` processes (one BLAS thread
    each) running `per_step` head-queries apiece of the oracle's CDC-03; a step
    runs from the barrier that releases every worker to the barrier that the
    last of them reaches.  shape = (S, D, M, G, top_k, sink, hot)."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[var] = "1"   # read by each worker's numpy at import
    barrier = ctx.Barrier(n_workers + 1)
    results = ctx.Queue()
    procs = [ctx.Process(target=_ref_worker, args=(1000 + i, shape, per_step, n_steps, barrier, results), daemon=True)
             for i in range(n_workers)]
    for pr in procs:
        pr.start()
    steps = []
    try:
        for _ in range(n_steps):
            barrier.wait(timeout=900)   # the first pass waits for every worker's unit
            t0 = time.perf_counter()
            barrier.wait(timeout=900)
            steps.append(time.perf_counter() - t0)
        worker_times = [results.get(timeout=120) for _ in procs]
    finally:
        for pr in procs:
            pr.join(timeout=30)
            if pr.is_alive():
                pr.terminate()
    return steps, worker_times


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if rank != 0:
        return 0
    w = dict(WORKLOAD)
    if args.layers:
        w["layers"] = args.layers
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    G = w["q_heads"] // w["kv_heads"]
    shape = (w["context"], w["head_dim"], w["pq_subspaces"], G, w["top_k"], w["sink_tokens"], w["hot_window"])
    hq_per_token = w["layers"] * w["q_heads"]
    step_hq = w["batch_per_gpu"] * world * hq_per_token          # head-queries of one decode step
    per_worker = min(-(-step_hq // cores), args.ref_cap)
    # one core alone first (same per-worker sample), then every core
    one_steps, _ = cpu_rate(1, per_worker, 2, shape)
    one_rate = per_worker / min(one_steps)
    steps, _ = cpu_rate(cores, per_worker, args.warmup + args.steps, shape)
    timed = steps[args.warmup:]
    step_s = statistics.median(timed)
    rate = cores * per_worker / step_s                            # head-queries/s, all cores
    tok_s = rate / hq_per_token
    sample = (f"{cores} processes (one per host core, one BLAS thread each) x {per_worker} head-queries per step "
              f"at S={w['context']}, D={w['head_dim']}, M={w['pq_subspaces']}: "
              + ("the whole decode step" if per_worker * cores >= step_hq else
                 f"a sample of {per_worker * cores} of the step's {step_hq} head-queries")
              + f"; one core alone: {one_rate:.1f} head-queries/s")
    line = {
        "impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (numpy)", "data": "synthetic",
        "config": config_for(w, world),
        "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample,
                         "single_core_value": one_rate / hq_per_token,
                         "parallel_efficiency": rate / (cores * one_rate),
                         "impl_note": "the oracle's restatement of the reference's numpy hybrid_pq_attention "
                                      "(compressed_attention.py:315-412) with the hot window"},
        "ms_per_step_min": min(timed) * 1e3, "ms_per_step_max": max(timed) * 1e3,
        "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- device arm
def _fill_layer(store, layer, gen):
    import torch
    B, H, cap, D = store.B, store.H, store.cap, store.D
    for b in range(B):
        scale = torch.rand((H, 1, D), generator=gen, device="cuda") * 1.5 + 0.5
        k = torch.randn((H, cap, D), generator=gen, device="cuda") * scale
        scale_v = torch.rand((H, 1, D), generator=gen, device="cuda") * 1.5 + 0.5
        v = torch.randn((H, cap, D), generator=gen, device="cuda") * scale_v
        for t in (k, v):
            cols = torch.argsort(torch.rand((H, D), generator=gen, device="cuda"), dim=1)[:, :4]
            z = torch.randn((H, cap, 4), generator=gen, device="cuda")
            chi = (torch.randn((H, cap, 4, 3), generator=gen, device="cuda") ** 2).sum(-1)
            tv = z / torch.sqrt(chi / 3.0) * 5.0
            t.scatter_(2, cols[:, None, :].expand(H, cap, 4), tv)
        store.k[layer, b] = k.to(store.k.dtype)
        store.v[layer, b] = v.to(store.v.dtype)


class Clocks:
    def __init__(self, gpu_index: int):
        self.path = tempfile.mktemp(suffix=".csv")
        self.proc = None
        self.gpu = gpu_index

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu),
                 "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 6:
                    continue
                try:
                    sm.append(float(parts[0]))
                    mx.append(float(parts[1]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[2:6]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def _time_graph(graph, n, barrier):
    """Device milliseconds of `n` replays of `graph`, between barriers."""
    import torch
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def _check_against_oracle(store, q, out, layers, units, scale, top_k, sink, hot):
    """The decode outputs of `units` (b, h) of `layers` against the oracle: PQ
    codes bit-exact, selected sets exact up to documented near-ties, outputs
    within max-abs 1e-2 and cosine 0.9999.  Raises RuntimeError on a mismatch."""
    import torch
    from oracle import hokv_oracle as O
    S, M, G = int(store.seq_len[0].item()), store.M, q.shape[2] // store.H
    worst, ties = 0.0, 0
    for l in layers:
        o_dev, (sel, _, cnt) = store.decode(l, q[l], scale, top_k, sink, hot, out_dtype=torch.float32,
                                            return_selection=True)
        for b, h in units:
            Kh = store.k[l, b, h, :S].float().cpu().numpy()
            Vh = store.v[l, b, h, :S].float().cpu().numpy()
            kk = store.cb_k[l, b, h].cpu().numpy()
            cb = store.codebook[l, b, h].cpu().numpy()
            cents = [cb[s_, :kk[s_]] for s_ in range(M)]
            codes = store.codes[l, b, h, :S, :M].cpu().numpy()
            if not np.array_equal(codes[:S - hot], O.pq_assign(Kh[:S - hot], cents)):
                raise RuntimeError(f"check failed: layer {l} unit {(b, h)}: PQ codes differ from the oracle")
            for g in range(G):
                hq = h * G + g
                qv = q[l, b, hq].float().cpu().numpy()
                rsel, _, rout = O.cdc03_hot_attention(qv, Kh, Vh, codes, cents, scale, top_k, sink, hot)
                got = np.sort(sel[b, hq, :int(cnt[b, hq])].cpu().numpy())
                if not np.array_equal(got, rsel):
                    approx = O.pq_gather(O.pq_tables(qv, cents), codes[:S - hot]) * np.float32(scale)
                    diff = np.setxor1d(got, rsel)
                    masked = approx.astype(np.float64)
                    masked[:sink] = -np.inf
                    bound = np.sort(masked)[-(top_k - sink)]
                    tol = 8 * np.spacing(np.float32(abs(bound)))
                    if len(diff) > 4 or any(abs(float(approx[t]) - bound) > tol for t in diff):
                        raise RuntimeError(f"check failed: layer {l} head {(b, hq)}: selection differs {diff}")
                    ties += len(diff)
                o = o_dev[b, hq].cpu().numpy()
                err = float(np.max(np.abs(o - rout)))
                worst = max(worst, err)
                if err > 1e-2 or O.cosine(o, rout) < 0.9999:
                    raise RuntimeError(f"check failed: layer {l} head {(b, hq)}: max-abs {err}")
                # the timed step's own output for this head (stored bf16: 2^-8 relative
                # rounding) agrees with the fp32 re-run
                if not torch.allclose(out[l, b, hq].float().cpu(), o_dev[b, hq].cpu(), atol=1e-2, rtol=2.0 ** -8):
                    raise RuntimeError(f"check failed: layer {l} head {(b, hq)}: timed output differs")
    return {"layers": list(layers), "units": [list(u) for u in units], "head_queries": len(layers) * len(units) * G,
            "max_abs": worst, "near_tie_tokens": ties, "passed": True}


# ----------------------------------------------------------------------------- extra workloads
def _fill_uniform(store, layer, gen, n_tokens):
    """Seeded synthetic K/V (the reference benchmark's distribution) for tokens
    [0, n_tokens) of every sequence and head of one layer, in place."""
    import torch
    B, H, D = store.B, store.H, store.D
    for b in range(B):
        for t in (store.k, store.v):
            scale = torch.rand((H, 1, D), generator=gen, device="cuda") * 1.5 + 0.5
            x = torch.randn((H, n_tokens, D), generator=gen, device="cuda") * scale
            cols = torch.argsort(torch.rand((H, D), generator=gen, device="cuda"), dim=1)[:, :4]
            z = torch.randn((H, n_tokens, 4), generator=gen, device="cuda")
            chi = (torch.randn((H, n_tokens, 4, 3), generator=gen, device="cuda") ** 2).sum(-1)
            x.scatter_(2, cols[:, None, :].expand(H, n_tokens, 4), z / torch.sqrt(chi / 3.0) * 5.0)
            t[layer, b, :, :n_tokens] = x.to(t.dtype)
            del x, z, chi


def long_context(world, rank, steps, contexts=(32768, 131072)):
    """TinyLlama-architecture KV geometry (4 KV heads, 32 query heads, head_dim
    64, PQ 8 x 8), 8 sequences sharded over the ranks, layers 1-21 compressed
    (top-128 with 4 sinks + a 256-token hot window): decode tokens/s of one
    step over the 21 layers at each context length, device-timed."""
    import torch
    from helix_online_kv import _lib as L
    from helix_online_kv.cdc03 import CDC03Store
    from helix_online_kv.sharding import max_over_ranks, shard_range
    B = len(shard_range(8, world, rank)) or 1
    H, Hq, D, M, Ls = 4, 32, 64, 8, 21
    res = {"geometry": "TinyLlama KV: 4 KV heads, 32 query heads, head_dim 64, PQ 8x8, 21 compressed layers",
           "sequences_total": 8, "sequences_per_gpu": B}
    gen = torch.Generator(device="cuda")
    gen.manual_seed(77 + rank)
    for S in contexts:
        store = CDC03Store(B, Ls, H, D, S, n_subspaces=M, dtype=torch.float16)
        for l in range(Ls):
            _fill_uniform(store, l, gen, S)
            store.calibrate(l, 128)
            store.assign(l, 0, S)
        store.seq_len.fill_(S)
        q = torch.randn((Ls, B, Hq, D), generator=gen, device="cuda").to(torch.float16)
        out = torch.empty_like(q)
        scale = 1.0 / np.sqrt(D)

        def step():
            for l in range(Ls):
                store.decode(l, q[l], scale, 128, 4, 256, out=out[l])

        step()
        torch.cuda.synchronize()
        L.device_status()
        g = torch.cuda.CUDAGraph()
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            with torch.cuda.graph(g, stream=st):
                step()
        torch.cuda.current_stream().wait_stream(st)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1), device="cuda") / steps
        Sc = S - 256
        step_bytes = Ls * (B * H * Sc * M + B * Hq * 128 * D * 2 * 2 + B * H * 256 * D * 2 * 2 + B * H * M * 128 * 8 * 4
                           + B * Hq * D * 2 * 2)
        res[f"ctx_{S}"] = {"ms_per_step": ms, "tokens_per_s": B * world / (ms / 1e3),
                           "us_per_layer": ms * 1e3 / Ls, "step_hbm_gbs": step_bytes / (ms * 1e-3) / 1e9,
                           "index_bytes_per_step": Ls * B * H * Sc * M}
        del g, store, q, out
        torch.cuda.empty_cache()
    return res


def head_sharded(world, rank, steps, S=16384, Ls=31):
    """One sequence (fewer sequences than GPUs) at the Llama-3-8B KV geometry
    (8 KV heads, 32 query heads, head_dim 128, PQ 16 x 8) and 16K context,
    31 layers, its KV heads split over the ranks; after every layer one
    all-gather of the [1, 32, 128] outputs over NCCL, whose result is the next
    layer's queries (a stand-in for the model's projections), so that each
    layer waits for the collective.  The step (decodes and collectives) is
    captured in a CUDA graph where the collective library allows it, else
    launched eagerly (the line names which); device-timed, max over ranks."""
    import torch
    from helix_online_kv.cdc03 import CDC03Store
    from helix_online_kv.sharding import gather_heads, head_shard, max_over_ranks
    H_all, G, D, M = 8, 4, 128, 16
    heads = head_shard(H_all, world, rank)
    H = len(heads)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(99 + rank)
    store = CDC03Store(1, Ls, max(H, 1), D, S, n_subspaces=M, dtype=torch.bfloat16) if H else None
    if store is not None:
        for l in range(Ls):
            _fill_uniform(store, l, gen, S)
            store.calibrate(l, 128)
            store.assign(l, 0, S)
        store.seq_len.fill_(S)
    q0 = torch.randn((1, H_all * G, D), generator=gen, device="cuda").to(torch.bfloat16)
    qs = slice(heads.start * G, heads.stop * G)
    scale = 1.0 / np.sqrt(D)

    def step():
        q = q0
        for l in range(Ls):
            if store is not None:
                o = store.decode(l, q[:, qs].contiguous(), scale, 128, 4, 256)
            else:
                o = torch.empty((1, 0, D), dtype=q.dtype, device="cuda")
            q = gather_heads(o, H_all, G)
        return q

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    # the step (decodes and collectives) captured in one CUDA graph when the
    # collective library allows it, else eager
    graph, mode = None, "eager"
    try:
        graph = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream()
        cs.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(cs):
            with torch.cuda.graph(graph, stream=cs):
                step()
        torch.cuda.current_stream().wait_stream(cs)
        graph.replay()
        torch.cuda.synchronize()
        mode = "CUDA graph"
    except Exception:   # noqa: BLE001 - capture unsupported here: time the eager step
        graph = None
        torch.cuda.synchronize()
    run = graph.replay if graph is not None else step
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), device="cuda") / steps
    del graph
    return {"geometry": "1 sequence, Llama-3-8B KV, 16K context, 31 layers, KV heads split over the GPUs",
            "kv_heads_per_gpu": H, "ms_per_step": ms, "tokens_per_s": 1e3 / ms, "launch": mode,
            "collective": "NCCL all-gather of the [1, 32, 128] attention outputs after every layer"
                          if world > 1 else "none (one GPU)"}


def tinyllama_generate(prompt=1024, new=256, seed=0):
    """TinyLlama-1.1B architecture with random-init fp16 weights (22 layers,
    d_model 2048, 32 heads, 4 KV heads, SwiGLU 5632, vocab 32000, RoPE 1e4):
    a uniform-random 1024-token prompt, batch 1, then 256 greedy decode steps,
    once through the dense cache (SDPA) and once through CDC03Cache
    (exact_layers=[0], calibration 128, hot window 256, top-128 with 4 sinks,
    PQ 8 x 8).  Device time of the prefill and of the decode loop; the two
    runs' last prefill logits and first decode-step logits (same input token)
    compared; greedy tokens shared with the dense run; cache bytes."""
    import torch
    import transformers
    from helix_online_kv.cdc03_attention import CDC03Cache
    from helix_online_kv.config import OnlineKVConfig
    cfg = transformers.LlamaConfig(vocab_size=32000, hidden_size=2048, intermediate_size=5632, num_hidden_layers=22,
                                   num_attention_heads=32, num_key_value_heads=4, max_position_embeddings=4096,
                                   rope_theta=10000.0)
    torch.manual_seed(seed)
    with torch.device("cuda"):
        model = transformers.LlamaForCausalLM(cfg)
    model = model.half().eval()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    ids = torch.randint(0, cfg.vocab_size, (1, prompt), generator=gen, device="cuda")
    kvc = OnlineKVConfig(calibration_tokens=128, hot_window=256, pq_subspaces=8, exact_layers=[0], top_k=128,
                         sink_tokens=4)
    ev = lambda: torch.cuda.Event(enable_timing=True)   # noqa: E731

    def run(make_cache, attn, prompt_ids, n_new, first_tok=None):
        cache = make_cache()
        if attn != "cdc03":
            model.config._attn_implementation = attn
        toks = []
        with torch.no_grad():
            a, b, c = ev(), ev(), ev()
            a.record()
            pre = model(prompt_ids, past_key_values=cache, use_cache=True).logits[:, -1:]
            tok = pre.argmax(-1) if first_tok is None else first_tok
            tok0 = tok
            b.record()
            first = None
            for i in range(n_new):
                logits = model(tok, past_key_values=cache, use_cache=True).logits[:, -1:]
                if first is None:
                    first = logits.float().flatten()
                tok = logits.argmax(-1)
                toks.append(tok)
            c.record()
            torch.cuda.synchronize()
        return (cache, torch.cat(toks, 1).flatten(), first, a.elapsed_time(b), b.elapsed_time(c),
                pre.float().flatten(), tok0)

    make_cdc03 = lambda: CDC03Cache(kvc, n_layers=22, batch=1, kv_heads=4, head_dim=64,   # noqa: E731
                                    capacity=prompt + new + 1, dtype=torch.float16).attach(model)
    # the dense run uses SDPA under a name of its own, so that, like "cdc03", it
    # skips the per-step mask construction transformers does for "sdpa"
    # (unpadded batch: causal prefill, maskless decode steps)
    from transformers import AttentionInterface
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    AttentionInterface.register("sdpa_nomask", sdpa_attention_forward)
    # each path runs once untimed over the same prompt and lengths first: torch's
    # SDPA backend plans once per new sequence length (tens of ms each), and
    # the second pass times the steady state of both paths alike
    run(transformers.DynamicCache, "sdpa_nomask", ids, new)
    dense, d_toks, d_first, d_pre, d_dec, d_plog, d_tok0 = run(transformers.DynamicCache, "sdpa_nomask", ids, new)
    dense_bytes = sum(t.element_size() * t.nelement() for layer in dense.layers for t in (layer.keys, layer.values))
    del dense
    run(make_cdc03, "cdc03", ids, new, first_tok=d_tok0)
    cache, c_toks, c_first, c_pre, c_dec, c_plog, _ = run(make_cdc03, "cdc03", ids, new, first_tok=d_tok0)
    model.config._attn_implementation = "sdpa"
    rep = cache.memory_report()
    agree = int((c_toks == d_toks).cumprod(0).sum().item())
    res = {"model": "TinyLlama-1.1B architecture, random-init fp16 weights", "prompt_tokens": prompt,
           "decode_steps": new,
           "dense_sdpa": {"attention": "torch SDPA, no per-step mask construction", "prefill_ms": d_pre, "decode_tokens_per_s": new / (d_dec / 1e3), "kv_bytes": dense_bytes},
           "cdc03_cache": {"prefill_ms": c_pre, "decode_tokens_per_s": new / (c_dec / 1e3),
                           "kv_bytes": rep["total_bytes"], "calibration_complete": rep["calibration_complete"]},
           "greedy_tokens_equal_to_dense_before_first_difference": agree,
           "prefill_logits_cosine": float(torch.nn.functional.cosine_similarity(c_plog, d_plog, dim=0).item()),
           "first_decode_step_logits_cosine": float(
               torch.nn.functional.cosine_similarity(c_first, d_first, dim=0).item()),
           "note": "HF eager decode loop (Python and launch overhead included), the second of two identical "
                   "runs of each path; CDC-03 attends the top-128 cold tokens plus the 256-token hot window of each "
                   "compressed layer, and random-init weights give near-uniform attention, so greedy tokens of "
                   "the two runs part early (the kernels' parity is tested against the oracle instead)"}
    del cache, model
    torch.cuda.empty_cache()
    return res


def path_a_sweep(reps=20):
    """Path A, the fused Q.K^T over scalar-VQ codes (fused_scalar_vq_qkt, the
    reference's Triton kernel triton_attention.py:25-66 restated as
    hokv_scalar_vq_qkt): one head_dim-128 query against S tokens of uint8
    codes and a 256-entry fp32 codebook, fp32 accumulation.  Device time per
    call (back-to-back calls after a warm-up) and the index bytes read per
    second; at 1M tokens the 128 MB of codes exceed L2."""
    import torch
    from helix_online_kv.triton_attention import fused_scalar_vq_qkt
    gen = torch.Generator(device="cuda")
    gen.manual_seed(21)
    D = 128
    q = torch.randn(D, generator=gen, device="cuda")
    cb = torch.randn(256, generator=gen, device="cuda")
    res = {}
    for S in (16384, 131072, 1048576):
        idx = torch.randint(0, 256, (S, D), generator=gen, device="cuda", dtype=torch.int32).to(torch.uint8)
        fused_scalar_vq_qkt(q, idx, cb, 0.088)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fused_scalar_vq_qkt(q, idx, cb, 0.088)
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / reps
        nbytes = S * D + S * 4   # codes in, scores out
        res[f"S_{S}"] = {"us": ms * 1e3, "gbs": nbytes / (ms * 1e-3) / 1e9}
        del idx
    return res


def prefill_attention_sweep(reps=10):
    """Exact causal prefill attention of one layer (hokv_prefill_attention)
    beside torch's SDPA on the same tensors: a 1024-token TinyLlama prompt
    (32 query / 4 KV heads, head_dim 64, f16), and 4K and 16K Llama-3-8B
    prompts (32 / 8 heads, head_dim 128, bf16), batch 1.  Device time per call
    (the mean of `reps` back-to-back calls after a warm-up), causal FLOPs
    4 * Sq * (Sq + 1) / 2 * D * H_q, the result's max deviation from SDPA."""
    import torch
    import torch.nn.functional as F
    from helix_online_kv.prefill import prefill_attention
    ev = lambda: torch.cuda.Event(enable_timing=True)   # noqa: E731
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5)
    res = {}
    for name, Hq, Hkv, S, D, dt in (("tinyllama_1k", 32, 4, 1024, 64, torch.float16),
                                    ("llama3_4k", 32, 8, 4096, 128, torch.bfloat16),
                                    ("llama3_16k", 32, 8, 16384, 128, torch.bfloat16)):
        q = torch.randn((1, S, Hq, D), generator=gen, device="cuda").to(dt).transpose(1, 2)
        k = torch.randn((1, Hkv, S, D), generator=gen, device="cuda").to(dt)
        v = torch.randn((1, Hkv, S, D), generator=gen, device="cuda").to(dt)
        ours_fn = lambda: prefill_attention(q, k, v, None, True)   # noqa: E731
        ref_fn = lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)   # noqa: E731
        out = {}
        for tag, fn in (("hokv", ours_fn), ("sdpa", ref_fn)):
            r = fn()
            torch.cuda.synchronize()
            a, b = ev(), ev()
            a.record()
            for _ in range(reps):
                fn()
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / reps
            flops = 4.0 * S * (S + 1) / 2 * D * Hq
            out[tag] = {"us": ms * 1e3, "tflops": flops / (ms * 1e-3) / 1e12}
            out[tag + "_out"] = r
        dev = (out.pop("hokv_out").float() - out.pop("sdpa_out").transpose(1, 2).float()).abs().max().item()
        res[name] = {"q_heads": Hq, "kv_heads": Hkv, "tokens": S, "head_dim": D, "dtype": str(dt).split(".")[-1],
                     "hokv_prefill_attention": out["hokv"], "torch_sdpa": out["sdpa"],
                     "max_abs_diff_vs_sdpa": dev}
        del q, k, v
    return res


def encoder_sweep(ns=(1, 16, 256, 4096, 32768), reps=5):
    """Online encoder sweep: N new fp16 K vectors per step assigned to per-(layer,
    head) k=256 codebooks, 22 layers x 4 KV heads x head_dim 64, for the scalar,
    vector (64-dim) and product (8 x 8) codebooks; plus the calibrations on 128
    tokens (scalar 10 iterations, vector / product up to 30).  Device time per
    step (all 88 codebooks of one kind), inputs resident."""
    import torch
    from helix_online_kv import _lib as L
    lib = L.lib()
    sets, D, M, sd, slots = 22 * 4, 64, 8, 8, 256
    gen = torch.Generator(device="cuda")
    gen.manual_seed(11)
    nmax, ncal = max(ns), 2048
    x = (torch.randn((sets, nmax, D), generator=gen, device="cuda")
         * (torch.rand((sets, 1, D), generator=gen, device="cuda") * 1.5 + 0.5)).to(torch.float16)
    cal = x[:, :ncal].float().contiguous()
    ev = lambda: torch.cuda.Event(enable_timing=True)   # noqa: E731

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        a, b = ev(), ev()
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    # codebooks: scalar (per set over its values), vector (64-dim), product (8 x 8), fitted on 2048 tokens
    sc_c = torch.zeros((sets, slots), dtype=torch.float32, device="cuda")
    sc_k = torch.zeros(sets, dtype=torch.int32, device="cuda")
    it = torch.zeros(sets * M, dtype=torch.int32, device="cuda")
    mse = torch.zeros(sets * M, dtype=torch.float64, device="cuda")
    vq_c = torch.zeros((sets, slots, D), dtype=torch.float32, device="cuda")
    vq_k = torch.zeros(sets, dtype=torch.int32, device="cuda")
    pq_c = torch.zeros((sets, M, slots, sd), dtype=torch.float32, device="cuda")
    pq_k = torch.zeros((sets, M), dtype=torch.int32, device="cuda")

    def fit_scalar(n_tok):
        data = cal[:, :n_tok].reshape(sets, n_tok * D).contiguous()
        ws = L.workspace(lib.hokv_scalar_kmeans_workspace_size(n_tok * D, sets))
        L.check(lib.hokv_scalar_kmeans(L.ptr(data), n_tok * D, n_tok * D, sets, slots, 10, 1e-3, L.ptr(sc_c),
                                       L.ptr(sc_k), L.ptr(it), L.ptr(mse), None, L.ptr(ws), ws.numel(), L.stream()),
                "scalar_kmeans")

    def fit_vq(n_tok):
        data = cal[:, :n_tok].contiguous()
        ws = L.workspace(lib.hokv_vq_kmeans_workspace_size(n_tok, D, sets))
        L.check(lib.hokv_vq_kmeans(L.ptr(data), n_tok, D, D, n_tok * D, sets, slots, 30, 1e-4, L.ptr(vq_c), slots,
                                   L.ptr(vq_k), L.ptr(it), L.ptr(mse), L.ptr(ws), ws.numel(), L.stream()), "vq_kmeans")

    def fit_pq(n_tok):
        data = cal[:, :n_tok].reshape(sets, n_tok, M, sd).permute(0, 2, 1, 3).contiguous()
        ws = L.workspace(lib.hokv_vq_kmeans_workspace_size(n_tok, sd, sets * M))
        L.check(lib.hokv_vq_kmeans(L.ptr(data), n_tok, sd, sd, n_tok * sd, sets * M, slots, 30, 1e-4, L.ptr(pq_c),
                                   slots, L.ptr(pq_k), L.ptr(it), L.ptr(mse), L.ptr(ws), ws.numel(), L.stream()),
                "pq_kmeans")

    res = {"codebooks": "22 layers x 4 KV heads, head_dim 64, k=256; fp16 inputs",
           "calibration_ms_128_tokens": {"scalar_10_iters": timed(lambda: fit_scalar(128)),
                                         "vector_64d": timed(lambda: fit_vq(128)),
                                         "product_8x8": timed(lambda: fit_pq(128))}}
    fit_scalar(ncal)
    fit_vq(ncal)
    fit_pq(ncal)
    torch.cuda.synchronize()
    out = torch.zeros((sets, nmax, D), dtype=torch.uint8, device="cuda")
    for n in ns:
        xv = x[:, :n]
        r = {}
        r["scalar_ms"] = timed(lambda: L.check(lib.hokv_scalar_assign(
            L.ptr(xv), L.F16, n * D, nmax * D, L.ptr(sc_c), slots, slots, L.ptr(out), nmax * D, sets, L.stream()),
            "scalar_assign"))
        order = L.dot_order_for(n, D)
        r["vector_ms"] = timed(lambda: L.check(lib.hokv_pq_assign(
            L.ptr(xv), L.F16, n, D, nmax * D, 1, D, L.ptr(vq_c), slots, slots * D, L.ptr(vq_k), 1, L.ptr(out), 1,
            nmax * D, sets, order, L.stream()), "vq_assign"))
        order = L.dot_order_for(n, sd)
        r["product_ms"] = timed(lambda: L.check(lib.hokv_pq_assign(
            L.ptr(xv), L.F16, n, D, nmax * D, M, sd, L.ptr(pq_c), slots, M * slots * sd, L.ptr(pq_k), M,
            L.ptr(out), M, nmax * D, sets, order, L.stream()), "pq_assign"))
        bytes_in = sets * n * D * 2
        for kind, per in (("scalar", D), ("vector", 1), ("product", M)):
            r[f"{kind}_gbs"] = (bytes_in + sets * n * per) / (r[f"{kind}_ms"] * 1e-3) / 1e9
        res[f"N_{n}"] = r
    L.device_status()
    return res


def run_ours(args):
    import torch
    import torch.distributed as dist

    from helix_online_kv import _lib as L
    from helix_online_kv.cdc03 import CDC03Store
    from helix_online_kv.sharding import gather_outputs, max_over_ranks

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    L.require_device()
    w = dict(WORKLOAD)
    if args.layers:
        w["layers"] = args.layers
    B, Ls, H, Hq, D, S, M = (w["batch_per_gpu"], w["layers"], w["kv_heads"], w["q_heads"], w["head_dim"],
                             w["context"], w["pq_subspaces"])
    top_k, sink, hot = w["top_k"], w["sink_tokens"], w["hot_window"]
    scale = 1.0 / np.sqrt(D)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1234 + rank)
    store = CDC03Store(B, Ls, H, D, S, n_subspaces=M, dtype=torch.bfloat16)
    t_setup = time.perf_counter()
    for layer in range(Ls):
        _fill_layer(store, layer, gen)
        store.calibrate(layer, w["pq_calibration_tokens"])
        store.assign(layer, 0, S)
    store.seq_len.fill_(S)
    torch.cuda.synchronize()
    L.device_status()
    t_setup = time.perf_counter() - t_setup
    q = (torch.randn((Ls, B, Hq, D), generator=gen, device="cuda")).to(torch.bfloat16)
    out = torch.empty_like(q)
    lib = L.lib()
    args_l = [store.args(l, q[l], out[l], scale, top_k, sink, hot) for l in range(Ls)]
    refs = [ctypes.byref(a) for a in args_l]

    def step(stream_ptr):
        for r in refs:
            st = lib.hokv_cdc03_decode(r, stream_ptr)
            if st:
                L.check(st, "cdc03_decode")

    def api_step():
        # the public Python API a model calls, one layer after another
        for l in range(Ls):
            store.decode(l, q[l], scale, top_k, sink, hot, out=out[l])

    # eager warm-up (sets kernel attributes, sizes the workspace), then one step in a graph
    step(L.stream())
    api_step()
    torch.cuda.synchronize()
    L.device_status()
    cap_stream = torch.cuda.Stream()

    def capture(fn):
        g = torch.cuda.CUDAGraph()
        cap_stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(cap_stream):
            with torch.cuda.graph(g, stream=cap_stream):
                fn()
        torch.cuda.current_stream().wait_stream(cap_stream)
        torch.cuda.synchronize()
        return g

    graph = capture(lambda: step(L.stream()))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    warm = max(args.warmup, 3)
    for _ in range(warm):
        graph.replay()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        ev0.record()
        for _ in range(args.steps):
            graph.replay()
        ev1.record()
        torch.cuda.synchronize()
        # the same K-step region again, for the spread of the measurement
        repeats = [_time_graph(graph, args.steps, barrier) for _ in range(args.repeats)]
    ms = max_over_ranks(ev0.elapsed_time(ev1), device="cuda")
    repeats = [max_over_ranks(r, device="cuda") / args.steps for r in repeats]
    barrier()
    ms_step = ms / args.steps
    tokens = B * world * args.steps
    value = tokens / (ms / 1e3)

    # per-kernel attribution: each stage alone, all layers in one graph, so the
    # average launch duration carries no host launch gaps (k7 re-reads the
    # candidate lists the step left, which is the same work)
    n_att = max(3, min(args.steps, 10))

    def stage_ms(fn, name):
        g = capture(lambda: [L.check(fn(r, L.stream()), name) for r in refs])
        g.replay()
        torch.cuda.synchronize()
        t = _time_graph(g, n_att, torch.cuda.synchronize)
        del g
        return t / (n_att * Ls)

    k6_ms = stage_ms(lib.hokv_cdc03_candidates, "candidates")
    k7_ms = stage_ms(lib.hokv_cdc03_attend, "attend")
    graph.replay()   # the step's own outputs again
    torch.cuda.synchronize()

    # algorithmic bytes per launch (one layer)
    Sc = S - hot
    ceff = float(store.cb_k[0].float().mean().item())
    units = B * H
    k6_bytes = units * Sc * M + units * M * ceff * (D // M) * 4 + B * Hq * D * 2
    k7_bytes = B * Hq * top_k * D * 2 * 2 + units * hot * D * 2 * 2 + B * Hq * D * 2 * 2
    peak, peak_kind = _peaks()
    k6_gbs = k6_bytes / (k6_ms * 1e-3) / 1e9
    k7_gbs = k7_bytes / (k7_ms * 1e-3) / 1e9
    s1 = ("k6_candidates (tables built in thread-block clusters)", k6_gbs, k6_bytes, k6_ms)
    s2 = ("k7_select_attend", k7_gbs, k7_bytes, k7_ms)
    dom, other = (s1, s2) if k6_ms >= k7_ms else (s2, s1)

    def roof(entry):
        name, gbs, nbytes, kms = entry
        key = "k7_select_attend" if name.startswith("k7") else "k6_candidates"
        return {"kernel": name, "bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                "traffic": _traffic_from_profiles(key), "algorithmic_bytes": nbytes, "avg_launch_ms": kms,
                "traffic_note": _profile_field(key, "traffic_note"),
                "peak_kind": f"{peak_kind} (hbm_gbs, MEASURED_PEAKS.json)" if peak_kind == "measured" else peak_kind}

    step_bytes = (k6_bytes + k7_bytes) * Ls

    # end to end through the public API (CDC03Store.decode per layer): pinned host
    # queries in, host outputs out, every step; captured in a graph (as a serving
    # loop would), and eager; at N > 1 every step also all-gathers the last
    # layer's outputs of every rank over NCCL
    q_host = q.cpu().pin_memory()
    out_host = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    api_graph = capture(api_step)
    gathered_host = None
    if world > 1:
        gathered_host = torch.empty((B * world, Hq, D), dtype=out.dtype).pin_memory()

    def e2e_loop(n, use_graph):
        for _ in range(n):
            q.copy_(q_host, non_blocking=True)
            if use_graph:
                api_graph.replay()
            else:
                api_step()
            out_host.copy_(out, non_blocking=True)
            if world > 1:
                gathered_host.copy_(gather_outputs(out[Ls - 1], sizes=[B] * world), non_blocking=True)

    e2e = {}
    for name, use_graph in (("graph", True), ("eager", False)):
        e2e_loop(2, use_graph)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        e2e_loop(args.steps, use_graph)
        e1.record()
        torch.cuda.synchronize()
        e2e[name] = max_over_ranks(e0.elapsed_time(e1), device="cuda")
    h2d = q.numel() * q.element_size()
    d2h = out.numel() * out.element_size() + (gathered_host.numel() * gathered_host.element_size() if world > 1 else 0)

    # VQ-assign throughput: PQ codes for a fresh 8192-token block of every (b, h) of one layer
    n_new = 8192
    torch.cuda.synchronize()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    store.assign(0, 0, n_new)
    a0.record()
    for _ in range(3):
        store.assign(0, 0, n_new)
    a1.record()
    torch.cuda.synchronize()
    as_ms = a0.elapsed_time(a1) / 3
    as_bytes = units * n_new * (D * 2 + M)
    as_gbs = as_bytes / (as_ms * 1e-3) / 1e9
    graph.replay()
    torch.cuda.synchronize()

    # the other workloads of the reference's benchmark set, each on its own
    # (its failure is reported, never the headline's)
    extras = {}
    if not args.no_extras:
        del graph, api_graph
        graph = api_graph = None
        torch.cuda.empty_cache()
        for name, fn in (("encoder_sweep", lambda: encoder_sweep()),
                         ("long_context", lambda: long_context(world, rank, max(3, min(args.steps, 10)))),
                         ("head_sharded_1seq", lambda: head_sharded(world, rank, max(3, min(args.steps, 10)))),
                         ("tinyllama_generate", lambda: tinyllama_generate() if world == 1 else {"skipped": "1 GPU only"}),
                         ("prefill_attention", lambda: prefill_attention_sweep() if world == 1 else {"skipped": "1 GPU only"}),
                         ("path_a_scalar_vq_qkt", lambda: path_a_sweep() if world == 1 else {"skipped": "1 GPU only"})):
            try:
                extras[name] = fn()
            except Exception as e:   # noqa: BLE001 - reported in the line
                extras[name] = {"error": f"{type(e).__name__}: {e}"}
            torch.cuda.synchronize()

    # CPU baseline (rank 0, N=1): the oracle on one host core, bounded sample;
    # the same leg checks the timed step's outputs of a few units against it
    cpu, check = None, None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import hokv_oracle as O
        check = _check_against_oracle(store, q, out, sorted({0, Ls - 1}), [(0, 0), (B - 1, H - 1)], scale, top_k,
                                      sink, hot)
        reps, t_cpu = 0, 0.0
        Kh = store.k[0, 0, 0, :S].float().cpu().numpy()
        Vh = store.v[0, 0, 0, :S].float().cpu().numpy()
        kk = store.cb_k[0, 0, 0].cpu().numpy()
        cbh = store.codebook[0, 0, 0].cpu().numpy()
        cents = [cbh[s, :kk[s]] for s in range(M)]
        codes = store.codes[0, 0, 0, :S, :M].cpu().numpy()
        qh = q[0, 0, :Hq // H].float().cpu().numpy()
        from threadpoolctl import threadpool_limits
        with threadpool_limits(limits=1):   # one core: BLAS single-threaded
            t0 = time.perf_counter()
            while time.perf_counter() - t0 < args.cpu_seconds:
                O.cdc03_hot_attention(qh[reps % len(qh)], Kh, Vh, codes, cents, scale, top_k, sink, hot)
                reps += 1
            t_cpu = time.perf_counter() - t0
        hq_s = reps / t_cpu
        cpu = {"value": hq_s / (Ls * Hq), "unit": "tokens/s", "cores": 1, "kind": "port",
               "sample": f"{reps} head-queries (S=16384, D=128, M=16) in {t_cpu:.1f} s on one core, "
                         f"scaled by {Ls * Hq} head-queries per token"}

    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": warm, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8 codes + fp32 exact scoring (bf16 K/V)", "data": "synthetic",
        "config": config_for(w, world),
        "value_per_gpu": value / world,
        "spread": {"repeats": args.repeats, "steps_each": args.steps,
                   "ms_per_step_median": statistics.median(repeats) if repeats else None,
                   "ms_per_step_min": min(repeats) if repeats else None,
                   "ms_per_step_max": max(repeats) if repeats else None},
        "roofline": roof(dom), "roofline_other": roof(other),
        "step_hbm_gbs": step_bytes / (ms_step * 1e-3) / 1e9, "step_frac": step_bytes / (ms_step * 1e-3) / 1e9 / peak,
        "step_algorithmic_bytes": step_bytes,
        "cpu_baseline": cpu,
        "e2e": {"value": tokens / (e2e["graph"] / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "path": "CDC03Store.decode for every layer (captured in a CUDA graph), pinned H2D of the queries "
                        "and D2H of the outputs every step"
                        + ("; NCCL all-gather of the last layer's outputs of every rank every step" if world > 1
                           else "")},
        "e2e_eager": {"value": tokens / (e2e["eager"] / 1e3), "unit": "tokens/s",
                      "path": "the same calls without a graph (host launch cost included)"},
        "vq_assign": {"value": as_gbs, "unit": "GB/s", "frac": as_gbs / peak, "vectors": units * n_new,
                      "ms": as_ms, "kernel": "k_pq_assign_tc (tcgen05 tf32 screen into tensor memory, exact fp32 "
                                             "rescoring of the candidates)"},
        "gpu_launches": args.steps * Ls * 2,   # k6_candidates + k7_select_attend per layer
        "check": check,
        "clocks": clk.summary(),
        "setup_s": t_setup,
    }
    line.update(extras)
    if rank == 0:
        print(json.dumps(line), flush=True)
    graph = api_graph = None
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


K6_PHASES = ["rows+queries staged", "dots", "ranges exchanged", "quantisation step", "own image entries",
             "cluster image barrier",
             "image to smem", "score own chunks", "histograms complete (cluster barrier)", "threshold",
             "list+rescore"]
K7_PHASES = ["hot window", "wait for k6", "selection", "attend selected", "combine+store"]


def run_phase_stamps(args):
    """One decode step of the workload with the profiling build of the library:
    per-phase durations of the last layer's two kernels from %globaltimer stamps
    (thread 0 of every CTA), as a JSON line."""
    import torch

    from helix_online_kv import _lib as L
    from helix_online_kv.cdc03 import CDC03Store
    torch.cuda.set_device(0)
    L.require_device()
    w = dict(WORKLOAD)
    if args.layers:
        w["layers"] = args.layers
    B, Ls, H, Hq, D, S, M = (w["batch_per_gpu"], w["layers"], w["kv_heads"], w["q_heads"], w["head_dim"],
                             w["context"], w["pq_subspaces"])
    top_k, sink, hot = w["top_k"], w["sink_tokens"], w["hot_window"]
    scale = 1.0 / np.sqrt(D)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1234)
    store = CDC03Store(B, Ls, H, D, S, n_subspaces=M, dtype=torch.bfloat16)
    for layer in range(Ls):
        _fill_layer(store, layer, gen)
        store.calibrate(layer, w["pq_calibration_tokens"])
        store.assign(layer, 0, S)
    store.seq_len.fill_(S)
    q = torch.randn((Ls, B, Hq, D), generator=gen, device="cuda").to(torch.bfloat16)
    out = torch.empty_like(q)
    for _ in range(max(args.warmup, 3) + 1):
        for l in range(Ls):
            store.decode(l, q[l], scale, top_k, sink, hot, out=out[l])
    torch.cuda.synchronize()
    L.device_status()
    buf = np.zeros(3 * 4096 * 16, dtype=np.uint64)
    L.check(L.lib().hokv_phase_stamps(buf.ctypes.data_as(ctypes.c_void_p), buf.size), "phase_stamps")
    st = buf.reshape(3, 4096, 16).astype(np.int64)
    n6 = min(B * H * 8, 4096)
    n7 = B * Hq
    k6 = st[0, :n6, :len(K6_PHASES) + 1]
    k7 = st[1, :n7, :len(K7_PHASES) + 1]
    t0 = int(k6[:, 0].min())

    def table(x, names):
        rows = []
        for i, name in enumerate(names, start=1):
            d = (x[:, i] - x[:, i - 1]) / 1e3
            e = (x[:, i] - t0) / 1e3
            rows.append({"phase": name, "median_us": float(np.median(d)), "max_us": float(d.max()),
                         "ends_at_median_us": float(np.median(e)), "ends_at_max_us": float(e.max())})
        return rows

    def starts(x):
        us = np.sort((x[:, 0] - t0) / 1e3)
        return {"quantiles_us": [float(np.quantile(us, q)) for q in (0, 0.1, 0.25, 0.5, 0.75, 0.9, 1.0)],
                "histogram_1us": {int(b): int(c) for b, c in zip(*np.unique(np.floor(us).astype(int),
                                                                              return_counts=True))}}

    line = {"metric": "phase stamps (us) of the last layer's decode kernels", "config": config_for(w, 1),
            "starts": {"k6": starts(k6), "k7": starts(k7)},
            "k6_ctas": n6, "k6_start_spread_us": float((k6[:, 0].max() - t0) / 1e3), "k6": table(k6, K6_PHASES),
            "k7_ctas": n7, "k7_start_median_us": float(np.median((k7[:, 0] - t0) / 1e3)),
            "k7_start_max_us": float((k7[:, 0].max() - t0) / 1e3), "k7": table(k7, K7_PHASES),
            "layer_end_us": float((max(k6[:, -1].max(), k7[:, -1].max()) - t0) / 1e3)}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--ref-cap", type=int, default=512,
                    help="reference arm: most head-queries per host core in one step (bounds a step's time)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the encoder sweep and the long-context decode (extra keys of the line)")
    ap.add_argument("--repeats", type=int, default=10,
                    help="after the timed region, time the same K steps this many more times (spread)")
    ap.add_argument("--layers", type=int, default=0,
                    help="layers to run (default: the workload's 31); fewer only for profiler captures, "
                         "whose JSON line is then not the workload's")
    ap.add_argument("--phase-stamps", action="store_true",
                    help="run one step with the profiling build (libhokv_stamps.so) and print per-phase times")
    ap.add_argument("--path-a-sweep", action="store_true",
                    help="only the Path A sweep (fused Q.K^T over scalar-VQ codes), one JSON line")
    ap.add_argument("--prefill-sweep", action="store_true",
                    help="only the prefill-attention sweep (hokv_prefill_attention beside SDPA), one JSON line")
    args = ap.parse_args()
    if args.path_a_sweep:
        print(json.dumps({"path_a_scalar_vq_qkt": path_a_sweep()}))
        return 0
    if args.prefill_sweep:
        print(json.dumps({"prefill_attention": prefill_attention_sweep()}))
        return 0
    if args.phase_stamps:
        os.environ["HOKV_LIB_VARIANT"] = "stamps"   # read when the package loads the library
        return run_phase_stamps(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
