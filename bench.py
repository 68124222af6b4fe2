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


def _traffic_from_profiles(kernel: str):
    """Per-launch DRAM bytes of `kernel` from the committed ncu summary, if any."""
    path = os.path.join(REPO, "profiles", f"{kernel}_llama3_16k.md")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return float(line.split(":", 1)[1].strip().split()[0])
    except OSError:
        pass
    return None


# ----------------------------------------------------------------------------- reference arm (CPU)
def _ref_unit(seed: int, S: int, D: int, M: int, G: int):
    from oracle import hokv_oracle as O
    K, V = O.gen_kv(seed, 1, 1, S, D)
    K = O.to_fp16_values(K[0, 0])
    V = O.to_fp16_values(V[0, 0])
    cents, _ = O.pq_fit(K[:128], M=M, sub_clusters=256)
    codes = O.pq_assign(K, cents)
    Q = O.gen_queries(seed, 1, G, D)[0]
    return K, V, codes, cents, Q


def _ref_worker(args):
    seed, n_queries, S, D, M, G, top_k, sink, hot = args
    from oracle import hokv_oracle as O
    global _REF_CACHE
    try:
        _REF_CACHE
    except NameError:
        _REF_CACHE = {}
    if seed not in _REF_CACHE:
        _REF_CACHE[seed] = _ref_unit(seed, S, D, M, G)
    K, V, codes, cents, Q = _REF_CACHE[seed]
    scale = 1.0 / np.sqrt(D)
    t0 = time.perf_counter()
    for i in range(n_queries):
        O.cdc03_hot_attention(Q[i % G], K, V, codes, cents, scale, top_k, sink, hot)
    return n_queries, time.perf_counter() - t0


def cpu_rate(n_workers: int, per_worker: int, reps: int, S: int, D: int, M: int, G: int, w):
    """Head-queries/s of the oracle's CDC-03 (numpy) on n_workers processes."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    # one BLAS thread per worker process (the workers read these when they import numpy)
    for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[var] = "1"
    jobs = [(1000 + i, per_worker, S, D, M, G, w["top_k"], w["sink_tokens"], w["hot_window"])
            for i in range(n_workers)]
    with ctx.Pool(n_workers) as pool:
        pool.map(_ref_worker, [(j[0], 1) + j[2:] for j in jobs])  # build per-worker data, warm
        rates = []
        for _ in range(reps):
            t0 = time.perf_counter()
            res = pool.map(_ref_worker, jobs)
            dt = time.perf_counter() - t0
            rates.append(sum(r[0] for r in res) / dt)
    return rates


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    w = WORKLOAD
    cores = os.cpu_count() or 1
    per_step = 16
    rates = cpu_rate(cores, per_step, args.warmup + args.steps, w["context"], w["head_dim"], w["pq_subspaces"],
                     w["q_heads"] // w["kv_heads"], w)
    timed = rates[args.warmup:]
    hq_per_token = w["layers"] * w["q_heads"]
    tok_s = statistics.median(timed) / hq_per_token
    line = {
        "impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 / tok_s, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (numpy)", "data": "synthetic",
        "config": dict(w, note="CPU oracle restatement of the reference's numpy hybrid_pq_attention with a hot window"),
        "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{cores} processes x {per_step} head-queries per step at S=16384"},
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


def run_ours(args):
    import torch
    import torch.distributed as dist

    from helix_online_kv import _lib as L
    from helix_online_kv.cdc03 import CDC03Store
    from helix_online_kv.sharding import max_over_ranks

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

    # eager warm-up (sets kernel attributes), then capture one step in a graph
    step(L.stream())
    torch.cuda.synchronize()
    L.device_status()
    graph = torch.cuda.CUDAGraph()
    cap_stream = torch.cuda.Stream()
    cap_stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cap_stream):
        with torch.cuda.graph(graph, stream=cap_stream):
            step(L.stream())
    torch.cuda.current_stream().wait_stream(cap_stream)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(args.warmup, 3)):
        graph.replay()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        ev0.record()
        for _ in range(args.steps):
            graph.replay()
        ev1.record()
        torch.cuda.synchronize()
    ms = max_over_ranks(ev0.elapsed_time(ev1), device="cuda")
    barrier()
    ms_step = ms / args.steps
    tokens = B * world * args.steps
    value = tokens / (ms / 1e3)

    # per-kernel attribution: each stage alone, all layers in one graph, so the
    # average launch duration carries no host launch gaps (k7 re-reads the
    # candidate lists the step left, which is the same work)
    n_att = max(3, min(args.steps, 10))

    def stage_ms(fn, name):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(cap_stream):
            with torch.cuda.graph(g, stream=cap_stream):
                for r in refs:
                    L.check(fn(r, L.stream()), name)
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(n_att):
            g.replay()
        t1.record()
        torch.cuda.synchronize()
        del g
        return t0.elapsed_time(t1) / (n_att * Ls)

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
                "peak_kind": f"{peak_kind} (hbm_gbs, MEASURED_PEAKS.json)" if peak_kind == "measured" else peak_kind}

    step_bytes = (k6_bytes + k7_bytes) * Ls

    # end-to-end through the public API: host (pinned) queries in, host outputs out
    q_host = q.cpu().pin_memory()
    out_host = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    for _ in range(2):
        q.copy_(q_host, non_blocking=True)
        graph.replay()
        out_host.copy_(out, non_blocking=True)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        q.copy_(q_host, non_blocking=True)
        graph.replay()
        out_host.copy_(out, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), device="cuda")
    e2e_value = tokens / (e2e_ms / 1e3)

    # VQ-assign throughput: PQ codes for a fresh 32768-token block of every (b, h) of one layer
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

    # CPU baseline: the oracle on one host core, bounded sample (rank 0, N=1)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import hokv_oracle as O
        reps, n_q, t_cpu = 0, 0, 0.0
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
        "warmup": max(args.warmup, 3), "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8 codes + fp32 exact scoring (bf16 K/V)", "data": "synthetic",
        "config": dict(w, global_batch=B * world, parallelism=f"sequence-sharded x{world}",
                       l2="inputs larger than L2 (%.2f GB algorithmic per step)" % (step_bytes / 1e9)),
        "roofline": roof(dom), "roofline_other": roof(other),
        "step_hbm_gbs": step_bytes / (ms_step * 1e-3) / 1e9, "step_frac": step_bytes / (ms_step * 1e-3) / 1e9 / peak,
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": q.numel() * q.element_size(),
                "d2h_bytes_per_step": out.numel() * out.element_size()},
        "vq_assign": {"value": as_gbs, "unit": "GB/s", "frac": as_gbs / peak, "vectors": units * n_new,
                      "ms": as_ms, "kernel": "k_pq_assign_seq (fp32 CUDA cores, 4 vectors per thread in registers)"},
        "gpu_launches": args.steps * Ls * 2,   # k6_candidates + k7_select_attend per layer
        "clocks": clk.summary(),
        "setup_s": t_setup,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    del graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=0,
                    help="layers to run (default: the workload's 31); fewer only for profiler captures, "
                         "whose JSON line is then not the workload's")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
