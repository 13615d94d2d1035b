#!/usr/bin/env python
"""Prefill throughput of the clef-rs B200 backend.

Workload (config 4, the default): the full random-init 32-layer hybrid backbone
([3 x DeltaNet + 1 x attention] x 8, hidden 2560, intermediate 9216, 16/32
DeltaNet heads of 128, 16/4 attention heads of 256) plus the linear schema head
read at each request's last token; one batch of 256 synthetic requests with
lengths U[256, 2048] and ids U[0, 248320) (seed 3), BF16 projections with F32
accumulation and an F32 residual stream and head. A step is one prefill of the
whole batch. Requests are independent and weights are replicated, so with N
GPUs the batch is divided over the ranks by the longest-processing-time rule
(strong scaling, no collective on the data path); the max over ranks of the
device time is reported, with each rank's token count and device time.
`--weak` gives every rank a batch of its own instead (seed 3 + 1000 * rank).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

`value` is measured with device-resident ids and logits (CUDA events on the
launching stream); `e2e` runs the public host API (clef_engine_prefill) from
pinned host ids to host logits. `--impl reference` times the CPU F32
restatement of the reference path (oracle/) on the host cores instead.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "clef-rs_b200"))

METRIC = "prefill tok/s"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="config4", choices=["config4", "config5", "flash"],
                    help="config4: one batch of 256 requests U[256,2048] divided over the GPUs; config5: one 16384-token "
                         "prefix computed once (rank 0) and broadcast, 64 suffixes U[512,4096] "
                         "sharded over GPUs")
    ap.add_argument("--weak", action="store_true",
                    help="config4 with a batch of --requests per rank (weak scaling) instead of "
                         "one batch divided over the ranks (strong scaling, the default)")
    ap.add_argument("--requests", type=int, default=256)
    ap.add_argument("--precision", default="bf16", choices=["bf16", "split"],
                    help="bf16: BF16 GEMM operands (default); split: split-BF16 activation operands and "
                         "F32 projection outputs (F32-class projections, twice the tensor work)")
    ap.add_argument("--flash-tokens", type=int, default=4096, choices=[256, 1024, 4096],
                    help="request length of the flash workload (the reference's published lengths)")
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-tokens", type=int, default=256)
    ap.add_argument("--profile-op", default=None,
                    choices=["gemm", "gemm_swiglu", "gemm_split", "scan", "scan1", "packed", "attention",
                             "attention_tc", "attention_prefix", "prologue", "head"],
                    help="run one operator on a profiling-sized case and exit (for ncu)")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--scan-seqs", type=int, default=64,
                    help="--profile-op scan: number of 1024-token sequences (ncu captures use 16)")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


# Published reference number for the `flash` workload: Metal mixed F16 prefill
# of one 4096-token request at the Flash geometry on an Apple M5 Pro, 1101 tok/s
# (docs/benchmarks/flash-metal-prefill/report.md:41-43 of the reference).
FLASH_REFERENCE_TOK_S = {4096: 1101.0, 1024: 1248.0, 256: 1151.0}


def workload_config(args, n_gpus):
    if args.workload == "flash":
        return {"precision": args.precision, "workload": f"flash geometry: 32-layer hybrid backbone (hidden 4096, intermediate 12288) "
                            f"+ linear schema head, one {args.flash_tokens}-token request per GPU per step",
                "vocab": 248320, "layers": args.layers, "hidden": 4096, "intermediate": 12288,
                "parallelism": f"dp{n_gpus} (one request per rank, weights replicated)",
                "baseline": "reference Metal mixed F16 on Apple M5 Pro (different hardware)",
                "l2": "not flushed: every step streams ~17 GB of weights, far above the 126 MB L2"}
    if args.workload == "config5":
        return {"precision": args.precision, "workload": "config5: 32-layer hybrid backbone + linear schema head, prefix reuse",
                "prefix_tokens": 16384, "suffixes_total": 64, "suffix_len": "U[512,4096]",
                "vocab": 248320, "layers": args.layers, "hidden": 2560, "intermediate": 9216,
                "parallelism": (f"dp{n_gpus} (suffixes LPT-sharded; prefix computed once on rank 0 and "
                                "broadcast to the other ranks by one NCCL broadcast of its device state)"),
                "l2": "not flushed: every step streams 8.4 GB of weights, far above the 126 MB L2"}
    batch = ({"requests_per_gpu": args.requests} if args.weak
             else {"requests": args.requests, "requests_per_gpu": round(args.requests / n_gpus, 2)})
    return {"workload": "config4: 32-layer hybrid backbone + linear schema head",
            "precision": args.precision, **batch, "prompt_len": "U[256,2048]", "vocab": 248320,
            "layers": args.layers, "hidden": 2560, "intermediate": 9216,
            "deltanet_heads": "16qk/32v x 128", "attention_heads": "16q/4kv x 256",
            "chunk": 64,
            "parallelism": f"dp{n_gpus} (" + ("one batch per rank" if args.weak
                                             else "one batch LPT-sharded over ranks") + ", weights replicated)",
            "l2": "not flushed: every step streams 8.4 GB of weights and tens of GB of "
                  "activations, far above the 126 MB L2"}


# ---------------------------------------------------------------------------
# CPU F32 path (oracle/): the reference's algorithm on the host cores.
# ---------------------------------------------------------------------------
def host_weights(cfg, seed=3, std=0.02, threads=8):
    """Seeded synthetic weights of the benchmark geometry, drawn on the host
    (same distributions as the engine's device init, not the same values)."""
    from concurrent.futures import ThreadPoolExecutor

    from clef_b200.config import weight_shapes
    shapes = weight_shapes(cfg)
    names = sorted(shapes)

    def make(i_name):
        i, name = i_name
        rng = np.random.default_rng([seed, i])
        shape = shapes[name]
        if name.endswith("A_log"):
            return name, rng.uniform(0, np.log(16), shape).astype(np.float32)
        if name.endswith("dt_bias"):
            return name, (0.1 * rng.standard_normal(shape, dtype=np.float32))
        w = std * rng.standard_normal(shape, dtype=np.float32)
        if name.endswith("linear_attn.norm.weight"):
            w += 1
        return name, w

    with ThreadPoolExecutor(threads) as ex:
        yield from ex.map(make, enumerate(names))


def build_cpu_model(cfg):
    import oracle
    m = oracle.Model(cfg)
    for name, w in host_weights(cfg):
        m.set_weight(name, w)
    m.check()
    return m


def cpu_sample_ids(args):
    from clef_b200 import workloads
    req = workloads.backbone_requests(n=args.requests, seed=3)[0]
    return req[: args.cpu_sample_tokens]


def time_cpu(model, ids, reps):
    t0 = time.perf_counter()
    for _ in range(reps):
        model.prefill(ids)
    return (time.perf_counter() - t0) / reps


def cpu_baseline(args, cfg):
    import oracle
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    model = build_cpu_model(cfg)
    ids = cpu_sample_ids(args)
    time_cpu(model, ids, 1)
    sec = time_cpu(model, ids, 2)
    return {"value": round(len(ids) / sec, 3), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"one {len(ids)}-token request of the config-4 batch through the full "
                      f"{cfg.num_hidden_layers}-layer F32 CPU path (oracle/oracle.cpp, OpenMP "
                      f"{threads} threads, host-drawn weights of the same distributions), mean of 2 runs"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from clef_b200.config import benchmark_config
    cfg = benchmark_config(args.layers, 7)
    import oracle
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    model = build_cpu_model(cfg)
    ids = cpu_sample_ids(args)
    for _ in range(args.warmup):
        model.prefill(ids)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        hidden, _ = model.prefill(ids)
        times.append(time.perf_counter() - t0)
    ms = 1000 * statistics.mean(times)
    tok_s = len(ids) / (ms / 1000)
    sample = (f"one {len(ids)}-token request of the config-4 batch per step through the full "
              f"{cfg.num_hidden_layers}-layer F32 CPU path (oracle/oracle.cpp: C++ restatement of the "
              f"reference's Candle CPU path; the Rust reference cannot be built here), "
              f"{threads} threads")
    line = {"metric": METRIC, "value": round(tok_s, 3), "unit": "tok/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True,
            "scaling": "weak" if (args.weak or args.workload == "flash") else "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "decisions_per_s": round(1000.0 / ms, 5),
            "config": workload_config(args, args.gpus),
            "cpu_baseline": {"value": round(tok_s, 3), "unit": "tok/s", "cores": threads,
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(tok_s, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "finite": bool(np.isfinite(hidden).all()),
            "native_libraries": mapped_repo_libraries()}
    print(json.dumps(line), flush=True)
    return 0


def mapped_repo_libraries():
    """Shared objects of this repository mapped into this process (Linux
    /proc/self/maps): the reference arm must map the oracle only, never the
    product library."""
    try:
        maps = Path("/proc/self/maps").read_text().splitlines()
    except OSError:
        return None
    root = str(ROOT)
    return sorted({line.split()[-1][len(root) + 1:] for line in maps
                   if line.split()[-1].startswith(root) and line.endswith(".so")})


# ---------------------------------------------------------------------------
# Clock sampling during the timed region.
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid):
        self.uuid = uuid
        self.proc = None
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", self.uuid], stdout=self.out, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.flush()
        rows = [r.split(",") for r in Path(self.out.name).read_text().splitlines() if r.strip()]
        os.unlink(self.out.name)
        sm, mx, reasons, watts, capped = [], None, set(), [], 0
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [x.strip() for x in r]
            try:
                sm.append(float(r[0]))
                mx = float(r[1])
            except (ValueError, IndexError):
                continue
            try:
                watts.append(float(r[2]))
            except (ValueError, IndexError):
                pass
            for n, v in zip(names, r[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
            if len(r) > 7 and r[7].lower() == "active":
                capped += 1
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "sm_mhz_range": [min(sm), max(sm)],
                "power_w": statistics.median(watts) if watts else None,
                "power_cap_frac": round(capped / len(sm), 3)}


# ---------------------------------------------------------------------------
# Our arm.
# ---------------------------------------------------------------------------
def _head_shapes(cfg):
    """(name, shape) of every joint-head tensor (head.rs:91-145)."""
    h, w, f = cfg["hidden_size"], cfg["width"], cfg["feedforward"]
    out = []

    def lin(n, o, i, bias):
        out.append((f"{n}.weight", (o, i)))
        if bias:
            out.append((f"{n}.bias", (o,)))

    def norm(n, k):
        out.extend([(f"{n}.weight", (k,)), (f"{n}.bias", (k,))])

    def attn(n):
        out.extend([(f"{n}.in_proj_weight", (3 * w, w)), (f"{n}.in_proj_bias", (3 * w,))])
        lin(f"{n}.out_proj", w, w, True)

    for r in range(cfg["routing_layers"]):
        p = f"evidence_layers.{r}"
        norm(f"{p}.query_norm", w)
        norm(f"{p}.memory_norm", w)
        attn(f"{p}.attention")
        norm(f"{p}.feedforward_norm", w)
        lin(f"{p}.feedforward.0", f, w, True)
        lin(f"{p}.feedforward.3", w, f, True)
    for li in range(cfg["layers"]):
        p = f"layers.{li}"
        for n in ("norm1", "norm2", "norm3"):
            norm(f"{p}.{n}", w)
        attn(f"{p}.self_attn")
        attn(f"{p}.multihead_attn")
        lin(f"{p}.linear1", f, w, True)
        lin(f"{p}.linear2", w, f, True)
    norm("hidden_norm", h)
    for n in ("memory_projection", "question_projection", "option_question_projection", "global_projection",
              "option_context_projection", "option_lexical_projection"):
        lin(n, w, h, False)
    out.append(("type_embedding.weight", (3, w)))
    for n in ("option_summary_norm", "field_norm", "option_norm"):
        norm(n, w)
    lin("residual_scorer.0", w, 4 * w, True)
    lin("residual_scorer.3", 1, w, True)
    out += [("prior_logit_scale", ()), ("joint_logit_scale", ()), ("residual_gate", ())]
    return out


def profile_op(args):
    """One operator on a case larger than L2 but a few GB at most: the inputs
    ncu captures (profiles/*.md give the command lines)."""
    import torch

    import clef_b200 as cb
    from clef_b200 import workloads
    torch.manual_seed(0)
    dev = "cuda"

    def timed(label, fn):
        # CUDA events on the launching (current) stream around each repetition.
        for _ in range(args.reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            print(f"{label}: {e0.elapsed_time(e1):.3f} ms", flush=True)

    if args.profile_op == "gemm_split":
        # Split-BF16 activation operand (hi | lo) against BF16 weights.
        M, K, N = 8192, 2560, 9216
        x2 = cb.split_bf16(torch.randn(M, K, device=dev))
        w = (0.02 * torch.randn(N, K, device=dev)).bfloat16()
        out = torch.empty(M, N, device=dev)
        timed(f"gemm_split {M}x{N}x{K} (tensor work 2x)", lambda: cb.gemm_split(x2, w, epilogue=cb.EPI_F32, out=out))
    elif args.profile_op == "packed":
        # DeltaKernel's largest accepted case: T = 4096, H = 32, dk = dv = 128.
        T, H, dk, dv = 4096, 32, 128, 128
        qk = torch.nn.functional.normalize(torch.randn(T, H, 2, dk, device=dev), dim=-1)
        packed = torch.cat([qk[:, :, 0] / dk ** 0.5, qk[:, :, 1], torch.randn(T, H, dv, device=dev),
                            torch.rand(T, H, 1, device=dev), torch.sigmoid(torch.randn(T, H, 1, device=dev))],
                           -1).contiguous()
        timed(f"delta_packed T={T} H={H}", lambda: cb.delta_packed(packed, dk, dv))
    elif args.profile_op in ("gemm", "gemm_swiglu"):
        M, K, N = 8192, 2560, 9216
        x = torch.randn(M, K, device=dev).bfloat16()
        w = (0.02 * torch.randn(N, K, device=dev)).bfloat16()
        w2 = (0.02 * torch.randn(N, K, device=dev)).bfloat16()
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        if args.profile_op == "gemm":
            timed(f"gemm {M}x{N}x{K}", lambda: cb.gemm(x, w, out=out))
        else:
            timed(f"gemm_swiglu {M}x{N}x{K}", lambda: cb.gemm_swiglu(x, w, w2, out=out))
    elif args.profile_op in ("scan", "scan1"):
        n = args.scan_seqs
        T, cu = (1024 * n, np.arange(0, 1024 * n + 1, 1024, dtype=np.int64)) if args.profile_op == "scan" \
            else (1024, None)
        inp = workloads.delta_operator_inputs(T=T, seed=1)
        qs, ks = workloads.scan_operands(inp)
        t = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda()
             for k, v in dict(q=qs, k=ks, v=inp["v"], g=inp["g"], b=inp["beta"]).items()}
        timed(f"delta_scan T={T}", lambda: cb.delta_scan(t["q"], t["k"], t["v"], t["g"], t["b"], cu_seqlens=cu))
    elif args.profile_op == "attention":
        T = 4096
        q = torch.randn(16, T, 256, device=dev).bfloat16()
        k = torch.randn(4, T, 256, device=dev).bfloat16()
        v = torch.randn(4, T, 256, device=dev).bfloat16()
        for _ in range(args.reps):
            cb.attention_gqa(q, k, v)
    elif args.profile_op in ("attention_tc", "attention_prefix"):
        # Token-major q/k and transposed V as the engine keeps them; the C ABI
        # is called directly so only the attention kernel runs per repetition.
        # attention_prefix: 2048 queries after a 16384-token shared prefix (the
        # shape of a config-5 suffix).
        T, P, H, Hkv = (4096, 0, 16, 4) if args.profile_op == "attention_tc" else (2048, 16384, 16, 4)
        Tk = T + P
        q = torch.randn(T, H, 256, device=dev).bfloat16()
        k = torch.randn(Tk, Hkv, 256, device=dev).bfloat16()
        vt = torch.randn(Hkv * 256, Tk, device=dev).bfloat16()
        o = torch.empty(T, H, 256, device=dev)
        st = torch.cuda.current_stream()
        ptr = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        flops = 2 * 2 * H * 256 * (T * P + T * (T + 1) // 2)
        for i in range(args.reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            rc = cb.lib.clef_attention_gqa_vt(ptr(q), ptr(k), ptr(vt), H, Hkv, T, Tk, 256, Tk, ptr(o),
                                              ctypes.c_void_p(st.cuda_stream))
            e1.record()
            assert rc == 0, cb.lib.clef_last_error().decode()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            print(f"{args.profile_op} T={T} prefix={P}: {ms:.3f} ms, {flops / ms / 1e9:.1f} TFLOP/s", flush=True)
    elif args.profile_op == "prologue":
        T, Hk, Hv = 16384, 16, 32
        width = 2 * Hk * 128 + Hv * 128
        ldp = width + Hv * 128 + 2 * Hv
        proj = torch.randn(T, ldp, device=dev)
        conv = 0.3 * torch.randn(width, 4, device=dev)
        dt, alog = 0.1 * torch.randn(Hv, device=dev), torch.rand(Hv, device=dev) * 2.7
        timed(f"delta_prologue T={T}",
              lambda: cb.delta_prologue(proj, width + Hv * 128, width + Hv * 128 + Hv, conv, dt, alog, Hk, Hv))
    elif args.profile_op == "head":
        # The learned joint schema head at the released geometry on one record
        # of T = 2048 tokens with 4 questions x 4 options (seeded weights).
        cfg = dict(hidden_size=2560, width=1024, routing_layers=2, layers=4, heads=16, feedforward=4096)
        head = cb.Head(cfg)
        rng = np.random.default_rng(5)

        def mat(o, i):
            return (rng.standard_normal((o, i)) / np.sqrt(i)).astype(np.float32)

        for name, shape in _head_shapes(cfg):
            n = int(np.prod(shape)) if shape else 1
            if len(shape) == 2:
                head.set_weight(name, mat(*shape))
            elif name.endswith(".weight") and "norm" in name:
                head.set_weight(name, np.ones(n, np.float32))
            else:
                head.set_weight(name, (0.02 * rng.standard_normal(n)).astype(np.float32))
        head.finalize()
        T, vocab = 2048, 4096
        hidden = torch.randn(T, 2560, device=dev)
        emb = 0.05 * torch.randn(vocab, 2560, device=dev)
        ids = rng.integers(0, vocab, T).astype(np.int32)
        qs = [(q % 3, (100 * q, 100 * q + 20), [(100 * q + 20 + 10 * o, 100 * q + 30 + 10 * o) for o in range(4)])
              for q in range(4)]
        for _ in range(args.reps):
            t0 = time.perf_counter()
            head.forward(hidden, emb, ids, qs)
            print(f"head T={T} 4x4 options: {1e3 * (time.perf_counter() - t0):.3f} ms (host clock, "
                  f"includes the metadata upload and the final synchronisation)", flush=True)
    torch.cuda.synchronize()
    print(f"profile-op {args.profile_op}: ok", flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.profile_op:
        return profile_op(args)
    import torch
    import torch.distributed as dist

    import clef_b200 as cb
    from clef_b200 import workloads
    from clef_b200.config import benchmark_config, flops_per_request, linear_flops_per_token

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600),
                                device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    def allmax(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def allsum(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    def allgather(values):
        t = torch.tensor(values, dtype=torch.float64, device="cuda")
        if world == 1:
            return [t.tolist()]
        every = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(every, t)
        return [e.tolist() for e in every]

    from clef_b200.config import flash_config
    cfg = flash_config(args.layers, 7) if args.workload == "flash" else benchmark_config(args.layers, 7)
    eng = cb.Engine(cfg, local)
    eng.init_random(3, 0.02)
    eng.finalize()
    split = args.precision == "split"
    eng.set_precision(cb.PRECISION_SPLIT if split else cb.PRECISION_BF16)
    from clef_b200.sharding import rank_shard
    prefix = None
    prefix_ms = None
    bcast_ms = None
    if args.workload == "config5":
        pre_ids, suffixes = workloads.prefix_workload()
        reqs = rank_shard(suffixes, rank, world, lambda r: flops_per_request(cfg, len(r), 16384))
        # The prefix state is computed once, on rank 0; the other ranks (same
        # seeded weights) receive its device allocation by one NCCL broadcast.
        from clef_b200.sharding import share_prefix
        prefix, prefix_ms, bcast_ms = share_prefix(
            lambda: eng.prefill([pre_ids], capture=len(pre_ids), logits=False)[2],
            lambda: eng.create_prefix(len(pre_ids)), rank, world, "cuda", torch.cuda.synchronize)
    elif args.workload == "flash":
        rng = np.random.default_rng(4096 + rank)
        reqs = [rng.integers(0, cfg.vocab_size, args.flash_tokens).astype(np.int32)]
    elif args.weak:
        reqs = workloads.backbone_requests(n=args.requests, seed=3 + 1000 * rank)
    else:
        batch = workloads.backbone_requests(n=args.requests, seed=3)
        reqs = rank_shard(batch, rank, world, lambda r: flops_per_request(cfg, len(r)))
    lens = np.array([len(r) for r in reqs], np.int64)
    offsets = np.zeros(len(reqs) + 1, np.int64)
    offsets[1:] = np.cumsum(lens)
    ids = np.concatenate(reqs).astype(np.int32)
    tokens = int(offsets[-1])
    ids_dev = torch.from_numpy(ids).cuda()
    logits_dev = torch.empty((len(reqs), 7), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()

    for _ in range(args.warmup):
        eng.prefill_device(ids_dev, offsets, logits_dev, initial=prefix, stream=stream)
    torch.cuda.synchronize()

    # ---- device-resident timed region ---------------------------------------
    uuid = str(torch.cuda.get_device_properties(local).uuid)
    sampler = ClockSampler(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
    eng.set_profiling(True)
    l0 = eng.launches()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler.start()
    barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(args.steps):
        eng.prefill_device(ids_dev, offsets, logits_dev, initial=prefix, stream=stream)
    end.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ms = start.elapsed_time(end) / args.steps
    launches = eng.launches() - l0
    stages = eng.stage_times()
    eng.set_profiling(False)
    logits = logits_dev.cpu().numpy()
    ms_max = allmax(ms)
    per_rank = [{"rank": r, "tokens": int(v[0]), "requests": int(v[1]), "device_ms": round(v[2], 3),
                 "gemm_ms": round(v[3], 3)}
                for r, v in enumerate(allgather([tokens, len(reqs), ms, stages["gemm"] / args.steps]))]

    # ---- end to end through the public host API ------------------------------
    ids_pin = torch.from_numpy(ids).pin_memory()
    lg_pin = torch.empty((len(reqs), 7), dtype=torch.float32).pin_memory()
    ids_np, lg_np = ids_pin.numpy(), lg_pin.numpy()
    eng.prefill_packed(ids_np, offsets, initial=prefix, logits_out=lg_np)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        eng.prefill_packed(ids_np, offsets, initial=prefix, logits_out=lg_np)
    e2e_s = (time.perf_counter() - t0) / args.steps
    barrier()
    e2e_max = allmax(e2e_s)
    assert np.array_equal(lg_np, logits), "host and device-resident prefill disagree"
    decisions = cb.decide(lg_np)

    total_tokens = allsum(tokens)
    total_reqs = allsum(len(reqs))
    value = total_tokens / (ms_max / 1000.0)

    # ---- roofline of the dominant kernel (the projection GEMMs) --------------
    pk, pk_kind = peaks()
    # Tensor-core work of the projections: twice the model's FLOPs when every
    # activation operand is a split (hi + lo) pair.
    lin_flops = tokens * linear_flops_per_token(cfg) * (2 if split else 1)
    gemm_ms = stages["gemm"] / args.steps
    achieved = lin_flops / (gemm_ms / 1000.0) / 1e12
    peak = float(pk.get("bf16_tflops_sustained", pk.get("bf16_tflops")))
    traffic = None
    tf = ROOT / "profiles" / "gemm_traffic.txt"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get("bytes_per_launch")
    roofline = {"bound": "tensor", "kernel": "gemm_pair_kernel (tcgen05 cta_group::2 projection GEMMs, all launches)"
                + (" with split-BF16 operands (tensor FLOPs = 2x model FLOPs)" if split else ""),
                "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4), "peak_source": f"{pk_kind} bf16_tflops_sustained",
                "traffic": traffic,
                "stage_ms_per_step": {k: round(v / args.steps, 3) for k, v in stages.items()}}
    # Memory-bound stages against the measured HBM copy bandwidth: algorithmic
    # bytes per token (the tensors each stage must read and write once) x tokens
    # x layers that run the stage, over its live CUDA-event time.
    hbm_peak = float(pk.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    n_delta = sum(1 for i in range(cfg.num_hidden_layers) if not cfg.is_attention(i))
    w_key, w_val = cfg.linear_num_key_heads * 128, cfg.linear_num_value_heads * 128
    w_gate, w_hid = cfg.linear_num_value_heads, cfg.hidden_size
    proj_b = 4 if split else 2  # projection output bytes
    op_b = 4 if split else 2    # GEMM operand bytes per element (split pair: hi + lo)
    per_token = {
        # conv rows in (q|k|v, a, b), q k v g beta out (F32)
        "delta_prologue": (n_delta, (2 * w_key + w_val + 2 * w_gate) * (proj_b + 4)),
        # q k v g beta in, o out (F32)
        "delta_scan": (n_delta, (2 * w_key + w_val + 2 * w_gate) * 4 + w_val * 4),
        # o (F32) and z in, y out (the out-projection's operand)
        "delta_epilogue": (n_delta, w_val * (4 + proj_b + op_b)),
        # h (F32) in, normed operand out; two norms per layer
        "norm": (2 * cfg.num_hidden_layers, w_hid * (4 + op_b)),
    }
    hbm_stages = {}
    for name, (n_layers, nbytes) in per_token.items():
        ms_stage = stages.get(name, 0.0) / args.steps
        if ms_stage > 0:
            gbs = tokens * n_layers * nbytes / (ms_stage / 1000.0) / 1e9
            hbm_stages[name] = {"bytes_per_token_layer": nbytes, "ms_per_step": round(ms_stage, 3),
                                "gbs": round(gbs, 1), "frac": round(gbs / hbm_peak, 3)}
    roofline["hbm_stages"] = hbm_stages
    roofline["hbm_peak_gbs"] = hbm_peak
    pre_len = 16384 if prefix is not None else 0
    total_flops = sum(flops_per_request(cfg, int(L), pre_len) for L in lens)
    line = {"metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 3),
            "higher_is_better": True,
            "scaling": "weak" if (args.weak or args.workload == "flash") else "strong",
            "vs_baseline": (round(value / FLASH_REFERENCE_TOK_S[args.flash_tokens], 1)
                            if args.workload == "flash" else None),
            "dtype": "bf16",
            "data": "synthetic (seeded ids and random-init weights)",
            "decisions_per_s": round(total_reqs / (ms_max / 1000.0), 2),
            "model_tflops": round(allsum(total_flops) / (ms_max / 1000.0) / 1e12, 1),
            "config": workload_config(args, world),
            "roofline": roofline,
            "e2e": {"value": round(total_tokens / e2e_max, 1), "unit": "tok/s",
                    "decisions_per_s": round(total_reqs / e2e_max, 2),
                    "h2d_bytes_per_step": int(ids.nbytes + offsets.nbytes),
                    "d2h_bytes_per_step": int(lg_np.nbytes)},
            "gpu_launches": int(launches),
            "ranks": per_rank,
            "prefix_ms_once": None if prefix_ms is None else round(allmax(prefix_ms), 1),
            "prefix_broadcast_ms": None if bcast_ms is None else round(allmax(bcast_ms), 2),
            "clocks": clocks,
            "decisions_finite": bool(all(np.isfinite([d.noul, d.confidence, d.score]).all()
                                         for d in decisions))}
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload == "config4":
        line["cpu_baseline"] = cpu_baseline(args, cfg)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if prefix is not None:
        prefix.close()
    eng.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
