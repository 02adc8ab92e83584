#!/usr/bin/env python3
"""Batch-1 greedy decode throughput of the B200 engine (one JSON line).

Workload (per GPU): the seeded Qwen2.5-0.5B-shape per-row int8 model, a
128-token uniform-random prompt prefilled untimed, then K timed greedy decode
steps (a "step" = one token through the whole model, LM head and argmax),
FP32 KV cache, as the reference's `bench` command runs it
(src/main.cpp:128-179 of mottopanikeiku/cpu-decode): one warm-up pass, then
rewind to the context and time.

* value: tokens/s with the model resident in HBM; steps chained on the device
  (the argmax of step t is the token of step t+1, no host round trip), timed
  with CUDA events on the launching stream.
* e2e: the same greedy loop through the C ABI call a user makes (dcb_step)
  with host buffers: the token goes in as a launch argument, the full logits
  vector (vocab floats) and the argmax come back to host memory every step.
* roofline: the step kernel's algorithmic bytes per token (the reference's own
  byte model) over its average launch time, against the measured HBM peak.
* cpu_baseline: the reference's own CPU engine (built from its sources into
  oracle/_ref) timed on this host's cores on a bounded sample.
* batched: 64 independent sequences per GPU (contexts 512-8192, KV pre-filled
  with seeded N(0,1) rows, 128 greedy steps), every projection one tensor-core
  GEMM over all of them; its own tokens/s, e2e and step roofline.

Several GPUs (torchrun) run independent replicas, one sequence each (and 64
each in the batched measurement), with no collective on the data path (weak
scaling); the job time is the max over ranks.
`--impl reference` times the reference CPU engine instead (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
CONTEXT = 128
SEED = 0
MODEL_CACHE = Path(os.environ.get("DCB_MODEL_CACHE", str(Path(tempfile.gettempdir()) / "dcb_models")))
METRIC = "batch-1 decode tokens/s at ctx 128/4096; achieved HBM GB/s vs B200 peak"


def load_package():
    import importlib.util
    if "cpu_decode_b200" in sys.modules:
        return sys.modules["cpu_decode_b200"]
    pkg = ROOT / "cpu-decode_b200"
    spec = importlib.util.spec_from_file_location("cpu_decode_b200", pkg / "__init__.py",
                                                  submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["cpu_decode_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def model_bytes_per_token(d, pos: int, kv_bytes: int = 4) -> int:
    """Algorithmic bytes of one token at cache position `pos` (the reference's
    byte model, src/kernels.cpp:184-185 and src/model.cpp:311-316): all weights
    and scales once, norms/biases, the embedding row, the new K/V row and the
    K/V rows 0..pos once."""
    H, I, L, V, kvd = d.hidden, d.intermediate, d.layers, d.vocab, d.kv_dim
    weights = L * (H * H + 2 * kvd * H + H * H + 2 * I * H + H * I) + V * H
    scales = 4 * (L * (H + 2 * kvd + H + 2 * I + H) + V)
    norms = 4 * (L * (3 * H + 2 * kvd) + H)
    embed = H + 4
    kv = L * 2 * kvd * kv_bytes * (1 + (pos + 1))
    return weights + scales + norms + embed + kv


def measured_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic(name: str, key: str = "dram_bytes_per_launch"):
    """DRAM bytes per launch (or per step) from the committed ncu summary, if present."""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    m = re.search(key + r":\s*([0-9.eE+]+)", p.read_text())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clocks sampled while the GPU is busy."""

    def __init__(self, index: int):
        self.path = Path(tempfile.mkstemp(suffix=".csv")[1])
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = [r.split(", ") for r in self.path.read_text().splitlines() if r.strip()]
        self.path.unlink(missing_ok=True)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if v.strip() == "Active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def host_cpu() -> dict:
    """The host's CPU model and logical core count (as tools/measure.py:61-70 records)."""
    name = ""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                name = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"model": name, "logical_cpus": os.cpu_count(), "usable_cpus": len(os.sched_getaffinity(0))}


def reference_bench(model_dir: Path, steps: int, repeats: int, threads: int) -> dict:
    """`cpu-decode bench` of the reference, built from its sources (oracle/_ref),
    as the reference's own measurement tool runs it (tools/measure.py:80-84):
    ctx 128, `steps` greedy steps, `repeats` repeats, the median tokens/s."""
    exe = ROOT / "oracle" / "_ref" / "cpu-decode"
    kernel = "simd512x4" if "avx512bw" in Path("/proc/cpuinfo").read_text() else "simd256"
    tokens = ",".join(str(t) for t in prompt_tokens())
    out = subprocess.run([str(exe), "bench", "--model", str(model_dir), "--tokens", tokens, "--context", str(CONTEXT),
                          "--steps", str(steps), "--repeats", str(repeats), "--threads", str(threads), "--kernel",
                          kernel], capture_output=True, text=True, check=True)
    res = json.loads(out.stdout)
    rates = [sample["tokens_per_second"] for sample in res["samples"]]
    return {"tokens_per_s": round(statistics.median(rates), 3), "repeats": len(rates), "kernel": kernel,
            "threads": threads}


def cpu_baseline(model_dir: Path, steps: int = 16) -> dict:
    """The reference CPU engine on this host's cores, on a bounded sample: all
    usable threads, and one thread, 3 repeats each (median)."""
    exe = ROOT / "oracle" / "_ref" / "cpu-decode"
    threads = len(os.sched_getaffinity(0))
    if exe.exists():
        full = reference_bench(model_dir, steps, 3, threads)
        one = reference_bench(model_dir, steps, 3, 1)
        return {"value": full["tokens_per_s"], "unit": "tokens/s", "cores": threads, "kind": "reference",
                "value_1_thread": one["tokens_per_s"], "host_cpu": host_cpu(),
                "sample": f"reference cpu-decode bench --kernel {full['kernel']}: ctx {CONTEXT}, {steps} greedy "
                          f"steps, median of 3 repeats, at {threads} threads and at 1 thread"}
    sys.path.insert(0, str(ROOT))
    import oracle
    orc = oracle.Oracle(model_dir, CONTEXT + steps + 1, threads=threads)
    prompt = prompt_tokens()
    for i, t in enumerate(prompt):
        logits = orc.step(t, i + 1 == len(prompt))
    nxt = oracle.argmax(logits)
    t0 = time.perf_counter()
    for _ in range(steps):
        nxt = oracle.argmax(orc.step(nxt))
    dt = time.perf_counter() - t0
    return {"value": round(steps / dt, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
            "host_cpu": host_cpu(),
            "sample": f"C restatement of the reference step: ctx {CONTEXT}, {steps} greedy steps"}


def headline_config(world: int) -> dict:
    """The workload of the headline line, identical in both arms."""
    return {"workload": "qwen2.5-0.5b-shape int8 (24x896, 14/2 heads, FFN 4864, vocab 151936), "
                        "batch 1, 128-token prompt + greedy decode, FP32 KV",
            "context": CONTEXT, "global_batch": world, "parallelism": f"replicas{world}",
            "l2": "inputs larger than L2 (496 MB of weights per step)"}


def prompt_tokens() -> list[int]:
    dcb = load_package()
    import cpu_decode_b200.synthetic as syn
    return syn.random_tokens(CONTEXT, syn.QWEN05.vocab, seed=SEED + 11)


def ensure_model() -> Path:
    load_package()
    import cpu_decode_b200.synthetic as syn
    return syn.ensure_random_model(MODEL_CACHE / f"qwen05_seed{SEED}", syn.QWEN05, seed=SEED)


def run_reference(args) -> None:
    """The reference's CPU engine (its `cpu-decode bench`, built from its
    sources) on this host's cores: the same steps, config, metric and unit as
    the B200 arm; median of 3 repeats at all usable threads, with the
    1-thread figure beside it. Rank 0 alone runs it."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    model = ensure_model()
    steps = max(1, args.steps)
    exe = ROOT / "oracle" / "_ref" / "cpu-decode"
    if not exe.exists():
        print(json.dumps({"impl": "reference", "unavailable": "reference CPU build (oracle/_ref) is missing"}))
        return
    threads = len(os.sched_getaffinity(0))
    full = reference_bench(model, steps, 3, threads)
    one = reference_bench(model, steps, 3, 1)
    v = full["tokens_per_s"]
    base = {"value": v, "unit": "tokens/s", "cores": threads, "kind": "reference", "value_1_thread": one["tokens_per_s"],
            "host_cpu": host_cpu(),
            "sample": f"reference cpu-decode bench --kernel {full['kernel']}: ctx {CONTEXT}, {steps} greedy steps, "
                      f"median of 3 repeats (1 warm-up step each, as the CLI runs it)"}
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": args.warmup, "ms_per_step": round(1000.0 / v, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 weights, f32 math",
            "data": "synthetic (seeded random-init weights N(0,0.02) and uniform token ids)",
            "config": headline_config(args.gpus), "cpu_baseline": base,
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-long", action="store_true", help="skip the ctx 4096 extra measurement")
    ap.add_argument("--no-batch", action="store_true", help="skip the batched 64-sequence measurement")
    ap.add_argument("--ncu-batch", type=int, default=0, metavar="SEQS",
                    help="the batched profiling case: SEQS sequences, --steps graph steps")
    ap.add_argument("--ncu-ctx", type=int, default=8192, help="largest context of the batched profiling case")
    ap.add_argument("--ncu-case", action="store_true",
                    help="the profiling case: KV rows 0..127 written from the host, then 5 decode launches")
    ap.add_argument("--ncu-long", type=int, default=0, metavar="CTX",
                    help="the long-context profiling case: KV rows 0..CTX-1 pre-filled, then 5 decode launches")
    ap.add_argument("--ncu-attention", type=int, default=0, metavar="L",
                    help="the isolated-attention profiling case: 5 calls at L positions, FP32 KV")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.ncu_case:
        ncu_case()
        return
    if args.ncu_long:
        ncu_case(args.ncu_long)
        return
    if args.ncu_attention:
        ncu_attention_case(args.ncu_attention)
        return
    if args.ncu_batch:
        ncu_batch_case(args.ncu_batch, max(1, args.steps), args.ncu_ctx)
        return

    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    dcb = load_package()
    model = ensure_model() if rank == 0 else None
    if dist:
        dist.barrier()
        model = ensure_model()
    import cpu_decode_b200.synthetic as syn
    d = syn.QWEN05
    K, W = max(1, args.steps), max(3, args.warmup)
    capacity = CONTEXT + K + W + 2
    eng = dcb.Engine(model, capacity, device=local)
    # A dedicated stream: the engine launches on it and the events are recorded on it.
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    eng.set_stream(stream.cuda_stream)
    prompt = prompt_tokens()

    # Prefill (untimed), seed token from the last prompt position.
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    for i, t in enumerate(prompt):
        eng.step_async(t, head=(i + 1 == len(prompt)), argmax_dev=tok.data_ptr())
    eng.synchronize()
    seed = tok.clone()

    def decode_window(n: int) -> None:
        for _ in range(n):
            eng.step_async(token_dev=tok.data_ptr(), head=True, argmax_dev=tok.data_ptr())

    # Warm-up, then a ~1 s untimed burst for the clock sampler, then rewind.
    clocks = ClockSampler(torch.cuda.current_device())
    decode_window(W)
    eng.synchronize()
    burst_end = time.time() + 1.0
    while time.time() < burst_end:
        eng.rewind(CONTEXT)
        tok.copy_(seed)
        decode_window(K)
        eng.synchronize()
    eng.rewind(CONTEXT)
    tok.copy_(seed)

    launches0 = eng.launch_count
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    start.record(stream)
    decode_window(K)
    end.record(stream)
    torch.cuda.synchronize()
    eng.synchronize()
    if dist:
        dist.barrier()
    clock_info = clocks.stop()
    ms = start.elapsed_time(end)
    gpu_launches = eng.launch_count - launches0
    generated_last = int(tok.item())
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = world * K / (ms / 1000.0)
    avg_bytes = sum(model_bytes_per_token(d, CONTEXT + i) for i in range(K)) / K
    per_launch_s = ms / 1000.0 / K
    peak, peak_kind = measured_peaks()
    achieved = avg_bytes / per_launch_s / 1e9

    # e2e through the public C ABI with host buffers (synchronous per step).
    eng.rewind(CONTEXT)
    nxt = int(seed.item())
    import ctypes
    pinned = torch.empty(d.vocab, dtype=torch.float32, pin_memory=True)  # the caller's logits buffer
    host_ptr = pinned.data_ptr()
    am = ctypes.c_int()
    lib = dcb.lib()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(K):
        rc = lib.dcb_step(eng._h, nxt, 1, host_ptr, ctypes.addressof(am))
        if rc:
            raise RuntimeError(lib.dcb_last_error().decode())
        nxt = am.value
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = world * K / e2e_s
    assert nxt == generated_last, "host-driven and device-chained greedy streams diverged"

    extra, tail = {}, {}
    if not args.no_batch:
        tail["batched"] = batched_decode(dcb, eng, d, dist, rank, world, W, eng_model_dir=model,
                                         cpu_sample=not args.no_cpu_baseline and world == 1)
    if dist and not args.no_long:
        split = kv_split_context(dcb, model, d, min(K, 32), W, local, dist, 32768)
        if rank == 0:
            tail["ctx32768_kv_split"] = split
    if rank == 0:
        # HBM read bandwidth of this GPU by the engine's own probe (the
        # reference's tools/bandwidth.cpp sweep), beside the measured peak.
        probe = dcb.read_bandwidth(mib=2048, passes=8, repeats=5, device=local)
        rates = sorted(x["GB_per_s"] for x in probe["samples"])
        extra["hbm_read_probe"] = {"GB_per_s_median": round(rates[len(rates) // 2], 1),
                                   "GB_per_s_max": round(rates[-1], 1), "array_bytes": probe["array_bytes"],
                                   "passes": probe["passes"], "kernel": probe["kernel"]}
    if rank == 0:
        extra["prefill128"] = prefill_time(dcb, model, local)
    if not args.no_long and rank == 0:
        extra["ctx4096"] = long_context(dcb, model, d, K, W, local, 4096)
        extra["ctx32768"] = long_context(dcb, model, d, min(K, 32), W, local, 32768)
        extra["gemv_sweep"] = gemv_sweep(dcb)
        extra["attention_sweep"] = attention_sweep(dcb)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": round(ms / K, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 weights, f32 math",
            "data": "synthetic (seeded random-init weights N(0,0.02) and uniform token ids)",
            "config": headline_config(world),
            "e2e": {"value": round(e2e_value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": d.vocab * 4 + 8},
            "gpu_launches": int(gpu_launches),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "algorithmic_bytes_per_launch": int(avg_bytes),
                         "traffic": profiled_traffic("role_step_kernel_ctx128.md"),
                         "kernel": "role_step_kernel"},
            "clocks": clock_info,
            "launch": eng.launch_info(),
        }
        # The reported CPU baseline runs at N=1 only: with other ranks alive
        # on the host it would measure contention, not the reference.
        if not args.no_cpu_baseline and world == 1:
            try:
                line["cpu_baseline"] = cpu_baseline(model)
            except Exception as exc:  # reported, never fatal
                line["cpu_baseline"] = {"value": None, "error": str(exc)[:200]}
        line.update(extra)
        if world > 1:
            line["scaling_limiter"] = (
                "batch-1 decode does not shard: the headline runs one independent replica per GPU (weak "
                "scaling, no collective); the multi-GPU work is `batched` (64 sequences per GPU, data parallel) "
                "and `ctx32768_kv_split` (one 32K stream, KV split over the GPUs, strong scaling bounded by the "
                "replicated dense part of every step and a per-layer NVLink exchange)")
        line.update(tail)  # last, so the multi-GPU results end the line
        print(json.dumps(line))
    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def ncu_case(ctx: int = CONTEXT) -> None:
    """Five decode launches at context `ctx` (128 by default) with few launches
    before them (the KV rows come from the host as seeded N(0,1) values, no
    prefill): launches 4 and 5 are the ones a profiler captures
    (`-k regex:decode_step -s 3 -c 2`)."""
    import torch
    dcb = load_package()
    import cpu_decode_b200.synthetic as syn
    model = ensure_model() if ctx <= CONTEXT else _long_model_dir(ensure_model())
    d = syn.QWEN05
    eng = dcb.Engine(model, ctx + 8)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    eng.set_stream(stream.cuda_stream)
    rng = np.random.default_rng(ctx)
    for l in range(d.layers):
        eng.kv_write(l, 0, rng.standard_normal((ctx, d.kv_dim), dtype=np.float32),
                     rng.standard_normal((ctx, d.kv_dim), dtype=np.float32))
    eng.set_position(ctx)
    tok = torch.full((1,), prompt_tokens()[-1], dtype=torch.int32, device="cuda")
    for _ in range(5):
        eng.step_async(token_dev=tok.data_ptr(), head=True, argmax_dev=tok.data_ptr())
    eng.synchronize()
    print(json.dumps({"ncu_case": f"decode_step_kernel ctx {ctx}", "launches": eng.launch_count,
                      "last_token": int(tok.item())}))
    eng.close()


def ncu_batch_case(seqs: int, steps: int, max_ctx: int = 8192) -> None:
    """The batched workload for a profiler: `seqs` sequences with the bench's
    seeded contexts (uniform [512, 8192]), KV pre-filled on the device, then
    `steps` graph steps. Capture with `-k regex:"gemm_i8|attention_kernel|
    combine_stage|stage_kernel|argmax_kernel"`: one step is
    1 + 9 x layers + 2 of these launches."""
    import torch
    dcb = load_package()
    import cpu_decode_b200.synthetic as syn
    model = ensure_model()
    d = syn.QWEN05
    eng = dcb.Engine(model, 1)
    rng = np.random.default_rng(100)
    ctxs = np.minimum(rng.integers(BATCH_CTX[0], BATCH_CTX[1] + 1, BATCH_SEQS)[:seqs], max_ctx)
    bat = dcb.Batch(eng, seqs, int(ctxs.max()) + steps + 2)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(2024)
    maxc = int(ctxs.max())
    for l in range(d.layers):
        k = torch.randn(maxc, d.kv_dim, device="cuda", generator=gen)
        v = torch.randn(maxc, d.kv_dim, device="cuda", generator=gen)
        torch.cuda.synchronize()
        for s in range(seqs):
            bat.kv_write(s, l, 0, k.data_ptr(), v.data_ptr(), count=int(ctxs[s]))
    for s in range(seqs):
        bat.set_position(s, int(ctxs[s]))
    bat.step(rng.integers(0, d.vocab, seqs).astype(np.int32), logits=False)
    bat.step_greedy(seqs, steps - 1)
    toks, _ = bat.read(seqs)
    print(json.dumps({"ncu_case": f"batched decode, {seqs} sequences", "steps": steps,
                      "kernels_per_step": bat.kernels_per_step(seqs), "last_tokens": toks[:4].tolist()}))
    bat.close()
    eng.close()


GEMV_SHAPES = [("qkv", 1152, 896, True), ("o", 896, 896, False), ("gate_up", 9728, 896, False),
               ("down", 896, 4864, False), ("lm_head", 151936, 896, False)]
ROTATE_BYTES = 300 << 20  # buffer copies cycled per shape: more than L2 (126 MB), so each call reads HBM


def _timed_calls(fn, n_calls: int, warmup: int = 3) -> tuple[float, float]:
    """Mean device time (ms) of one fn(i) call, CUDA events on the current
    stream: issued one by one, and replayed as a CUDA graph of n_calls
    back-to-back calls (no host launch cost)."""
    import torch
    for i in range(warmup):
        fn(i)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for i in range(n_calls):
        fn(warmup + i)
    e.record()
    torch.cuda.synchronize()
    eager = s.elapsed_time(e) / n_calls
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=torch.cuda.current_stream()):
        for i in range(n_calls):
            fn(i)
    graph.replay()
    torch.cuda.synchronize()
    s.record()
    graph.replay()
    e.record()
    torch.cuda.synchronize()
    graphed = s.elapsed_time(e) / n_calls
    del graph
    return eager, graphed


def prefill_time(dcb, model: Path, device: int, repeats: int = 5) -> dict:
    """The bench's 128-token prompt entering an empty engine: the reference's
    loop (src/main.cpp:134-137, one step per token, the LM head on the last)
    against dcb_prefill (up to 64 positions per batched tensor-core step).
    Wall time of the host call sequence, median of `repeats` after two warm-up
    rounds; both return once the K/V rows are written and the last logits are
    on the host. The two paths' last logits are compared."""
    prompt = prompt_tokens()
    n = len(prompt)
    eng = dcb.Engine(model, n + 8, device=device)

    def loop():
        eng.reset()
        for i, t in enumerate(prompt):
            out = eng.step(t, head=(i + 1 == n))
        return out

    def batched():
        eng.reset()
        return eng.prefill(prompt)

    def dump_loop():
        # the reference's `logits` command: the head on every token (src/main.cpp:93-114)
        eng.reset()
        rows = np.zeros((n, eng.vocab), np.float32)
        for i, t in enumerate(prompt):
            rows[i] = eng.step(t)[0]
        return rows, None

    def dump_batched():
        eng.reset()
        return eng.prefill_logits(prompt)

    times = {}
    results = {}
    for name, fn in (("token_by_token", loop), ("batched", batched), ("logits_dump_loop", dump_loop),
                     ("logits_dump_batched", dump_batched)):
        for _ in range(2):
            fn()
        samples = []
        for _ in range(repeats):
            t0 = time.perf_counter()
            logits, best = fn()
            samples.append(time.perf_counter() - t0)
        times[name] = sorted(samples)[len(samples) // 2]
        results[name] = (logits.copy(), best)
    eng.close()
    diff = float(np.abs(results["batched"][0] - results["token_by_token"][0]).max())
    dump_diff = float(np.abs(results["logits_dump_batched"][0] - results["logits_dump_loop"][0]).max())
    return {"prompt_tokens": n, "token_by_token_ms": round(times["token_by_token"] * 1e3, 3),
            "batched_ms": round(times["batched"] * 1e3, 3),
            "speedup": round(times["token_by_token"] / times["batched"], 2),
            "batched_tokens_per_s": round(n / times["batched"], 1),
            "max_abs_logit_diff": diff, "argmax_equal": results["batched"][1] == results["token_by_token"][1],
            "logits_dump": {"what": "every position's logits to host memory (the reference's logits command)",
                            "token_by_token_ms": round(times["logits_dump_loop"] * 1e3, 3),
                            "batched_ms": round(times["logits_dump_batched"] * 1e3, 3),
                            "speedup": round(times["logits_dump_loop"] / times["logits_dump_batched"], 2),
                            "max_abs_logit_diff": dump_diff}}


def gemv_sweep(dcb) -> dict:
    """The isolated per-row int8 GEMV at the five projection shapes (int8
    uniform [-127, 127], scales uniform [1e-4, 1e-3], x N(0,1)): algorithmic
    bytes = rows*cols + 4*rows (scales) + 4*cols (x) + 4*rows (y) [+ 4*rows bias]."""
    import torch
    peak, _ = measured_peaks()
    g = torch.Generator(device="cuda").manual_seed(1)
    out = {}
    for name, rows, cols, bias in GEMV_SHAPES:
        copies = max(2, -(-ROTATE_BYTES // (rows * cols)))
        w = [torch.randint(-127, 128, (rows, cols), dtype=torch.int8, device="cuda", generator=g) for _ in range(copies)]
        sc = torch.rand(rows, device="cuda", generator=g) * 9e-4 + 1e-4
        b = torch.randn(rows, device="cuda", generator=g) if bias else None
        x = torch.randn(cols, device="cuda", generator=g)
        y = torch.empty(rows, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream

        def call(i):
            dcb.gemv_i8(w[i % copies].data_ptr(), sc.data_ptr(), b.data_ptr() if bias else None, x.data_ptr(),
                        y.data_ptr(), rows, cols, stream)
        ms, ms_graph = _timed_calls(call, max(20, 2 * copies))
        nbytes = rows * cols + 4 * rows + 4 * cols + 4 * rows + (4 * rows if bias else 0)
        gbs = nbytes / (ms_graph / 1000.0) / 1e9
        out[name] = {"rows": rows, "cols": cols, "us_per_call": round(ms_graph * 1000.0, 2),
                     "us_per_call_eager": round(ms * 1000.0, 2), "bytes": nbytes,
                     "achieved_gbs": round(gbs, 1), "frac": round(gbs / peak, 4)}
        del w
    return out


def attention_sweep(dcb) -> dict:
    """Isolated GQA decode attention: 14 query heads over 2 KV heads, head_dim
    64, one query at position L-1 with RoPE theta 1e6, q/K/V N(0,1). KV bytes =
    L*2*2*64*{4,2}, each KV head read once for its 7 query heads."""
    import torch
    peak, _ = measured_peaks()
    heads, kvh, dim = 14, 2, 64
    g = torch.Generator(device="cuda").manual_seed(2)
    out = {}
    for kv, dt, es in (("f32", torch.float32, 4), ("f16", torch.float16, 2)):
        for length in (128, 1024, 4096, 32768):
            nbytes = length * 2 * kvh * dim * es
            copies = max(2, -(-ROTATE_BYTES // nbytes))
            k = [torch.randn(length, kvh * dim, device="cuda", generator=g).to(dt) for _ in range(copies)]
            v = [torch.randn(length, kvh * dim, device="cuda", generator=g).to(dt) for _ in range(copies)]
            q = torch.randn(heads * dim, device="cuda", generator=g)
            o = torch.empty(heads * dim, device="cuda")
            stream = torch.cuda.current_stream().cuda_stream

            def call(i):
                dcb.attention(q.data_ptr(), k[i % copies].data_ptr(), v[i % copies].data_ptr(), kv, o.data_ptr(),
                              length, heads, kvh, dim, 1e6, stream)
            ms, ms_graph = _timed_calls(call, max(20, 2 * copies))
            gbs = nbytes / (ms_graph / 1000.0) / 1e9
            out[f"{kv}_{length}"] = {"us_per_call": round(ms_graph * 1000.0, 2),
                                     "us_per_call_eager": round(ms * 1000.0, 2), "kv_bytes": nbytes,
                                     "achieved_gbs": round(gbs, 1), "frac": round(gbs / peak, 4)}
            del k, v
    return out


def ncu_attention_case(length: int) -> None:
    """Five calls of the isolated attention at `length` positions (the sweep's
    shape: 14 query heads over 2 KV heads, head_dim 64, FP32 KV, N(0,1) q/K/V,
    RoPE theta 1e6): a profiler captures the third."""
    import torch
    dcb = load_package()
    torch.cuda.set_stream(torch.cuda.Stream())
    heads, kvh, dim = 14, 2, 64
    g = torch.Generator(device="cuda").manual_seed(2)
    k = torch.randn(length, kvh * dim, device="cuda", generator=g)
    v = torch.randn(length, kvh * dim, device="cuda", generator=g)
    q = torch.randn(heads * dim, device="cuda", generator=g)
    o = torch.empty(heads * dim, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(5):
        dcb.attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), "f32", o.data_ptr(), length, heads, kvh, dim, 1e6, stream)
    torch.cuda.synchronize()
    print(json.dumps({"ncu_case": f"isolated attention, {length} positions", "out0": float(o[0].item())}))


BATCH_SEQS = 64           # independent sequences per GPU
BATCH_CTX = (512, 8192)   # per-sequence context, uniform
BATCH_STEPS = 128         # greedy steps each


def batched_decode(dcb, eng, d, dist, rank: int, world: int, warmup: int, kv: str = "f32",
                   eng_model_dir: Path | None = None, cpu_sample: bool = False) -> dict:
    """Batched multi-stream decode: 64 independent sequences per GPU, contexts
    uniform in [512, 8192] (seeded per rank), KV caches pre-filled with seeded
    N(0,1) rows, 128 greedy steps, every projection one tcgen05 int8 GEMM over
    all sequences. Data-parallel over ranks (replicated weights, no
    collective); tokens/s = all ranks' sequences x steps / max-over-ranks time.
    The step is one CUDA graph; steps chain on the device (each sequence's
    argmax is its next token). e2e: dcb_batch_step with host token and argmax
    buffers every step."""
    import ctypes
    import torch
    K = BATCH_STEPS
    rng = np.random.default_rng(100 + rank)
    ctxs = rng.integers(BATCH_CTX[0], BATCH_CTX[1] + 1, BATCH_SEQS)
    cap = int(ctxs.max()) + warmup + K + 2
    bat = dcb.Batch(eng, BATCH_SEQS, cap, kv_dtype=kv)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(2024 + rank)
    maxc = int(ctxs.max())
    for l in range(d.layers):
        k = torch.randn(maxc, d.kv_dim, device="cuda", generator=gen)
        v = torch.randn(maxc, d.kv_dim, device="cuda", generator=gen)
        torch.cuda.synchronize()
        for s in range(BATCH_SEQS):
            bat.kv_write(s, l, 0, k.data_ptr(), v.data_ptr(), count=int(ctxs[s]))
    del k, v
    toks = rng.integers(0, d.vocab, BATCH_SEQS).astype(np.int32)

    def reset():
        for s in range(BATCH_SEQS):
            bat.set_position(s, int(ctxs[s]))

    stream = torch.cuda.ExternalStream(bat.stream)
    reset()
    bat.step(toks, logits=False)
    bat.step_greedy(BATCH_SEQS, warmup - 1)
    bat.read(BATCH_SEQS)
    clocks = ClockSampler(torch.cuda.current_device())
    burst_end = time.time() + 1.0
    while time.time() < burst_end:
        reset()
        bat.step_greedy(BATCH_SEQS, 32)
        bat.read(BATCH_SEQS)
    reset()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    s_ev.record(stream)
    bat.step_greedy(BATCH_SEQS, K)
    e_ev.record(stream)
    torch.cuda.synchronize()
    bat.read(BATCH_SEQS)
    clock_info = clocks.stop()
    ms = s_ev.elapsed_time(e_ev)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    # Algorithmic bytes of one step on one GPU: every weight once (shared by all
    # sequences), each sequence's embedding row, new K/V row and K/V rows 0..pos.
    kvb = 4 if kv == "f32" else 2
    per_token_kv = d.layers * 2 * d.kv_dim * kvb
    weights_once = model_bytes_per_token(d, 0, kvb) - 2 * per_token_kv - (d.hidden + 4)
    step_bytes = [weights_once + sum((d.hidden + 4) + per_token_kv * (1 + int(c) + i + 1) for c in ctxs)
                  for i in range(K)]
    avg_bytes = sum(step_bytes) / K
    peak, peak_kind = measured_peaks()
    gbs = avg_bytes / (ms / 1000.0 / K) / 1e9

    # e2e through the C ABI with host buffers (tokens in, argmax out, every step).
    reset()
    lib = dcb.lib()
    host_toks = toks.copy()
    am = np.zeros(BATCH_SEQS, np.int32)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(K):
        rc = lib.dcb_batch_step(bat._h, BATCH_SEQS, host_toks.ctypes.data, None, am.ctypes.data)
        if rc:
            raise RuntimeError(lib.dcb_last_error().decode())
        host_toks[:] = am
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    kernels = bat.kernels_per_step(BATCH_SEQS)
    bat.close()
    cpu = batched_cpu_baseline(eng_model_dir, d, ctxs[:2]) if (rank == 0 and cpu_sample) else None
    return {
        "workload": "64 independent sequences per GPU, contexts uniform [512, 8192] (seeded), KV pre-filled with "
                    "seeded N(0,1) rows, 128 greedy steps, FP32 KV, qwen2.5-0.5b-shape int8",
        "gpus": world, "parallelism": f"dp{world}", "scaling": "weak",
        "tokens_per_s": round(world * BATCH_SEQS * K / (ms / 1000.0), 1),
        "ms_per_step": round(ms / K, 4),
        "mean_context": float(np.mean(ctxs)),
        "e2e": {"value": round(world * BATCH_SEQS * K / e2e_s, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": 4 * BATCH_SEQS, "d2h_bytes_per_step": 4 * (bat.slots + 1)},
        "gpu_launches": int(kernels * K),
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs / peak, 4), "peak_kind": peak_kind,
                     "algorithmic_bytes_per_step": int(avg_bytes), "kernel": "whole step (graph)",
                     "traffic": profiled_traffic("batched_decode_64seq.md", "dram_bytes_per_step")},
        "clocks": clock_info,
        "cpu_baseline": cpu,
    }


def batched_cpu_baseline(model_dir: Path, d, contexts, steps: int = 2) -> dict:
    """The reference has no batch: it decodes each sequence with its own
    engine, and cannot take a pre-filled KV cache. The C restatement of its
    step over a caller-owned cache stands in (kind "port"): two of the
    batch's sequences at their own contexts (seeded N(0,1) KV rows), a few
    greedy steps each, all host threads; tokens/s of that sample."""
    sys.path.insert(0, str(ROOT))
    import oracle
    threads = len(os.sched_getaffinity(0))
    rng = np.random.default_rng(7)
    total, elapsed = 0, 0.0
    for ctx in contexts:
        ctx = int(ctx)
        orc = oracle.Oracle(model_dir, ctx + steps + 1, threads=threads)
        kc, vc = orc.kv_view()
        for l in range(d.layers):
            kc[l, :ctx] = rng.standard_normal((ctx, d.kv_dim), dtype=np.float32)
            vc[l, :ctx] = rng.standard_normal((ctx, d.kv_dim), dtype=np.float32)
        orc.pos = ctx
        tok = 1234
        t0 = time.perf_counter()
        for _ in range(steps):
            tok = oracle.argmax(orc.step(tok))
        elapsed += time.perf_counter() - t0
        total += steps
    return {"value": round(total / elapsed, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"C restatement of the reference step, one sequence at a time: contexts "
                      f"{[int(c) for c in contexts]}, {steps} greedy steps each"}


def _long_model_dir(model: Path) -> Path:
    """The same model with max_position_embeddings raised for long contexts."""
    long_dir = MODEL_CACHE / "qwen05_seed0_long"
    long_dir.mkdir(parents=True, exist_ok=True)
    cfg = json.loads((model / "config.json").read_text())
    cfg["max_position_embeddings"] = 40960
    (long_dir / "config.json").write_text(json.dumps(cfg))
    link = long_dir / "model.safetensors"
    if not link.exists():
        link.symlink_to((model / "model.safetensors").resolve())
    return long_dir


def kv_split_context(dcb, model, d, K, W, device, dist, ctx: int) -> dict:
    """One stream at `ctx` pre-filled positions with its KV cache split over
    all ranks (one GPU each): each rank keeps a contiguous range, the last one
    also the new tokens; every rank runs the whole step and the ranks merge the
    per-head attention partials over NVLink each layer. Same seeded K/V rows as
    the one-GPU measurement. Device-chained greedy steps, time = max over
    ranks (strong scaling: the total work is fixed)."""
    import torch
    rank, world = dist.get_rank(), dist.get_world_size()
    if rank == 0:
        _long_model_dir(model)
    dist.barrier()
    long_dir = MODEL_CACHE / "qwen05_seed0_long"
    out = {}
    for kvt in ("f32",):
        begin, end = dcb.kv_shard_ranges(ctx, world)[rank]
        cap = (end if end is not None else ctx + K + W + 2) - begin
        eng = dcb.Engine(long_dir, cap, kv_dtype=kvt, device=device)
        stream = torch.cuda.current_stream()
        eng.set_stream(stream.cuda_stream)
        peers = dcb.split_kv(eng, begin, end)
        rng = np.random.default_rng(ctx)
        top = ctx if end is None else end
        for l in range(d.layers):  # the same rows as the one-GPU run draws, this rank's slice
            k = rng.standard_normal((ctx, d.kv_dim), dtype=np.float32)
            v = rng.standard_normal((ctx, d.kv_dim), dtype=np.float32)
            eng.kv_write(l, begin, k[begin:top], v[begin:top])
        tok = torch.full((1,), 1234, dtype=torch.int32, device="cuda")
        eng.set_position(ctx)
        for _ in range(W):
            eng.step_async(token_dev=tok.data_ptr(), head=True, argmax_dev=tok.data_ptr())
        eng.synchronize()
        eng.set_position(ctx)
        tok.fill_(1234)
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record(stream)
        for _ in range(K):
            eng.step_async(token_dev=tok.data_ptr(), head=True, argmax_dev=tok.data_ptr())
        e.record(stream)
        torch.cuda.synchronize()
        eng.synchronize()
        ms = torch.tensor([s.elapsed_time(e)], device="cuda")
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        last = torch.tensor([int(tok.item())], device="cuda", dtype=torch.int64)
        lmax, lmin = last.clone(), last.clone()
        dist.all_reduce(lmax, op=dist.ReduceOp.MAX)
        dist.all_reduce(lmin, op=dist.ReduceOp.MIN)
        # Parity: a few host-driven steps with logits on the split (every rank
        # steps together), then one unsplit engine on rank 0 over the same
        # rows and tokens.
        S = 3
        eng.set_position(ctx)
        nxt = 1234
        split_logits, split_tokens = [], []
        for _ in range(S):
            lg, best = eng.step(nxt)
            split_logits.append(lg.copy())
            split_tokens.append(int(best))
            nxt = int(best)
        dist.barrier()
        eng.close()
        for p in peers:
            dcb.ipc_close(p)
        parity = None
        if rank == 0:
            one = dcb.Engine(long_dir, ctx + S + 2, kv_dtype=kvt, device=device)
            rng = np.random.default_rng(ctx)
            for l in range(d.layers):
                k = rng.standard_normal((ctx, d.kv_dim), dtype=np.float32)
                v = rng.standard_normal((ctx, d.kv_dim), dtype=np.float32)
                one.kv_write(l, 0, k, v)
            one.set_position(ctx)
            nxt, diff, toks = 1234, 0.0, []
            for i in range(S):
                lg, best = one.step(nxt)
                diff = max(diff, float(np.abs(lg - split_logits[i]).max()))
                toks.append(int(best))
                nxt = int(best)
            one.close()
            parity = {"steps": S, "max_abs_logit_diff": diff, "tokens_equal": toks == split_tokens}
        dist.barrier()
        t = float(ms.item())
        out[kvt] = {"gpus": world, "tokens_per_s": round(K / (t / 1000.0), 2), "ms_per_step": round(t / K, 5),
                    "ranks_agree": bool(lmax.item() == lmin.item()), "vs_one_gpu": parity}
    return out


def long_context(dcb, model, d, K, W, device, ctx: int = 4096) -> dict:
    """The full model at a long context: KV rows 0..ctx-1 pre-filled with
    seeded N(0,1) values (as if already rotated), then greedy steps, F16 and
    FP32 KV."""
    import torch
    import cpu_decode_b200.synthetic as syn
    out = {}
    long_dir = _long_model_dir(model)
    rng = np.random.default_rng(ctx)
    kv = [(rng.standard_normal((ctx, d.kv_dim), dtype=np.float32), rng.standard_normal((ctx, d.kv_dim), dtype=np.float32))
          for _ in range(d.layers)]
    for kvt in ("f32", "f16"):
        eng = dcb.Engine(long_dir, ctx + K + W + 2, kv_dtype=kvt, device=device)
        stream = torch.cuda.current_stream()
        assert stream.cuda_stream, "the engine must launch on the stream the events are recorded on"
        eng.set_stream(stream.cuda_stream)
        for l, (k, v) in enumerate(kv):
            eng.kv_write(l, 0, k, v)
        tok = torch.full((1,), 1234, dtype=torch.int32, device="cuda")
        eng.set_position(ctx)
        for _ in range(W):
            eng.step_async(token_dev=tok.data_ptr(), head=True, argmax_dev=tok.data_ptr())
        eng.synchronize()
        eng.set_position(ctx)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record(stream)
        for _ in range(K):
            eng.step_async(token_dev=tok.data_ptr(), head=True, argmax_dev=tok.data_ptr())
        e.record(stream)
        torch.cuda.synchronize()
        eng.synchronize()
        ms = s.elapsed_time(e)
        kvb = 4 if kvt == "f32" else 2
        avg = sum(model_bytes_per_token(d, ctx + i, kvb) for i in range(K)) / K
        peak, _ = measured_peaks()
        gbs = avg / (ms / 1000.0 / K) / 1e9
        out[kvt] = {"tokens_per_s": round(K / (ms / 1000.0), 2), "ms_per_step": round(ms / K, 5),
                    "achieved_gbs": round(gbs, 1), "frac": round(gbs / peak, 4), "bytes_per_token": int(avg)}
        eng.close()
    return out


if __name__ == "__main__":
    main()
