"""Benchmark of the batched multi-adapter LoRA hot path.

Workload (per GPU, weak scaling): T = 16384 token rows x 4096 features,
output 4096, 64 adapter slots + __base__, max_rank 16, per-slot rank uniform
in {0,4,8,16}, 20% of rows on __base__, A ~ U(-1/64,1/64), B ~ N(0,0.02),
scale = 16/r, base output y ~ N(0,1) updated in place; bf16.  Seeded
synthetic data (the reference publishes no dataset for this path).

One step = one pass of the hot path as a wrapped Linear runs it: device
segment table (3 small kernels) + SGMV shrink + SGMV expand (fused scale and
add-back).  Inputs (x 128 MiB + y 128 MiB per GPU) exceed the 126 MB L2.

Prints one JSON line (rank 0).  ``--impl reference`` times the reference's CPU
algorithm (the oracle port of layers.py:112-134, numpy fp32 with all host
threads) on the same workload instead.
"""

from __future__ import annotations

import argparse
import json
import os
import shutil
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "mixed-adapter tokens/s at 1/2/4/8 B200; SGMV achieved HBM GB/s vs peak"
T_TOKENS, K_IN, N_OUT, SLOTS, MAX_RANK = 16384, 4096, 4096, 65, 16
SEG_ONE_LAUNCH_ROWS = 1024  # rows the one-launch segment builder takes (csrc/segments.cuh)
SEG_SCAN_PLACE_INTS = 12288  # count-matrix size up to which scan and placement are one launch
SEG_ROWS_PER_BLOCK = 256     # rows per count block of the segment builder
E2E_CHUNKS = 4  # row chunks of the host-buffer pipeline (e2e leg; 4: 5.40 ms, 8: 5.62, 16: 6.04 per step)
ELEM = 2  # bf16


def workload(seed: int):
    """Host-side description of the synthetic config-2 batch (numpy)."""
    rng = np.random.default_rng(seed)
    ranks = np.array([0] + list(rng.choice([0, 4, 8, 16], size=SLOTS - 1)), dtype=np.int32)
    wi = rng.integers(1, SLOTS, size=T_TOKENS).astype(np.int64)
    wi[rng.random(T_TOKENS) < 0.2] = 0
    scales = np.array([0.0] + [16.0 / r if r else 0.0 for r in ranks[1:]], dtype=np.float32)
    return ranks, wi, scales


def algorithmic_bytes(ranks, wi):
    """Per-launch algorithmic bytes (shrink, expand, combined step figure)."""
    active = ranks[wi] > 0
    t_act = int(active.sum())
    used = np.unique(wi[active])
    rsum = int(ranks[used].sum())
    shrink = t_act * K_IN * ELEM + K_IN * rsum * ELEM + t_act * MAX_RANK * ELEM
    expand = t_act * MAX_RANK * ELEM + rsum * N_OUT * ELEM + 2 * t_act * N_OUT * ELEM
    combined = t_act * (K_IN + 2 * N_OUT) * ELEM + (K_IN + N_OUT) * rsum * ELEM
    return t_act, shrink, expand, combined


def kernel_source_digest() -> str:
    """sha256 over the library's CUDA / C sources and header (the code a
    profile of the kernels describes)."""
    import hashlib

    h = hashlib.sha256()
    csrc = ROOT / "polylora_b200" / "csrc"
    for path in sorted(list(csrc.glob("*.cu")) + list(csrc.glob("*.cuh")) + list(csrc.glob("*.h"))) + [
            ROOT / "include" / "polylora_b200.h"]:
        h.update(path.name.encode())
        h.update(path.read_bytes())
    return h.hexdigest()


def traffic_record(kernel: str):
    """DRAM bytes per launch of `kernel` from the committed ncu summary, when
    that summary was captured on these exact sources; else (None, reason)."""
    path = ROOT / "profiles" / "traffic_cfg2.json"
    if not path.exists():
        return None, "no ncu traffic record in profiles/"
    rec = json.loads(path.read_text())
    entry = rec.get("kernels", {}).get(kernel)
    if entry is None:
        return None, f"profiles/traffic_cfg2.json has no capture of {kernel}"
    if rec.get("source_sha256") != kernel_source_digest():
        return None, "profiles/traffic_cfg2.json was captured on other kernel sources"
    return int(entry["dram_bytes_per_launch"]), "ncu capture of this build (profiles/traffic_cfg2.json)"


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.out = None

    def start(self):
        if shutil.which("nvidia-smi") is None:
            return
        self.out = tempfile.TemporaryFile(mode="w+")
        self.proc = subprocess.Popen(
            ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
             "-lms", "100"], stdout=self.out, stderr=subprocess.DEVNULL)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.seek(0)
        rows = [r.split(",") for r in self.out.read().strip().splitlines() if r.strip()]
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
                for name, flag in zip(names, r[5:9]):
                    if flag.strip().lower() == "active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus: int):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def cpu_baseline(seed: int, budget_s: float = 12.0, max_steps: int | None = None):
    """Oracle port of the reference's CPU path on the host cores (fp32)."""
    from oracle import sgmv_ref

    ranks, wi, scales = workload(seed)
    rng = np.random.default_rng(seed + 1)
    A = np.zeros((SLOTS, K_IN, MAX_RANK), np.float32)
    B = np.zeros((SLOTS, MAX_RANK, N_OUT), np.float32)
    for s in range(1, SLOTS):
        r = int(ranks[s])
        A[s, :, :r] = rng.uniform(-1 / 64, 1 / 64, (K_IN, r))
        B[s, :r] = rng.normal(0, 0.02, (r, N_OUT))
    x = rng.standard_normal((T_TOKENS, 1, K_IN), dtype=np.float32)
    y = rng.standard_normal((T_TOKENS, 1, N_OUT), dtype=np.float32)
    seq = np.ones(T_TOKENS, np.int32)
    sgmv_ref.lora_forward_grouped(x, A, B, seq, wi, ranks, scales, y)  # warm-up
    times = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        sgmv_ref.lora_forward_grouped(x, A, B, seq, wi, ranks, scales, y)
        times.append(time.perf_counter() - t0)
        if max_steps is not None and len(times) >= max_steps:
            break
        if max_steps is None and time.perf_counter() - t_start > budget_s:
            break
    per = statistics.median(times)
    return {
        "value": T_TOKENS / per,
        "unit": "tokens/s",
        "cores": os.cpu_count(),
        "kind": "port",
        "sample": f"full config-2 batch ({T_TOKENS} tokens, fp32 numpy, rows grouped by slot), "
                  f"median of {len(times)} passes",
    }


def reference_own_cpu(seed: int = 0, rows: int = 2048, budget_s: float = 6.0) -> dict:
    """The reference's own CPU code from baseline/_ref, unmodified, on the host
    cores (all threads): (1) MultiLoraLinear._reference_forward
    (src/polylora/layers.py:112-134, a Python loop over rows with .item()
    reads) on the first `rows` rows of the config-2 batch, in fp32 and bf16;
    (2) BASELINE config 1, the reference PolyLoraModel with
    use_triton_kernels=False around a DeBERTa-v3-small-shaped encoder (fp32,
    random init, 4 adapters, batch 8 x 128 right-padded), one forward."""
    import types

    import torch

    out: dict = {"threads": os.cpu_count()}
    try:
        sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
        from polylora import PolyLoraConfig as RefConfig, PolyLoraModel as RefModel
        from polylora.layers import MultiLoraLinear as RefLinear
        from polylora.store import CpuLayerWeights as RefWeights
    except Exception as exc:  # noqa: BLE001
        return {"unavailable": f"reference not importable from baseline/_ref: {type(exc).__name__}: {exc}"}
    torch.set_num_threads(os.cpu_count() or 1)
    ranks_np, wi_np, scales_np = workload(seed)

    def timed(fn):
        fn()
        times, t_end = [], time.perf_counter() + budget_s
        while len(times) < 3 or (time.perf_counter() < t_end and len(times) < 50):
            t0 = time.perf_counter()
            fn()
            times.append(time.perf_counter() - t0)
        return statistics.median(times), len(times)

    for dtype, name in ((torch.float32, "fp32"), (torch.bfloat16, "bf16")):
        g = torch.Generator().manual_seed(seed + 1)
        A = torch.zeros(SLOTS, K_IN, MAX_RANK)
        B = torch.zeros(SLOTS, MAX_RANK, N_OUT)
        for s_ in range(1, SLOTS):
            r = int(ranks_np[s_])
            A[s_, :, :r] = (torch.rand(K_IN, r, generator=g) * 2 - 1) / 64
            B[s_, :r] = torch.randn(r, N_OUT, generator=g) * 0.02
        cache = types.SimpleNamespace(A={"m": A.to(dtype)}, B={"m": B.to(dtype)},
                                      ranks={"m": torch.from_numpy(ranks_np)}, scales={"m": torch.from_numpy(scales_np)})
        layer = types.SimpleNamespace(cache=cache, module_name="m")
        x = torch.randn(rows, 1, K_IN, generator=g).to(dtype)
        base = torch.randn(rows, 1, N_OUT, generator=g).to(dtype)
        seq = torch.ones(rows, dtype=torch.int32)
        idx = torch.from_numpy(wi_np[:rows])
        sec, n = timed(lambda: RefLinear._reference_forward(layer, x, base, seq, idx))
        out[f"reference_forward_{name}"] = {"tokens_per_s": rows / sec, "ms_per_pass": sec * 1e3, "passes": n,
                                           "sample": f"first {rows} rows of the config-2 batch (T=16384), {name}"}

    # BASELINE config 1 through the reference's model wrapper on the CPU
    torch.manual_seed(0)
    enc = _deberta_v3_small().float()
    targets = ["query_proj", "key_proj", "value_proj", "dense"]
    shapes = {n: (m.in_features, m.out_features) for n, m in enc.named_modules()
              if isinstance(m, torch.nn.Linear) and any(n == t or n.endswith("." + t) for t in targets)}
    model = RefModel(enc, RefConfig(max_gpu_adapters=4, max_rank=16, target_modules=targets, use_triton_kernels=False))
    rng = np.random.default_rng(0)
    for i, r in enumerate((4, 8, 8, 16)):
        layers = {}
        for mod, (k, n_out) in shapes.items():
            a = torch.empty(r, k)
            torch.nn.init.kaiming_uniform_(a, a=5 ** 0.5)
            layers[mod] = RefWeights(A=a.t().contiguous(), B=torch.randn(r, n_out) * 0.02, rank=r, scale=2.0)
        model.adapter_store.add_adapter(f"a{i}", layers, {"r": r, "lora_alpha": 2 * r})
    lens = rng.integers(32, 129, size=8)
    ids = [["__base__", "a0", "a1", "a2", "a3"][int(j)] for j in rng.integers(0, 5, size=8)]
    input_ids = torch.from_numpy(rng.integers(0, 128100, size=(8, 128))).long()
    mask = (torch.arange(128)[None, :] < torch.from_numpy(lens)[:, None]).long()
    with torch.inference_mode():
        sec, n = timed(lambda: model(input_ids=input_ids, attention_mask=mask, adapter_ids=ids))
    out["cfg1_model_forward"] = {"ms_per_forward": sec * 1e3, "non_pad_tokens_per_s": int(lens.sum()) / sec,
                                 "forwards": n, "workload": "BASELINE config 1: DeBERTa-v3-small-shaped encoder "
                                 "(6 layers, hidden 768), fp32 CPU, 36 wrapped Linears, 4 adapters ranks {4,8,8,16}, "
                                 "batch 8 x 128 right-padded, lengths U[32,128]; reference PolyLoraModel, "
                                 "use_triton_kernels=False"}
    return out


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and rank != 0:
        return
    cb = cpu_baseline(seed=0, max_steps=max(args.steps, 1))
    line = {
        "impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * T_TOKENS / cb["value"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "BASELINE config 2 SGMV op, T=16384, K=N=4096, 64 slots, max_rank 16",
                   "path": "reference CPU algorithm (layers.py:112-134), oracle port, host cores"},
        "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "reference_own": reference_own_cpu(seed=0),
    }
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    import torch.distributed as dist

    from polylora_b200 import _native
    from polylora_b200.host_io import HostLoraPipeline
    from polylora_b200.sgmv import (build_segments, sgmv_expand, sgmv_lora_a_fwd, sgmv_lora_b_fwd, sgmv_shrink,
                                    sgmv_shrink_expand)

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", torch.cuda.current_device())
    ranks_np, wi_np, scales_np = workload(seed=rank)
    t_act, b_shrink, b_expand, b_comb = algorithmic_bytes(ranks_np, wi_np)

    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    ranks = torch.from_numpy(ranks_np).to(dev)
    colmask = (torch.arange(MAX_RANK, device=dev)[None, :] < ranks[:, None]).float()
    A = ((torch.rand(SLOTS, K_IN, MAX_RANK, device=dev, generator=g) * 2 - 1) / 64 * colmask[:, None, :]).to(torch.bfloat16)
    Bw = (torch.randn(SLOTS, MAX_RANK, N_OUT, device=dev, generator=g) * 0.02 * colmask[:, :, None]).to(torch.bfloat16)
    scales = torch.from_numpy(scales_np).to(dev)
    wi = torch.from_numpy(wi_np).to(dev)
    seq = torch.ones(T_TOKENS, dtype=torch.int32, device=dev)
    x = torch.randn(T_TOKENS, 1, K_IN, device=dev, generator=g).to(torch.bfloat16)
    y = torch.randn(T_TOKENS, 1, N_OUT, device=dev, generator=g).to(torch.bfloat16)
    stream = torch.cuda.Stream(device=dev)

    tmp_buf = torch.empty(T_TOKENS, 1, MAX_RANK, device=dev, dtype=torch.bfloat16)

    def step(tmp_out=None):
        table = build_segments(wi, seq, ranks, 1)
        tmp = tmp_buf if tmp_out is None else tmp_out
        sgmv_shrink_expand(x, A, Bw, y, table, ranks, scales, tmp=tmp)
        return table, tmp

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident timed region: the step captured once as a CUDA graph
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            table, tmp = step()
        for _ in range(max(args.warmup, 3)):
            graph.replay()
    torch.cuda.synchronize()
    status = _native.device_status(clear=True)
    if status:
        raise RuntimeError(f"device status {status:#x} after warm-up")

    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    ids = [v for v in visible.split(",") if v.strip().isdigit()]
    sampler = ClockSampler(int(ids[local]) if local < len(ids) else local)
    barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        ev1.record(stream)
    ev1.synchronize()
    barrier()
    torch.cuda.synchronize()
    elapsed_ms = max_over_ranks(ev0.elapsed_time(ev1))
    ms_per_step = elapsed_ms / args.steps

    # ---- per-kernel durations with L2 flushed before every launch: CUDA events on
    # `stream` around replays of a graph [flush, kernel] minus replays of [flush],
    # the flush writing 256 MiB then reading another 256 MiB (L2 is 126 MB)
    flush_w = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush_r = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    flush_sink = torch.empty((), dtype=torch.float32, device=dev)

    def flush():
        flush_w.fill_(7)
        torch.sum(flush_r, dim=0, out=flush_sink)

    def graph_of(fns):
        with torch.cuda.stream(stream):
            for f in fns:
                f()
            torch.cuda.synchronize()
            gk = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gk, stream=stream):
                for f in fns:
                    f()
            gk.replay()
        torch.cuda.synchronize()
        return gk

    def replay_ms(gk, reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            a.record(stream)
            for _ in range(reps):
                gk.replay()
            b.record(stream)
        b.synchronize()
        return a.elapsed_time(b) / reps

    def time_kernel(fn, reps):
        g_flush = graph_of([flush])
        g_both = graph_of([flush, fn])
        samples = sorted(replay_ms(g_both, reps) - replay_ms(g_flush, reps) for _ in range(3))
        return samples[1]

    reps = max(args.steps // 2, 10)
    shrink_ms = time_kernel(lambda: sgmv_shrink(x, A, table, ranks, out=tmp), reps)
    expand_ms = time_kernel(lambda: sgmv_expand(tmp, Bw, y, table, ranks, scales), reps)
    pair_ms = time_kernel(lambda: sgmv_shrink_expand(x, A, Bw, y, table, ranks, scales, tmp=tmp), reps)
    seg_ms = time_kernel(lambda: build_segments(wi, seq, ranks, 1), reps)
    count_blocks = (T_TOKENS + SEG_ROWS_PER_BLOCK - 1) // SEG_ROWS_PER_BLOCK
    seg_launches = 1 if T_TOKENS <= SEG_ONE_LAUNCH_ROWS else (2 if count_blocks * SLOTS <= SEG_SCAN_PLACE_INTS else 3)
    del flush_w, flush_r
    clocks = sampler.stop()

    # ---- end to end through the public drop-in operators with host buffers
    x_h = x.cpu().pin_memory()
    y_h = y.cpu().pin_memory()
    meta_h = [t.cpu().pin_memory() for t in (seq, wi, ranks, scales)]
    out_h = torch.empty_like(y_h).pin_memory()
    x_d, y_d = torch.empty_like(x), torch.empty_like(y)
    meta_d = [torch.empty_like(t) for t in (seq, wi, ranks, scales)]
    A_b = A  # adapter slots stay resident (GPU tier), as in serving

    def serial_step():  # the reference operators as a host-buffer caller uses them: in, compute, out
        x_d.copy_(x_h, non_blocking=True)
        y_d.copy_(y_h, non_blocking=True)
        for d_, h_ in zip(meta_d, meta_h):
            d_.copy_(h_, non_blocking=True)
        t = sgmv_lora_a_fwd(x_d, A_b, meta_d[0], meta_d[1], meta_d[2])
        sgmv_lora_b_fwd(t, Bw, meta_d[0], meta_d[1], meta_d[2], meta_d[3], y_d)
        out_h.copy_(y_d, non_blocking=True)

    pipe = HostLoraPipeline(dev, chunks=E2E_CHUNKS)
    ranks_d, scales_d = meta_d[2], meta_d[3]
    ranks_d.copy_(meta_h[2])
    scales_d.copy_(meta_h[3])

    def pipelined_step():  # the package's host-buffer entry, in place: only the table's rows cross the bus
        pipe(x_h, A_b, Bw, meta_h[0], meta_h[1], ranks_d, scales_d, y_h, y_h)

    pipe_all = HostLoraPipeline(dev, chunks=E2E_CHUNKS, active_rows=False)

    def all_rows_step():  # the same call moving every row by copies
        pipe_all(x_h, A_b, Bw, meta_h[0], meta_h[1], ranks_d, scales_d, y_h, out_h)

    def time_e2e(fn):
        with torch.cuda.stream(stream):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e_steps = max(3, min(args.steps, 20))
            e0.record(stream)
            for _ in range(e_steps):
                fn()
            e1.record(stream)
        e1.synchronize()
        return max_over_ranks(e0.elapsed_time(e1)) / e_steps

    serial_ms = time_e2e(serial_step)
    all_rows_ms = time_e2e(all_rows_step)
    e2e_ms = time_e2e(pipelined_step)  # last: it adds each step's delta into y_h
    meta_bytes = sum(t.numel() * t.element_size() for t in meta_h[:2])
    h2d = t_act * (K_IN + N_OUT) * ELEM + meta_bytes  # x and base-output rows of the active tokens
    d2h = t_act * N_OUT * ELEM
    status = _native.device_status(clear=True)
    if status:
        raise RuntimeError(f"device status {status:#x} during the bench")

    peak, peak_kind = measured_peaks()
    achieved_expand = b_expand / (expand_ms * 1e-3) / 1e9
    achieved_shrink = b_shrink / (shrink_ms * 1e-3) / 1e9
    stream = _native.stream_kernels() != 0
    fused = _native.stream_kernels() == 2  # the combined call is one kernel (K = N = 4096 fits it)
    k_shrink = "sgmv_shrink_stream_kernel<bf16>" if stream else "sgmv_shrink_mma_kernel<16,bf16>"
    k_expand = "sgmv_expand_stream_kernel<bf16>" if stream else "sgmv_expand_mma_kernel<16,bf16>"
    k_fused = "sgmv_shrink_stream_kernel<bf16, fused>"
    traffic, traffic_source = traffic_record(k_expand)
    traffic_shrink, _ = traffic_record(k_shrink)
    traffic_fused, traffic_fused_source = traffic_record(k_fused)
    b_pair = b_shrink + b_expand
    achieved_pair = b_pair / (pair_ms * 1e-3) / 1e9
    if fused:  # the step's dominant kernel is the fused one
        roofline = {"kernel": k_fused, "bound": "hbm", "achieved": achieved_pair, "peak": peak, "unit": "GB/s",
                    "frac": achieved_pair / peak, "peak_source": peak_kind, "traffic": traffic_fused,
                    "traffic_source": traffic_fused_source, "algorithmic_bytes_per_launch": b_pair,
                    "avg_launch_ms": pair_ms}
    else:
        roofline = {"kernel": k_expand, "bound": "hbm", "achieved": achieved_expand, "peak": peak, "unit": "GB/s",
                    "frac": achieved_expand / peak, "peak_source": peak_kind, "traffic": traffic,
                    "traffic_source": traffic_source, "algorithmic_bytes_per_launch": b_expand,
                    "avg_launch_ms": expand_ms}

    # the reference's own GPU path (its Triton kernels) on this B200, same batch
    triton_ref = _triton_pair_cfg2(dev, x, A, Bw, seq, wi, ranks, scales, y) if world == 1 else None
    # BASELINE config 3 at this N: row-parallel model forward with the NCCL all-gather in the step
    try:
        cfg3 = _cfg3_row_parallel(world, rank, dev, steps=3, warmup=2)
    except Exception as exc:  # noqa: BLE001 - reported in the line, not fatal
        cfg3 = {"unavailable": f"{type(exc).__name__}: {exc}"}

    cb = cpu_baseline(seed=0) if (rank == 0 and world == 1 and not args.no_cpu_baseline) else None
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    value = world * T_TOKENS / (ms_per_step * 1e-3)
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {
            "workload": "BASELINE config 2 SGMV op: T=16384 token rows per GPU, K=N=4096, 64 slots + __base__, "
                        "max_rank 16, ranks U{0,4,8,16}, 20% base rows",
            "step": ("device segment table + sgmv shrink + sgmv expand (fused scale/add-back) issued as one call: "
                     + ("one fused kernel, each CTA expanding the share it has just shrunk" if fused
                        else "two kernels, the expand overlapping the shrink's end") + "; CUDA graph"),
            "l2": "step: inputs larger than L2 (x 128 MiB + y 128 MiB per GPU); per-kernel times: L2 flushed "
                  "(256 MiB write + 256 MiB read) before every launch, outside the timed difference",
            "parallelism": f"row data-parallel x{world}, independent slot caches, no collective in the step",
            "active_tokens_per_gpu": t_act,
        },
        "roofline": roofline,
        "kernels": {
            "shrink": {"kernel": k_shrink, "avg_launch_ms": shrink_ms, "bytes": b_shrink, "gbs": achieved_shrink,
                       "frac": achieved_shrink / peak, "traffic": traffic_shrink},
            "expand": {"kernel": k_expand, "avg_launch_ms": expand_ms, "bytes": b_expand, "gbs": achieved_expand,
                       "frac": achieved_expand / peak, "traffic": traffic},
            "segments": {"avg_ms": seg_ms, "launches": seg_launches},
            "shrink_expand_call": {"kernel": k_fused if fused else f"{k_shrink} + {k_expand}", "avg_ms": pair_ms,
                                   "bytes": b_pair, "gbs": achieved_pair, "frac": achieved_pair / peak,
                                   "traffic": traffic_fused if fused else None},
            "step_combined_gbs": b_comb / (ms_per_step * 1e-3) / 1e9,
        },
        "cpu_baseline": cb,
        "e2e": {"value": world * T_TOKENS / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                "path": f"HostLoraPipeline in place ({E2E_CHUNKS} row chunks; per chunk: seq_lens, "
                        "weight_indices in by copy, segment table, the table's x and base-output rows read "
                        "from pinned host memory by plora_gather_token_rows, shrink + expand, the table's "
                        "output rows written back by plora_scatter_token_rows on a second stream; rows of "
                        "__base__ / rank-0 tokens stay in host memory, unchanged); slot weights, ranks, "
                        "scalings resident",
                "all_rows_ms_per_step": all_rows_ms,
                "all_rows_path": "the same pipeline copying every row in and out (x, base output in on one copy "
                                 "stream, output out on another)",
                "serial_ms_per_step": serial_ms,
                "serial_path": "sgmv_lora_a_fwd + sgmv_lora_b_fwd (C-ABI) on one stream: pinned host x/y/metadata "
                               "in, y out"},
        "gpu_launches": (seg_launches + (1 if fused else 2)) * args.steps,
        "clocks": clocks,
        "triton_reference": triton_ref,
        "model_cfg3": cfg3,
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _triton_pair_cfg2(dev, x, A, Bw, seq, wi, ranks, scales, y):
    """The reference's own GPU path on this B200: its unmodified Triton
    sgmv_lora_a_fwd + sgmv_lora_b_fwd (src/polylora/sgmv.py:141-175, 278-328,
    from baseline/_ref) against this library's operators of the same
    signatures, eager calls as layers.py:42-58 makes them, on the benched
    config-2 batch; L2 flushed before each pair (loop [flush, pair] minus loop
    [flush]).  None fields and a reason when the reference is not installed."""
    import torch

    from polylora_b200.sgmv import sgmv_lora_a_fwd, sgmv_lora_b_fwd

    try:
        sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
        from polylora.sgmv import sgmv_lora_a_fwd as ref_a, sgmv_lora_b_fwd as ref_b
    except Exception as exc:  # noqa: BLE001
        return {"unavailable": f"reference not importable from baseline/_ref: {type(exc).__name__}: {exc}"}
    flush_w = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush_r = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    sink = torch.empty((), dtype=torch.float32, device=dev)

    def flush():
        flush_w.fill_(7)
        torch.sum(flush_r, dim=0, out=sink)

    def loop_ms(fns, reps=20):
        for _ in range(3):
            for f in fns:
                f()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            for f in fns:
                f()
        b.record()
        b.synchronize()
        return a.elapsed_time(b) / reps

    out = y.clone()
    ours = lambda: sgmv_lora_b_fwd(sgmv_lora_a_fwd(x, A, seq, wi, ranks), Bw, seq, wi, ranks, scales, out)  # noqa: E731
    theirs = lambda: ref_b(ref_a(x, A, seq, wi, ranks), Bw, seq, wi, ranks, scales, out)  # noqa: E731
    # agreement on a fresh N(0, 1) base output (the benched y has been updated in place many times)
    y = torch.randn(y.shape, device=dev, generator=torch.Generator(device=dev).manual_seed(7)).to(y.dtype)
    y_o, y_r = y.clone(), y.clone()
    sgmv_lora_b_fwd(sgmv_lora_a_fwd(x, A, seq, wi, ranks), Bw, seq, wi, ranks, scales, y_o)
    ref_b(ref_a(x, A, seq, wi, ranks), Bw, seq, wi, ranks, scales, y_r)
    torch.cuda.synchronize()
    delta = (y_r.float() - y.float()).abs().max().item()
    t_flush = loop_ms([flush])
    res = {"path": "eager sgmv_lora_a_fwd + sgmv_lora_b_fwd pair, L2 flushed before each pair",
           "max_abs_diff_over_max_delta": (y_o.float() - y_r.float()).abs().max().item() / max(delta, 1e-30)}
    for name, fn in (("triton_reference", theirs), ("ours", ours)):
        ms = loop_ms([flush, fn]) - t_flush
        res[name] = {"us_per_pair": ms * 1e3, "tokens_per_s": T_TOKENS / (ms * 1e-3)}
    res["speedup"] = res["triton_reference"]["us_per_pair"] / res["ours"]["us_per_pair"]
    import triton

    res["triton"] = triton.__version__
    del flush_w, flush_r
    return res


# ---------------------------------------------------------------- config-2 op sweep
SWEEP_T = (1, 16, 256, 4096, 16384)


def run_sweep(args):
    """BASELINE config 2 at every T of its sweep: the step (segment table +
    shrink + expand as one call) as a CUDA graph, timed back to back and with
    L2 flushed before each step (difference of graphs [flush, step] and [flush])."""
    import torch

    from polylora_b200.sgmv import build_segments, sgmv_shrink_expand

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    g = torch.Generator(device=dev).manual_seed(1000)
    ranks_np, _, scales_np = workload(seed=0)
    ranks = torch.from_numpy(ranks_np).to(dev)
    scales = torch.from_numpy(scales_np).to(dev)
    colmask = (torch.arange(MAX_RANK, device=dev)[None, :] < ranks[:, None]).float()
    A = ((torch.rand(SLOTS, K_IN, MAX_RANK, device=dev, generator=g) * 2 - 1) / 64 * colmask[:, None, :]).to(torch.bfloat16)
    Bw = (torch.randn(SLOTS, MAX_RANK, N_OUT, device=dev, generator=g) * 0.02 * colmask[:, :, None]).to(torch.bfloat16)
    flush_w = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush_r = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    sink = torch.empty((), dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    rows = []
    for T in SWEEP_T:
        rng = np.random.default_rng(T)
        wi_np = rng.integers(1, SLOTS, size=T).astype(np.int64)
        wi_np[rng.random(T) < 0.2] = 0
        wi = torch.from_numpy(wi_np).to(dev)
        seq = torch.ones(T, dtype=torch.int32, device=dev)
        x = torch.randn(T, 1, K_IN, device=dev, generator=g).to(torch.bfloat16)
        y = torch.randn(T, 1, N_OUT, device=dev, generator=g).to(torch.bfloat16)
        tmp = torch.empty(T, 1, MAX_RANK, device=dev, dtype=torch.bfloat16)

        def step():
            table = build_segments(wi, seq, ranks, 1)
            sgmv_shrink_expand(x, A, Bw, y, table, ranks, scales, tmp=tmp)

        def flush():
            flush_w.fill_(7)
            torch.sum(flush_r, dim=0, out=sink)

        def graph_of(fns):
            with torch.cuda.stream(stream):
                for _ in range(3):
                    for f in fns:
                        f()
                torch.cuda.synchronize()
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=stream):
                    for f in fns:
                        f()
                gr.replay()
            torch.cuda.synchronize()
            return gr

        def replay_ms(gr, reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                a.record(stream)
                for _ in range(reps):
                    gr.replay()
                b.record(stream)
            b.synchronize()
            return a.elapsed_time(b) / reps

        reps = max(args.steps, 20)
        g_step, g_flush, g_both = graph_of([step]), graph_of([flush]), graph_of([flush, step])
        warm = replay_ms(g_step, reps)
        cold = sorted(replay_ms(g_both, reps) - replay_ms(g_flush, reps) for _ in range(3))[1]
        _, b_s, b_e, _ = algorithmic_bytes(ranks_np, wi_np)
        rows.append({"T": T, "active_tokens": int((ranks_np[wi_np] > 0).sum()),
                     "us_per_step_back_to_back": round(warm * 1e3, 2), "us_per_step_l2_flushed": round(cold * 1e3, 2),
                     "tokens_per_s": T / (warm * 1e-3), "sgmv_gbs_l2_flushed": (b_s + b_e) / (cold * 1e-3) / 1e9})
        del x, y, tmp
    big = rows[-1]
    line = {
        "metric": METRIC, "value": big["tokens_per_s"], "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": 3, "ms_per_step": big["us_per_step_back_to_back"] / 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "BASELINE config 2 op sweep, T in {1,16,256,4096,16384}, K=N=4096, 64 slots, "
                               "max_rank 16; step = segment table + shrink + expand (one call), CUDA graph"},
        "sweep": rows,
    }
    print(json.dumps(line), flush=True)


def run_triton_compare(args):
    """The reference's own GPU path on this B200: its Triton `sgmv_lora_a_fwd` +
    `sgmv_lora_b_fwd` (src/polylora/sgmv.py:141-175, 278-328, unmodified, from
    the pip install under baseline/_ref) beside this library's operators of the
    same signatures, eager, on the config-2 sweep inputs.  Each step is the
    pair of calls as `layers.py:42-58` makes them (the reference's host syncs
    included); times are CUDA events over back-to-back steps, and with L2
    flushed before every step (loop [flush, step] minus loop [flush])."""
    import torch

    from polylora_b200.sgmv import sgmv_lora_a_fwd, sgmv_lora_b_fwd

    ref_dir = ROOT / "baseline" / "_ref"
    try:
        sys.path.insert(0, str(ref_dir))
        from polylora.sgmv import sgmv_lora_a_fwd as ref_a, sgmv_lora_b_fwd as ref_b
    except Exception as exc:  # noqa: BLE001 - reported, not fatal
        print(json.dumps({"workload": "cfg2-triton", "unavailable": f"reference not importable from {ref_dir.name}: "
                          f"{type(exc).__name__}: {exc}"}), flush=True)
        return
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    g = torch.Generator(device=dev).manual_seed(1000)
    ranks_np, _, scales_np = workload(seed=0)
    ranks = torch.from_numpy(ranks_np).to(dev)
    scales = torch.from_numpy(scales_np).to(dev)
    colmask = (torch.arange(MAX_RANK, device=dev)[None, :] < ranks[:, None]).float()
    A = ((torch.rand(SLOTS, K_IN, MAX_RANK, device=dev, generator=g) * 2 - 1) / 64 * colmask[:, None, :]).to(torch.bfloat16)
    Bw = (torch.randn(SLOTS, MAX_RANK, N_OUT, device=dev, generator=g) * 0.02 * colmask[:, :, None]).to(torch.bfloat16)
    flush_w = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush_r = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    sink = torch.empty((), dtype=torch.float32, device=dev)

    def flush():
        flush_w.fill_(7)
        torch.sum(flush_r, dim=0, out=sink)

    def loop_ms(fns, reps):
        for _ in range(3):
            for f in fns:
                f()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            for f in fns:
                f()
        b.record()
        b.synchronize()
        return a.elapsed_time(b) / reps

    rows = []
    reps = max(args.steps, 20)
    for T in SWEEP_T:
        rng = np.random.default_rng(T)
        wi_np = rng.integers(1, SLOTS, size=T).astype(np.int64)
        wi_np[rng.random(T) < 0.2] = 0
        wi = torch.from_numpy(wi_np).to(dev)
        seq = torch.ones(T, dtype=torch.int32, device=dev)
        x = torch.randn(T, 1, K_IN, device=dev, generator=g).to(torch.bfloat16)
        y0 = torch.randn(T, 1, N_OUT, device=dev, generator=g).to(torch.bfloat16)
        y = y0.clone()

        def ours():
            sgmv_lora_b_fwd(sgmv_lora_a_fwd(x, A, seq, wi, ranks), Bw, seq, wi, ranks, scales, y)

        def theirs():
            ref_b(ref_a(x, A, seq, wi, ranks), Bw, seq, wi, ranks, scales, y)

        # agreement on fresh outputs: max |difference| over the largest LoRA delta
        y_o, y_r = y0.clone(), y0.clone()
        sgmv_lora_b_fwd(sgmv_lora_a_fwd(x, A, seq, wi, ranks), Bw, seq, wi, ranks, scales, y_o)
        ref_b(ref_a(x, A, seq, wi, ranks), Bw, seq, wi, ranks, scales, y_r)
        torch.cuda.synchronize()
        delta = (y_r.float() - y0.float()).abs().max().item()
        diff = (y_o.float() - y_r.float()).abs().max().item()
        row = {"T": T, "active_tokens": int((ranks_np[wi_np] > 0).sum()),
               "max_abs_diff_over_max_delta": diff / delta if delta else diff}
        t_flush = loop_ms([flush], reps)
        for name, fn in (("triton_reference", theirs), ("ours", ours)):
            warm = loop_ms([fn], reps)
            cold = loop_ms([flush, fn], reps) - t_flush
            row[name] = {"us_back_to_back": round(warm * 1e3, 2), "us_l2_flushed": round(cold * 1e3, 2),
                         "tokens_per_s": T / (warm * 1e-3)}
        row["speedup_back_to_back"] = row["triton_reference"]["us_back_to_back"] / row["ours"]["us_back_to_back"]
        row["speedup_l2_flushed"] = row["triton_reference"]["us_l2_flushed"] / row["ours"]["us_l2_flushed"]
        rows.append(row)
        del x, y, y0, y_o, y_r
    import triton

    print(json.dumps({"workload": "cfg2-triton", "n_gpus": 1, "dtype": "bf16", "data": "synthetic",
                      "config": "BASELINE config 2 op sweep (K=N=4096, 64 slots + __base__, max_rank 16, ranks "
                                "U{0,4,8,16}, 20% base rows); step = sgmv_lora_a_fwd + sgmv_lora_b_fwd, eager",
                      "triton": triton.__version__, "sweep": rows}), flush=True)


def _graph_timer(stream):
    """(graph_of, replay_ms): capture callables as one CUDA graph after three
    eager warm-up passes; mean device time of `reps` back-to-back replays."""
    import torch

    def graph_of(fns):
        with torch.cuda.stream(stream):
            for _ in range(3):
                for f in fns:
                    f()
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                for f in fns:
                    f()
            gr.replay()
        torch.cuda.synchronize()
        return gr

    def replay_ms(gr, reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            a.record(stream)
            for _ in range(reps):
                gr.replay()
            b.record(stream)
        b.synchronize()
        return a.elapsed_time(b) / reps

    return graph_of, replay_ms


# BASELINE config 4's decode step at the op level: the seven wrapped Linears of
# one Llama-3-8B layer (in -> out features), 256 decode tokens over 128 slots of
# max_rank 64, ranks {8, 16, 32, 64}, Zipf(1.1) adapter popularity.
CFG4_LINEARS = (("q_proj", 4096, 4096), ("k_proj", 4096, 1024), ("v_proj", 4096, 1024), ("o_proj", 4096, 4096),
                ("gate_proj", 4096, 14336), ("up_proj", 4096, 14336), ("down_proj", 14336, 4096))


def run_cfg4_ops(args):
    """Shrink, expand and the combined call for each Linear shape of config 4's
    decode step, under both work splits, with L2 flushed before every launch
    (difference of graphs [flush, op] and [flush]).  Algorithmic bytes: the
    LoRA weights of the slots in the batch at their ranks, x / y rows, tmp."""
    import torch

    from polylora_b200 import _native
    from polylora_b200.sgmv import build_segments, sgmv_expand, sgmv_shrink, sgmv_shrink_expand

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    ns, R, T = CFG4_ADAPTERS, CFG4_RANK, 256
    rng = np.random.default_rng(2)
    ranks_np = rng.choice([8, 16, 32, 64], size=ns).astype(np.int32)
    pop = 1.0 / np.arange(1, ns + 1) ** 1.1
    pop /= pop.sum()
    wi_np = rng.choice(ns, size=T, p=pop).astype(np.int64)
    used = np.unique(wi_np)
    ranks = torch.from_numpy(ranks_np).to(dev)
    scales = torch.full((ns,), 2.0, device=dev)
    wi = torch.from_numpy(wi_np).to(dev)
    seq = torch.ones(T, dtype=torch.int32, device=dev)
    table = build_segments(wi, seq, ranks, 1)
    g = torch.Generator(device=dev).manual_seed(3)
    colmask = (torch.arange(R, device=dev)[None, :] < ranks[:, None]).float()
    flush_w = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush_r = torch.ones(64 << 20, dtype=torch.float32, device=dev)
    sink = torch.empty((), dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    graph_of, replay_ms = _graph_timer(stream)

    def flush():
        flush_w.fill_(7)
        torch.sum(flush_r, dim=0, out=sink)

    g_flush = graph_of([flush])
    reps = max(args.steps, 20)
    rows = []
    prev = _native.weight_split_tokens_per_sm()
    try:
        linears = [lin for lin in CFG4_LINEARS if args.linear in (None, lin[0])]
        splits = [sp for sp in (("token_split", 0), ("weight_split", 1 << 40)) if args.split in (None, sp[0])]
        for name, K, N in linears:
            A = ((torch.rand(ns, K, R, device=dev, generator=g) * 2 - 1) / 64 * colmask[:, None, :]).to(torch.bfloat16)
            Bw = (torch.randn(ns, R, N, device=dev, generator=g) * 0.02 * colmask[:, :, None]).to(torch.bfloat16)
            x = torch.randn(T, 1, K, device=dev, generator=g).to(torch.bfloat16)
            y = torch.randn(T, 1, N, device=dev, generator=g).to(torch.bfloat16)
            tmp = torch.empty(T, 1, R, device=dev, dtype=torch.bfloat16)
            rk_used = int(ranks_np[used].sum())
            b_shrink = rk_used * K * 2 + T * K * 2 + T * R * 2
            b_expand = rk_used * N * 2 + T * N * 4 + T * R * 2
            ops = {
                "shrink": (lambda: sgmv_shrink(x, A, table, ranks, out=tmp), b_shrink),
                "expand": (lambda: sgmv_expand(tmp, Bw, y, table, ranks, scales), b_expand),
                "shrink_expand": (lambda: sgmv_shrink_expand(x, A, Bw, y, table, ranks, scales, tmp=tmp),
                                  b_shrink + b_expand),
            }
            row = {"linear": name, "K": K, "N": N}
            for split, thr in splits:
                _native.weight_split_tokens_per_sm(thr)
                for op, (fn, nbytes) in ops.items():
                    g_both = graph_of([flush, fn])
                    us = sorted(replay_ms(g_both, reps) - replay_ms(g_flush, reps) for _ in range(3))[1] * 1e3
                    row[f"{split}_{op}_us"] = round(us, 2)
                    row[f"{split}_{op}_gbs"] = round(nbytes / (us * 1e-6) / 1e9, 1)
                    del g_both
            rows.append(row)
            del A, Bw, x, y, tmp
    finally:
        _native.weight_split_tokens_per_sm(prev)
    split_name = splits[-1][0]
    layer_us = sum(r[f"{split_name}_shrink_expand_us"] for r in rows)
    line = {
        "metric": METRIC, "value": T / (layer_us * 1e-6), "unit": "tokens/s", "n_gpus": 1, "steps": reps,
        "warmup": 3, "ms_per_step": layer_us / 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "BASELINE config 4 decode, op level: the 7 LoRA Linears of one Llama-3-8B layer, "
                               "256 tokens over 128 slots (max_rank 64, ranks {8,16,32,64}, Zipf(1.1)), "
                               f"{len(used)} distinct adapters; value = tokens/s through the combined calls "
                               f"({split_name}) of the Linears listed, L2 flushed before each launch"},
        "linears": rows,
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- model workloads
# DeBERTa-v3-large-shaped encoder (random init, bf16), LoRA on
# query/key/value projections and every `dense` Linear (6 per layer), 32 GPU
# slots, ranks {4, 8, 16} (a rank-0 adapter is represented by __base__ rows: the
# adapter store rejects rank 0, as the reference's does), batch 256 x 512
# right-padded with lengths U[64, 512], 25 % of rows on __base__, uniform
# popularity.  Rows are sharded over the GPUs (strong scaling of one batch)
# and the outputs all-gathered.
CFG3_ROWS, CFG3_SEQ, CFG3_SLOTS = 256, 512, 32
CFG3_TARGETS = ["query_proj", "key_proj", "value_proj", "dense"]


def _deberta_v3_large():
    from transformers import DebertaV2Config, DebertaV2Model

    cfg = DebertaV2Config(
        vocab_size=128100, hidden_size=1024, num_hidden_layers=24, num_attention_heads=16,
        intermediate_size=4096, max_position_embeddings=512, relative_attention=True,
        position_buckets=256, norm_rel_ebd="layer_norm", share_att_key=True, pos_att_type=["p2c", "c2p"],
        max_relative_positions=-1, position_biased_input=False, type_vocab_size=0, layer_norm_eps=1e-7,
        hidden_dropout_prob=0.0, attention_probs_dropout_prob=0.0,
    )
    return DebertaV2Model(cfg).eval()


def _cfg3_setup(dev):
    """BASELINE config 3 on `dev`: the wrapped DeBERTa-v3-large-shaped encoder,
    its 32 synthetic adapters and the 256 x 512 right-padded batch (seeded)."""
    import torch

    from polylora_b200 import PolyLoraConfig, PolyLoraModel
    from polylora_b200.store import CpuLayerWeights

    torch.manual_seed(0)
    torch.set_default_dtype(torch.bfloat16)
    with torch.device(dev):
        base = _deberta_v3_large()
    torch.set_default_dtype(torch.float32)
    shapes = {n: (m.in_features, m.out_features) for n, m in base.named_modules()
              if isinstance(m, torch.nn.Linear) and any(n == t or n.endswith("." + t) for t in CFG3_TARGETS)}
    model = PolyLoraModel(base, PolyLoraConfig(max_gpu_adapters=CFG3_SLOTS, max_rank=16, target_modules=CFG3_TARGETS))
    assert set(shapes) == set(model.target_module_names), "target matching differs"
    g = torch.Generator().manual_seed(1)
    rng = np.random.default_rng(2)
    ranks = rng.choice([4, 8, 16], size=CFG3_SLOTS)
    for a in range(CFG3_SLOTS):
        r = int(ranks[a])
        layers = {
            name: CpuLayerWeights(
                A=(torch.rand(k, r, generator=g) * 2 - 1) / np.sqrt(k),
                B=torch.randn(r, n, generator=g) * 0.02,
                rank=r, scale=2.0,
            )
            for name, (k, n) in shapes.items()
        }
        model.adapter_store.add_adapter(f"adapter{a}", layers, {"r": r, "lora_alpha": 2 * r})
    lens = rng.integers(64, CFG3_SEQ + 1, size=CFG3_ROWS)
    ids = [("__base__" if rng.random() < 0.25 else f"adapter{int(rng.integers(CFG3_SLOTS))}") for _ in range(CFG3_ROWS)]
    input_ids = torch.randint(0, 128100, (CFG3_ROWS, CFG3_SEQ), generator=g).to(dev)
    mask = (torch.arange(CFG3_SEQ)[None, :] < torch.from_numpy(lens)[:, None]).long().to(dev)
    return model, base, ids, input_ids, mask, int(lens.sum())


def _cfg3_row_parallel(world, rank, dev, steps, warmup):
    """The config-3 forward under RowParallel (equal rows per rank, NCCL
    all-gather of the outputs inside the timed step).  Returns tokens/s and
    the split of the step: each rank's shard forward alone (max and min over
    ranks: the load imbalance) and the all-gather alone (the collective)."""
    import torch
    import torch.distributed as dist

    from polylora_b200.rowshard import RowParallel, partition_rows

    model, _, ids, input_ids, mask, tokens = _cfg3_setup(dev)
    fn = lambda adapter_ids, **kw: model(adapter_ids=adapter_ids, **kw).last_hidden_state  # noqa: E731
    lora_fn = RowParallel(fn, row_cost=RowParallel.EQUAL_ROWS)
    bounds = partition_rows([CFG3_SEQ] * CFG3_ROWS, world, lambda n: 1)
    s0, s1 = bounds[rank]
    shard = dict(input_ids=input_ids[s0:s1], attention_mask=mask[s0:s1])

    def max_min(v):
        if world == 1:
            return v, v
        t = torch.tensor([v, -v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t[0]), -float(t[1])

    def timed(step, n):
        with torch.inference_mode():
            for _ in range(max(warmup, 2)):
                step()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(n):
                step()
            e1.record()
            e1.synchronize()
            if world > 1:
                dist.barrier()
        return e0.elapsed_time(e1) / n

    step_ms = max_min(timed(lambda: lora_fn(ids, input_ids=input_ids, attention_mask=mask), steps))[0]
    shard_max, shard_min = max_min(timed(lambda: fn(ids[s0:s1], **shard), steps))
    out = {"ms_per_forward": step_ms, "tokens_per_s": tokens / (step_ms * 1e-3),
           "padded_tokens_per_s": CFG3_ROWS * CFG3_SEQ / (step_ms * 1e-3), "non_pad_tokens": tokens,
           "shard_forward_ms_max": shard_max, "shard_forward_ms_min": shard_min, "steps": steps}
    if world > 1:
        from polylora_b200.rowshard import all_gather_rows

        local = torch.zeros(s1 - s0, CFG3_SEQ, 1024, device=dev, dtype=torch.bfloat16)
        gather_ms = max_min(timed(lambda: all_gather_rows(local, bounds), steps))[0]
        out["all_gather_ms"] = gather_ms
        out["limiter"] = ("all-gather" if gather_ms > shard_max - shard_min else "row imbalance")
    del model
    torch.cuda.empty_cache()
    return out


def run_model_cfg3(args):
    import torch
    import torch.distributed as dist

    from polylora_b200.rowshard import RowParallel

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", torch.cuda.current_device())
    model, base, ids, input_ids, mask, tokens = _cfg3_setup(dev)

    # the encoder computes every row at the padded length: balance shards by rows
    lora_fn = RowParallel(lambda adapter_ids, **kw: model(adapter_ids=adapter_ids, **kw).last_hidden_state,
                          row_cost=RowParallel.EQUAL_ROWS)
    base_fn = RowParallel(lambda adapter_ids, **kw: base(**kw).last_hidden_state, row_cost=RowParallel.EQUAL_ROWS)

    def barrier():
        if world > 1:
            dist.barrier()

    def timed(fn, steps, warmup):
        with torch.inference_mode():
            for _ in range(max(warmup, 3)):
                fn(ids, input_ids=input_ids, attention_mask=mask)
            torch.cuda.synchronize()
            barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(steps):
                fn(ids, input_ids=input_ids, attention_mask=mask)
            e1.record()
            e1.synchronize()
            barrier()
        ms = e0.elapsed_time(e1) / steps
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    gpu_ids = [v for v in visible.split(",") if v.strip().isdigit()]
    sampler = ClockSampler(int(gpu_ids[local]) if local < len(gpu_ids) else local)
    sampler.start()
    ms_lora = timed(lora_fn, args.steps, args.warmup)
    clocks = sampler.stop()
    ms_base = timed(base_fn, max(2, args.steps // 2), 2)
    if rank == 0:
        line = {
            "metric": METRIC, "value": tokens / (ms_lora * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_lora, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {
                "workload": "BASELINE config 3: DeBERTa-v3-large-shaped encoder (24 layers, hidden 1024, 16 heads, "
                            "FFN 4096), random init, bf16; LoRA on query/key/value/dense (144 Linears); 32 GPU "
                            "slots, ranks {4,8,16}, 25% __base__ rows; batch 256 x 512 right-padded, lengths "
                            "U[64,512]; one forward per step, rows sharded over the GPUs (equal rows: compute is per padded row) + all-gather",
                "non_pad_tokens": tokens, "padded_tokens": CFG3_ROWS * CFG3_SEQ,
            },
            "padded_tokens_per_s": CFG3_ROWS * CFG3_SEQ / (ms_lora * 1e-3),
            "base_model_ms_per_step": ms_base,
            "lora_overhead_frac": ms_lora / ms_base - 1.0,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# Llama-3-8B-shaped decoder (32 layers, hidden 4096, 32 query
# / 8 KV heads, FFN 14336, vocab 128256), random init, bf16; LoRA on q/k/v/o/
# gate/up/down (224 Linears); 128 adapters resident in 128 GPU slots, max_rank
# 64, ranks {8, 16, 32, 64}, Zipf(1.1) popularity.  Two steps: prefill of
# 64 x 1024 tokens and decode of 256 x 1 token (one forward each, no KV history);
# rows sharded over the GPUs (strong scaling) and the outputs all-gathered.
CFG4_ADAPTERS, CFG4_RANK = 128, 64
CFG4_TARGETS = ["q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"]


def _llama3_8b():
    from transformers import LlamaConfig, LlamaModel

    cfg = LlamaConfig(vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                      num_attention_heads=32, num_key_value_heads=8, max_position_embeddings=8192,
                      rope_theta=500000.0, use_cache=False)
    return LlamaModel(cfg).eval()


def run_model_cfg4(args):
    import torch
    import torch.distributed as dist

    from polylora_b200 import PolyLoraConfig, PolyLoraModel
    from polylora_b200.rowshard import RowParallel
    from polylora_b200.store import CpuLayerWeights

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", torch.cuda.current_device())
    torch.manual_seed(0)
    torch.set_default_dtype(torch.bfloat16)
    with torch.device(dev):
        base = _llama3_8b()
    torch.set_default_dtype(torch.float32)
    shapes = {n: (m.in_features, m.out_features) for n, m in base.named_modules()
              if isinstance(m, torch.nn.Linear) and any(n == t or n.endswith("." + t) for t in CFG4_TARGETS)}
    model = PolyLoraModel(base, PolyLoraConfig(max_gpu_adapters=CFG4_ADAPTERS, max_rank=CFG4_RANK,
                                               target_modules=CFG4_TARGETS))
    # random rank-64 factors per distinct (in, out) shape; an adapter of rank r
    # uses their first r columns / rows (values do not change the timing)
    g = torch.Generator().manual_seed(1)
    src = {}
    for k, n in set(shapes.values()):
        src[(k, n)] = ((torch.rand(k, CFG4_RANK, generator=g) * 2 - 1) / np.sqrt(k),
                       torch.randn(CFG4_RANK, n, generator=g) * 0.02)
    rng = np.random.default_rng(2)
    ranks = rng.choice([8, 16, 32, 64], size=CFG4_ADAPTERS)
    for a in range(CFG4_ADAPTERS):
        r = int(ranks[a])
        layers = {name: CpuLayerWeights(A=src[kn][0][:, :r], B=src[kn][1][:r], rank=r, scale=2.0)
                  for name, kn in shapes.items()}
        model.adapter_store.add_adapter(f"adapter{a}", layers, {"r": r, "lora_alpha": 2 * r})
    pop = 1.0 / np.arange(1, CFG4_ADAPTERS + 1) ** 1.1
    pop /= pop.sum()

    def batch(rows, seq):
        ids = [f"adapter{int(i)}" for i in rng.choice(CFG4_ADAPTERS, size=rows, p=pop)]
        input_ids = torch.randint(0, 128256, (rows, seq), generator=g).to(dev)
        mask = torch.ones(rows, seq, dtype=torch.long, device=dev)
        return ids, input_ids, mask

    def barrier():
        if world > 1:
            dist.barrier()

    def timed(fn, ids, input_ids, mask, steps, warmup):
        with torch.inference_mode():
            for _ in range(max(warmup, 2)):
                fn(ids, input_ids=input_ids, attention_mask=mask)
            torch.cuda.synchronize()
            barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(steps):
                fn(ids, input_ids=input_ids, attention_mask=mask)
            e1.record()
            e1.synchronize()
            barrier()
        ms = e0.elapsed_time(e1) / steps
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    def time_graphed_decode(model, base, ids, input_ids, steps):
        """Decode forward replayed as one CUDA graph per call (GraphedForward;
        unpadded rows, so no mask), beside the base model captured the same way."""
        from polylora_b200.graphed import GraphedForward, eager_mask_decisions

        with torch.inference_mode():
            graphed = GraphedForward(model, ids, input_ids=input_ids)
            static_ids = input_ids.clone()
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                for _ in range(2):
                    base(input_ids=static_ids)
            torch.cuda.current_stream().wait_stream(side)
            base_graph = torch.cuda.CUDAGraph()
            with eager_mask_decisions(), torch.cuda.graph(base_graph):  # as GraphedForward captures
                base(input_ids=static_ids)
            ref = model(input_ids=input_ids, adapter_ids=ids).last_hidden_state
            match = bool(torch.equal(graphed(ids, input_ids=input_ids), ref))
            out = {}
            for key, fn in (("ms_per_step", lambda: graphed(ids, input_ids=input_ids)),
                            ("base_model_ms_per_step", base_graph.replay)):
                for _ in range(3):
                    fn()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(steps):
                    fn()
                e1.record()
                e1.synchronize()
                out[key] = e0.elapsed_time(e1) / steps
            del base_graph, graphed
        out["tokens_per_s"] = input_ids.numel() / (out["ms_per_step"] * 1e-3)
        out["lora_overhead_frac"] = out["ms_per_step"] / out["base_model_ms_per_step"] - 1.0
        out["equals_eager_forward"] = match
        return out

    lora_fn = RowParallel(lambda adapter_ids, **kw: model(adapter_ids=adapter_ids, **kw).last_hidden_state)
    base_fn = RowParallel(lambda adapter_ids, **kw: base(**kw).last_hidden_state)
    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    gpu_ids = [v for v in visible.split(",") if v.strip().isdigit()]
    sampler = ClockSampler(int(gpu_ids[local]) if local < len(gpu_ids) else local)
    res = {}
    sampler.start()
    phases = (("prefill", 64, 1024), ("decode", 256, 1))
    if args.workload == "cfg4-decode":
        phases = phases[1:]
    for name, rows, seq in phases:
        ids, input_ids, mask = batch(rows, seq)
        ms = timed(lora_fn, ids, input_ids, mask, args.steps, args.warmup)
        ms_base = timed(base_fn, ids, input_ids, mask, max(2, args.steps // 2), 2)
        res[name] = {"rows": rows, "seq": seq, "tokens": rows * seq, "distinct_adapters": len(set(ids)),
                     "ms_per_step": ms, "tokens_per_s": rows * seq / (ms * 1e-3),
                     "base_model_ms_per_step": ms_base, "lora_overhead_frac": ms / ms_base - 1.0}
        if name == "decode" and world == 1:
            res[name]["graphed"] = time_graphed_decode(model, base, ids, input_ids, args.steps)
    clocks = sampler.stop()
    if rank == 0:
        pre = res.get("prefill") or res["decode"]
        line = {
            "metric": METRIC, "value": pre["tokens_per_s"], "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": pre["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {
                "workload": "BASELINE config 4: Llama-3-8B-shaped decoder (32 layers, hidden 4096, 32/8 heads, FFN "
                            "14336), random init, bf16; LoRA on q/k/v/o/gate/up/down (224 Linears); 128 adapters "
                            "in 128 GPU slots, max_rank 64, ranks {8,16,32,64}, Zipf(1.1) popularity; value = "
                            "prefill 64 x 1024 tokens/s; decode 256 x 1 below; rows sharded over the GPUs + "
                            "all-gather" if "prefill" in res else
                            "BASELINE config 4 decode leg only: 256 x 1 tokens/s (Llama-3-8B-shaped, 128 adapters, "
                            "max_rank 64, Zipf(1.1))",
            },
            **res, "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# adapter churn on a DeBERTa-v3-small-shaped encoder (6
# layers, hidden 768, 12 heads, FFN 3072; bf16, random init), LoRA on
# query/key/value/dense.  A catalog of 1024 PEFT adapters (ranks {8, 16},
# alpha 2r) sits on the disk tier, the CPU LRU holds 256 and the GPU 32 slots;
# each batch is 128 rows x 256 tokens with adapter ids Zipf(0.9) over the
# catalog, so slots are evicted and refilled (and CPU misses parsed from disk)
# in every batch.  A batch carries ~88 distinct adapters, more than the 32
# slots (the reference raises there), so each rank serves its rows as
# micro-batches of <= 32 distinct adapters.
CFG5_CATALOG, CFG5_SLOTS, CFG5_CPU, CFG5_ROWS, CFG5_SEQ = 1024, 32, 256, 128, 256


def _deberta_v3_small():
    from transformers import DebertaV2Config, DebertaV2Model

    cfg = DebertaV2Config(
        vocab_size=128100, hidden_size=768, num_hidden_layers=6, num_attention_heads=12,
        intermediate_size=3072, max_position_embeddings=512, relative_attention=True,
        position_buckets=256, norm_rel_ebd="layer_norm", share_att_key=True, pos_att_type=["p2c", "c2p"],
        max_relative_positions=-1, position_biased_input=False, type_vocab_size=0, layer_norm_eps=1e-7,
        hidden_dropout_prob=0.0, attention_probs_dropout_prob=0.0,
    )
    return DebertaV2Model(cfg).eval()


def run_model_cfg5(args):
    import torch
    import torch.distributed as dist
    from safetensors.torch import save_file

    from polylora_b200 import PolyLoraConfig, PolyLoraModel
    from polylora_b200.rowshard import RowParallel
    from polylora_b200.store import _entry_dirname

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", torch.cuda.current_device())
    torch.manual_seed(0)
    torch.set_default_dtype(torch.bfloat16)
    with torch.device(dev):
        base = _deberta_v3_small()
    torch.set_default_dtype(torch.float32)
    shapes = {n: (m.in_features, m.out_features) for n, m in base.named_modules()
              if isinstance(m, torch.nn.Linear) and any(n == t or n.endswith("." + t) for t in CFG3_TARGETS)}
    disk_dir = Path(tempfile.mkdtemp(prefix=f"plora_cfg5_r{rank}_"))
    model = PolyLoraModel(base, PolyLoraConfig(
        max_gpu_adapters=CFG5_SLOTS, max_rank=16, target_modules=CFG3_TARGETS,
        max_cpu_adapters=CFG5_CPU, disk_cache_dir=disk_dir, prefetch_workers=args.prefetch_workers))
    assert set(shapes) == set(model.target_module_names), "target matching differs"
    store = model.adapter_store
    # catalog: PEFT directories written where the disk tier keeps them (no copy);
    # adapters share random factors per shape (values do not change the timing)
    g = torch.Generator().manual_seed(1)
    src = {kn: ((torch.rand(16, kn[0], generator=g) * 2 - 1) / np.sqrt(kn[0]),
                torch.randn(kn[1], 16, generator=g) * 0.02) for kn in set(shapes.values())}
    rng = np.random.default_rng(5)
    ranks = rng.choice([8, 16], size=CFG5_CATALOG)
    t_setup = time.perf_counter()
    for a in range(CFG5_CATALOG):
        aid, r = f"adapter{a}", int(ranks[a])
        path = disk_dir / _entry_dirname(aid)
        path.mkdir(parents=True, exist_ok=True)
        (path / "adapter_config.json").write_text(json.dumps(
            {"peft_type": "LORA", "r": r, "lora_alpha": 2 * r, "lora_dropout": 0.0,
             "target_modules": CFG3_TARGETS}))
        sd = {}
        for name, kn in shapes.items():
            sd[f"base_model.model.{name}.lora_A.weight"] = src[kn][0][:r].to(torch.bfloat16).contiguous()
            sd[f"base_model.model.{name}.lora_B.weight"] = src[kn][1][:, :r].to(torch.bfloat16).contiguous()
        save_file(sd, str(path / "adapter_model.safetensors"))
        store.disk_cache.add_adapter(aid, path)
    t_setup = time.perf_counter() - t_setup
    disk_loads = [0]
    load_from_disk = store._load_adapter_from_disk_cache

    def counting_load(aid):
        disk_loads[0] += 1
        return load_from_disk(aid)

    store._load_adapter_from_disk_cache = counting_load
    pop = 1.0 / np.arange(1, CFG5_CATALOG + 1) ** 0.9
    pop /= pop.sum()

    def make_batch():
        ids = [f"adapter{int(i)}" for i in rng.choice(CFG5_CATALOG, size=CFG5_ROWS, p=pop)]
        input_ids = torch.randint(0, 128100, (CFG5_ROWS, CFG5_SEQ), generator=g).to(dev)
        return ids, input_ids

    micro_batches = [0]
    # attribution of a batch's time (timed pass with prefetch, this rank): host
    # seconds in the slot policy (CPU-tier gets, disk loads left on the critical
    # path, refill issue) and device time of each micro-batch forward (events
    # around the base model call, after the policy; includes waits for refills)
    attrib = {"on": False, "host_s": 0.0, "fwd": []}
    prepare = model.prepare_lora_context

    def timed_prepare(*a, **k):
        t = time.perf_counter()
        try:
            return prepare(*a, **k)
        finally:
            if attrib["on"]:
                attrib["host_s"] += time.perf_counter() - t

    model.prepare_lora_context = timed_prepare
    inner_forward = base.forward

    def timed_forward(*a, **k):
        if not attrib["on"]:
            return inner_forward(*a, **k)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        out = inner_forward(*a, **k)
        e1.record()
        attrib["fwd"].append((e0, e1))
        return out

    base.forward = timed_forward

    def groups_of(adapter_ids):
        order = list(dict.fromkeys(adapter_ids))
        for i in range(0, len(order), CFG5_SLOTS):
            group = set(order[i:i + CFG5_SLOTS])
            yield [j for j, a in enumerate(adapter_ids) if a in group]

    def serve(adapter_ids, input_ids):
        """This rank's rows as micro-batches of <= 32 distinct adapters (in order of first use)."""
        out = torch.empty(input_ids.shape + (768,), device=dev, dtype=torch.bfloat16)
        for rows in groups_of(adapter_ids):
            idx = torch.tensor(rows, device=dev)
            res = model(input_ids=input_ids.index_select(0, idx), adapter_ids=[adapter_ids[j] for j in rows])
            out.index_copy_(0, idx, res.last_hidden_state)
            micro_batches[0] += 1
        return out

    lora_fn = RowParallel(lambda adapter_ids, input_ids: serve(adapter_ids, input_ids), row_cost=RowParallel.EQUAL_ROWS)

    def step(ids, x):
        return lora_fn(ids, input_ids=x)
    nw = max(args.warmup, 3)
    batches = [make_batch() for _ in range(2 * (nw + args.steps))]
    cache = model.adapter_cache

    def barrier():
        if world > 1:
            dist.barrier()

    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    gpu_ids = [v for v in visible.split(",") if v.strip().isdigit()]
    sampler = ClockSampler(int(gpu_ids[local]) if local < len(gpu_ids) else local)
    def run_pass(seq, prefetch, attribute=False):
        """Warm-up then timed batches; with `prefetch`, each step first queues the
        next batch's adapters for the CPU tier's prefetch thread (this rank's rows).
        With `attribute`, the timed batches feed `attrib`."""
        def my_ids(ids):
            lo, hi = len(ids) * rank // world, len(ids) * (rank + 1) // world
            return ids[lo:hi]

        for i, (ids, x) in enumerate(seq[:nw]):
            if prefetch and i + 1 < len(seq):
                model.prefetch(my_ids(seq[i + 1][0]))
            step(ids, x)
        torch.cuda.synchronize()
        barrier()
        st0, ld0, mbs0 = dict(cache.stats), disk_loads[0], micro_batches[0]
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        attrib["on"] = attribute
        for i, (ids, x) in enumerate(seq[nw:], start=nw):
            if prefetch and i + 1 < len(seq):
                model.prefetch(my_ids(seq[i + 1][0]))
            step(ids, x)
        attrib["on"] = False
        e1.record()
        e1.synchronize()
        store.wait_prefetches()
        barrier()
        return e0.elapsed_time(e1) / args.steps, st0, ld0, mbs0

    with torch.inference_mode():
        ms_nopf, _, _, _ = run_pass(batches[: nw + args.steps], prefetch=False)
        sampler.start()
        ms, stats0, loads0, mb0 = run_pass(batches[nw + args.steps:], prefetch=True, attribute=True)
        clocks = sampler.stop()
        fwd_ms = sum(a.elapsed_time(b) for a, b in attrib["fwd"]) / args.steps
        # the last batch's micro-batches again, each right after a first run that made
        # its adapters resident: the forwards without refills or policy misses
        ids, x = batches[-1]
        n = x.shape[0]
        lo, hi = n * rank // world, n * (rank + 1) // world
        my_ids_, my_x = ids[lo:hi], x[lo:hi]
        resident_ms = 0.0
        for rows in groups_of(my_ids_):
            sub_ids = [my_ids_[j] for j in rows]
            sub_x = my_x.index_select(0, torch.tensor(rows, device=dev))
            model(input_ids=sub_x, adapter_ids=sub_ids)
            torch.cuda.synchronize()
            attrib["on"], attrib["fwd"] = True, []
            model(input_ids=sub_x, adapter_ids=sub_ids)
            attrib["on"] = False
            torch.cuda.synchronize()
            resident_ms += sum(a.elapsed_time(b) for a, b in attrib["fwd"])
        # the same batches through the base model alone
        torch.cuda.synchronize()
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b0.record()
        for ids, x in batches[-args.steps:]:
            n = x.shape[0]
            lo, hi = n * rank // world, n * (rank + 1) // world
            base(input_ids=x[lo:hi])
        b1.record()
        b1.synchronize()
        ms_base = b0.elapsed_time(b1) / args.steps
    if world > 1:
        t = torch.tensor([ms, ms_base, ms_nopf], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_base, ms_nopf = float(t[0]), float(t[1]), float(t[2])
    delta = {k: cache.stats[k] - stats0[k] for k in cache.stats}
    shutil.rmtree(disk_dir, ignore_errors=True)
    if rank == 0:
        tokens = CFG5_ROWS * CFG5_SEQ
        line = {
            "metric": METRIC, "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {
                "workload": "BASELINE config 5: adapter churn, DeBERTa-v3-small-shaped encoder (6 layers, hidden "
                            "768, 12 heads, FFN 3072), bf16, random init; LoRA on query/key/value/dense (36 "
                            "Linears); 1024-adapter PEFT catalog (ranks {8,16}) on the disk tier, CPU LRU 256, "
                            "32 GPU slots; batches 128 x 256 tokens, adapter ids Zipf(0.9); one batch per step "
                            "(rank 0's stats), rows sharded over the GPUs, micro-batches of <= 32 distinct adapters; "
                            f"value with the next batch's adapters prefetched from disk on the CPU tier's "
                            f"{args.prefetch_workers} worker thread(s)",
            },
            "ms_per_step_without_prefetch": ms_nopf,
            "tokens_per_s_without_prefetch": CFG5_ROWS * CFG5_SEQ / (ms_nopf * 1e-3),
            "per_step_rank0": {
                "micro_batches": (micro_batches[0] - mb0) / args.steps,
                "gpu_slot_misses": delta["misses"] / args.steps, "gpu_slot_hits": delta["hits"] / args.steps,
                "evictions": delta["evictions"] / args.steps,
                "refill_h2d_MB": delta["h2d_bytes"] / args.steps / 1e6,
                "disk_loads": (disk_loads[0] - loads0) / args.steps,
            },
            "attribution_rank0_ms_per_step": {
                "slot_policy_host": attrib["host_s"] * 1e3 / args.steps,
                "micro_batch_forwards_device": fwd_ms,
                "micro_batch_forwards_device_resident": resident_ms,
                "device_idle_or_between_forwards": ms - fwd_ms,
                "note": "slot_policy_host: host time in the slot policy (CPU-tier gets, disk loads on the "
                        "critical path, refill issue); micro_batch_forwards_device: events around each "
                        "micro-batch's base-model call (LoRA kernels included, and waits for its refills); "
                        "_resident: the last batch's micro-batches re-run with their adapters resident; "
                        "device_idle_or_between_forwards: the step minus the forwards",
            },
            "catalog_setup_s": t_setup,
            "base_model_ms_per_step": ms_base, "lora_overhead_frac": ms / ms_base - 1.0,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_profile(args):
    """A small case for ncu: the config-2 inputs (x and y 128 MiB each, larger
    than L2), three steps of segment table + combined shrink/expand call as
    plain launches, then the shrink and the expand operators once each.
    Prints the kernel-source digest the capture describes."""
    import torch

    from polylora_b200.sgmv import build_segments, sgmv_expand, sgmv_shrink, sgmv_shrink_expand

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    ranks_np, wi_np, scales_np = workload(seed=0)
    g = torch.Generator(device=dev).manual_seed(1000)
    ranks = torch.from_numpy(ranks_np).to(dev)
    colmask = (torch.arange(MAX_RANK, device=dev)[None, :] < ranks[:, None]).float()
    A = ((torch.rand(SLOTS, K_IN, MAX_RANK, device=dev, generator=g) * 2 - 1) / 64 * colmask[:, None, :]).to(torch.bfloat16)
    Bw = (torch.randn(SLOTS, MAX_RANK, N_OUT, device=dev, generator=g) * 0.02 * colmask[:, :, None]).to(torch.bfloat16)
    scales = torch.from_numpy(scales_np).to(dev)
    wi = torch.from_numpy(wi_np).to(dev)
    seq = torch.ones(T_TOKENS, dtype=torch.int32, device=dev)
    x = torch.randn(T_TOKENS, 1, K_IN, device=dev, generator=g).to(torch.bfloat16)
    y = torch.randn(T_TOKENS, 1, N_OUT, device=dev, generator=g).to(torch.bfloat16)
    tmp = torch.empty(T_TOKENS, 1, MAX_RANK, device=dev, dtype=torch.bfloat16)
    for _ in range(3):
        table = build_segments(wi, seq, ranks, 1)
        sgmv_shrink_expand(x, A, Bw, y, table, ranks, scales, tmp=tmp)
    # then the two operators apart (the standalone stream shrink and expand), once each
    sgmv_shrink(x, A, table, ranks, out=tmp)
    sgmv_expand(tmp, Bw, y, table, ranks, scales)
    torch.cuda.synchronize()
    print(json.dumps({"workload": "profile", "kernel_source_sha256": kernel_source_digest(),
                      "active_tokens": int((ranks_np[wi_np] > 0).sum())}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["cfg2", "profile", "cfg2-sweep", "cfg2-triton", "cfg3", "cfg4", "cfg4-decode",
                                           "cfg4-ops", "cfg5"],
                    default="cfg2",
                    help="cfg2: the SGMV op step (default, the headline line); cfg3: model forward")
    ap.add_argument("--prefetch-workers", type=int, default=1,
                    help="cfg5: worker threads of the CPU tier's prefetch of queued batches")
    ap.add_argument("--linear", default=None, help="cfg4-ops: only this Linear (e.g. gate_proj)")
    ap.add_argument("--split", choices=["token_split", "weight_split"], default=None,
                    help="cfg4-ops: only this work split")
    args = ap.parse_args()
    if args.workload == "profile" and args.impl != "reference":
        run_profile(args)
    elif args.workload == "cfg2-sweep" and args.impl != "reference":
        run_sweep(args)
    elif args.workload == "cfg2-triton" and args.impl != "reference":
        run_triton_compare(args)
    elif args.workload == "cfg4-ops" and args.impl != "reference":
        run_cfg4_ops(args)
    elif args.workload in ("cfg3", "cfg4", "cfg4-decode", "cfg5"):
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": f"{args.workload} is timed for this library "
                              "only; the reference arm covers the config-2 op"}), flush=True)
        elif args.workload == "cfg3":
            run_model_cfg3(args)
        elif args.workload == "cfg5":
            run_model_cfg5(args)
        else:
            run_model_cfg4(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
