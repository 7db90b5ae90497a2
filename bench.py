#!/usr/bin/env python
"""Benchmark of the EmbeddingGemma encoder path on N B200s.

Metric: EmbeddingGemma embeddings/s at 256×512 tokens.
Workload: benchmark config 2 — the EmbeddingGemma-300m-shaped encoder with
random-init weights (seed 0, bf16 widened to fp32) on a batch of 256
sequences × 512 tokens, all full length, ids from seed 1. A step is one
forward of that batch (ids → L2-normalised 768-d embeddings) on every GPU,
plus the NCCL gather of the embeddings onto rank 0 when N > 1. By default
each GPU is an independent replica with its own 256×512 batch (weak
scaling, no collective on the data path besides that gather);
--global-batch G splits one G-sequence batch into contiguous per-GPU
slices instead (strong scaling: G = 256 is the 8-GPU target point, and
--batch 32 --seq 2048 --global-batch 32 is config 5).

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
       [--precision split|split_tf32|tf32] [--checkpoint bf16|f32] [--global-batch G]
       [--workload encoder|ragged|eg2|cluster|matmul]
(N > 1 under torchrun). Rank 0 prints one JSON line.

--impl reference times the reference's CPU path on this host: the Go
reference cannot be built here (no Go toolchain), so the CPU restatement
in oracle/ (float32 arithmetic of the reference, all host threads) stands
in for it on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "EmbeddingGemma embeddings/s at 256×512 tok, 1/2/4/8 B200; % TC/HBM roofline"
UNIT = "embeddings/s"
BATCH, SEQ = 256, 512
CPU_SAMPLE_SEQS = 4  # sequences of 512 tokens per CPU-baseline step


def model_work(cfg: dict, T: int):
    """Algorithmic FLOPs of one sequence of T tokens (all valid)."""
    H, F, D = cfg["hidden_size"], cfg["intermediate_size"], cfg["head_dim"]
    Hq, Hkv, L = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["num_hidden_layers"]
    linear = 2 * (H * Hq * D + 2 * H * Hkv * D + Hq * D * H + 3 * H * F) * L * T
    w = cfg["sliding_window"] // 2 + 1
    i = np.arange(T)
    local_pairs = int(np.sum(np.minimum(T - 1, i + w - 1) - np.maximum(0, i - w + 1) + 1)) if T > w else T * T
    glob = sum(1 for l in range(L) if (l + 1) % 6 == 0)
    attn = 4 * Hq * D * (glob * T * T + (L - glob) * local_pairs)
    head = 2 * (768 * 3072 + 3072 * 768)
    return linear, attn, head


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16": d["bf16_tflops"],
                "bf16_sustained": d["bf16_tflops_sustained"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


def host_cpu() -> dict:
    """Host CPU model name and core counts (lscpu), for the CPU baseline."""
    info = {"model_name": None, "cpus": os.cpu_count()}
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        for line in out.splitlines():
            k, _, v = line.partition(":")
            k, v = k.strip(), v.strip()
            if k == "Model name":
                info["model_name"] = v
            elif k in ("Core(s) per socket", "Socket(s)", "Thread(s) per core"):
                info[k.lower().replace("(s)", "s").replace(" ", "_")] = int(v)
    except (OSError, ValueError, subprocess.SubprocessError):
        pass
    return info


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.lines = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", ",".join(str(g) for g in self.gpus)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "power_w_max": max(power) if power else None,
                "samples": len(sm), "reasons": sorted(reasons)}


def cpu_time_sample(cfg, w32, ids, lengths, threads):
    from oracle import oracle as O

    om = O.OracleModel(cfg, w32)
    t0 = time.perf_counter()
    om.embed_padded(ids, lengths, mode=O.F32, threads=threads)
    return time.perf_counter() - t0


def f32_weights(w):
    from ai_b200.synthetic import bf16_to_f32

    return {k: bf16_to_f32(v) for k, v in w.items()}


def run_reference(args, rank, world, cfg):
    """Reference arm: the CPU path on this host's cores (rank 0 only)."""
    if rank != 0:
        return
    from ai_b200 import synthetic as S

    threads = os.cpu_count() or 1
    w = f32_weights(S.make_weights(cfg, seed=0))
    ids = S.make_ids(CPU_SAMPLE_SEQS, SEQ, 1)
    lengths = np.full(CPU_SAMPLE_SEQS, SEQ, np.int32)
    for _ in range(args.warmup):
        cpu_time_sample(cfg, w, ids, lengths, threads)
    times = [cpu_time_sample(cfg, w, ids, lengths, threads) for _ in range(args.steps)]
    per_step = sum(times) / len(times)
    value = CPU_SAMPLE_SEQS / per_step
    sample = (f"{CPU_SAMPLE_SEQS} sequences x {SEQ} tokens of config 2 per step "
              f"(same weights and ids seed), oracle float32 mode = the reference's arithmetic")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: random-init weights seed 0 (bf16), ids seed 1",
        "config": {"workload": "config 2: 256 x 512 tokens, all full length (CPU: bounded sample)",
                   "seq_len": SEQ, "parallelism": "host threads"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "host_cpu": host_cpu(), "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "Go reference unbuildable here (no Go toolchain on this box or the GPU box); "
                "timed CPU restatement of its float32 path",
    }
    print(json.dumps(line), flush=True)


PREC_NAMES = {"split": "split_fp16", "split_tf32": "split_tf32", "tf32": "tf32"}


def prec_code(gemma, name: str) -> int:
    return {"split": gemma.PREC_SPLIT, "split_tf32": gemma.PREC_SPLIT_TF32, "tf32": gemma.PREC_TF32}[name]


def rank_slice(total: int, world: int, rank: int):
    """Contiguous [start, stop) of `total` sequences for `rank`, sizes within one."""
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def run_ours(args, rank, local_rank, world, cfg):
    import torch
    import torch.distributed as dist

    from ai_b200 import gemma
    from ai_b200 import synthetic as S

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    prec = prec_code(gemma, args.precision)
    if args.checkpoint == "f32":
        w = S.make_weights_f32(cfg, seed=0, norm_std=args.norm_std)
    else:
        w = S.make_weights(cfg, seed=0, norm_std=args.norm_std)
    opts = [gemma.WeightsBF16()] if args.weights == "bf16" else []
    strong = args.global_batch is not None
    if strong:
        # the fixed global batch (ids seed 1) cut into contiguous per-rank slices
        lo, hi = rank_slice(args.global_batch, world, rank)
        ids_np = S.make_ids(args.global_batch, SEQ, 1)[lo:hi]
        if world > 1 and args.global_batch % world != 0:
            raise SystemExit("--global-batch must be a multiple of the number of GPUs")
    else:
        # replicas: each rank embeds its own batch
        ids_np = S.make_ids(BATCH, SEQ, 1 if rank == 0 else 1000 + rank)
    nb = ids_np.shape[0]
    model = gemma.from_synthetic(cfg, w, device=local_rank, max_batch_tokens=nb * SEQ, options=opts)
    dim = model.Dim()
    len_np = np.full(nb, SEQ, np.int32)
    d_ids = torch.from_numpy(ids_np).to(dev)
    d_len = torch.from_numpy(len_np).to(dev)
    out = torch.empty((nb, dim), dtype=torch.float32, device=dev)
    # the embeddings meet on rank 0 in one NCCL gather per step (the only
    # collective of the multi-GPU path)
    gathered = [torch.empty_like(out) for _ in range(world)] if (world > 1 and rank == 0) else None
    stream = torch.cuda.current_stream(dev)
    ev = []  # per timed step: (forward start, forward end, gather end)

    def step(record=False):
        if record:
            e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            e[0].record(stream)
        model.embed_device(d_ids, d_len, nb, SEQ, dim, out, stream, prec)
        if record:
            e[1].record(stream)
        if world > 1:
            dist.gather(out, gathered, dst=0)
        if record:
            e[2].record(stream)
            ev.append(e)

    def sync_all():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
            torch.cuda.synchronize(dev)

    for _ in range(max(args.warmup, 3)):
        step()
    model.check()
    model.read_profile()  # discard warm-up counts

    # ---- device-timed value (inputs resident in HBM): exactly K steps of
    # the production path (the forward replayed from its CUDA graph, no
    # per-launch events)
    sampler = ClockSampler(list(range(world)) if rank == 0 else [])
    sync_all()
    if rank == 0:
        sampler.start()
        time.sleep(0.5)
    model.read_profile()  # discard earlier counts
    sync_all()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step(record=True)
    e1.record(stream)
    sync_all()
    ms = e0.elapsed_time(e1)
    timed_launches = sum(v["launches"] for v in model.read_profile().values())
    # ---- per-phase device time of another K steps (CUDA-event pairs around
    # every launch, which run the forward eagerly): the roofline and the
    # phase split
    model.set_profiling(True)
    for _ in range(args.steps):
        step()
    sync_all()
    model.set_profiling(False)
    prof = model.read_profile()
    fwd_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / len(ev)
    gather_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / len(ev)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    per_rank = torch.tensor([fwd_ms, gather_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        parts = [torch.zeros_like(per_rank) for _ in range(world)]
        dist.all_gather(parts, per_rank)
        per_rank_all = [[round(float(x), 3) for x in q.tolist()] for q in parts]
    else:
        per_rank_all = [[round(fwd_ms, 3), round(gather_ms, 3)]]
    ms_max = float(t.item())
    per_step_s = ms_max / 1e3 / args.steps
    total_seqs = args.global_batch if strong else world * BATCH
    value = total_seqs / per_step_s

    # ---- five windows of at least 1 s each (3 warm-ups above), median
    win_steps = max(args.steps, int(math.ceil(1.0 / per_step_s)))
    windows = []
    for _ in range(args.windows):
        sync_all()
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(win_steps):
            step()
        a1.record(stream)
        sync_all()
        tw = torch.tensor([a0.elapsed_time(a1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(tw, op=dist.ReduceOp.MAX)
        windows.append(total_seqs * win_steps / (float(tw.item()) / 1e3))
    clocks = sampler.stop() if rank == 0 else None
    model.check()

    # ---- end to end through the public host API (pinned host buffers)
    ids_pin = torch.from_numpy(ids_np).pin_memory().numpy()
    len_pin = torch.from_numpy(len_np).pin_memory().numpy()
    out_pin = torch.empty((nb, dim), dtype=torch.float32).pin_memory().numpy()
    host_res = torch.empty((nb, dim), dtype=torch.float32, device=dev)
    g2 = [torch.empty_like(host_res) for _ in range(world)] if (world > 1 and rank == 0) else None

    def e2e_step():
        model.embed_padded(ids_pin, len_pin, dim, prec, out=out_pin)
        if world > 1:
            host_res.copy_(torch.from_numpy(out_pin), non_blocking=False)
            dist.gather(host_res, g2, dst=0)
            if rank == 0:
                torch.cat(g2).cpu()

    e2e_step()
    sync_all()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    sync_all()
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = total_seqs * args.steps / float(te.item())

    # ---- roofline of the dominant kernel family (the tcgen05 GEMM)
    pk = peaks()
    linear, attn, head = model_work(cfg, SEQ)
    gemm_phases = ["gemm_qkv", "gemm_o", "gemm_gate_up", "gemm_down"]
    gemm_ms = sum(prof[p]["ms"] for p in gemm_phases)
    gemm_launches = sum(prof[p]["launches"] for p in gemm_phases)
    gemm_flops = linear * nb * args.steps
    tf32_peak = pk["bf16_sustained"] / 2.0
    achieved = gemm_flops / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else None
    # split-fp16: bf16-checkpoint projections have an exact fp16 form (two
    # passes; non-zero norm gains go on A); an fp32 checkpoint's come in two
    # fp16 parts (three passes: A_hi·B_hi, A_hi·B_lo, A_lo·B_hi)
    h16 = prec == gemma.PREC_SPLIT
    if h16:
        arith, passes = ("split_fp16", 2) if args.checkpoint == "bf16" else ("split_fp16_b2", 3)
    elif prec == gemma.PREC_TF32:
        arith, passes = "tf32", 1
    else:
        lo_b = args.checkpoint == "f32" or args.norm_std > 0
        arith, passes = "split_tf32", (3 if lo_b else 2)
    traffic = None
    tp = ROOT / "profiles" / "gemm_traffic.json"
    if tp.exists() and h16 and args.checkpoint == "bf16":
        traffic = json.loads(tp.read_text()).get("bytes_per_launch")
    peak = pk["bf16_sustained"] if h16 else tf32_peak
    roofline = {
        "bound": "tensor",
        "kernel": (f"gemm_pair_kernel (tcgen05 cta_group::2 kind::f16 {arith}, all encoder projections)" if h16 else
                   f"gemm_pair_kernel (tcgen05 cta_group::2 kind::tf32 {arith}, all encoder projections)"),
        "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
        "frac": achieved / peak if achieved else None, "traffic": traffic,
        "traffic_source": ("profiles/gemm_traffic.json: ncu dram bytes of the four encoder GEMMs at batch 64, "
                           "scaled x4 to a 256-sequence launch (traffic grows with M)") if traffic else None,
        "peak_source": (f"{pk['source']} bf16 sustained {pk['bf16_sustained']} TFLOP/s "
                        + ("(dense fp16 runs at the bf16 rate)" if h16 else "/ 2 (dense TF32 runs at half the bf16 rate)")),
        "issued_mma_passes": passes,
        "issued_frac": (achieved * passes / peak) if achieved else None,
        "frac_of_tf32_peak": achieved / tf32_peak if achieved else None,
        "launches": gemm_launches,
    }
    phases = {p: round(v["ms"] / args.steps, 3) for p, v in prof.items()}
    attn_ms = prof["attention"]["ms"]
    launches_total = timed_launches  # the library's kernels launched in the timed K steps

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            w32 = w if args.checkpoint == "f32" else f32_weights(w)
            ids_s = ids_np[:CPU_SAMPLE_SEQS]
            secs = cpu_time_sample(cfg, w32, ids_s, len_np[:CPU_SAMPLE_SEQS], threads)
            cpu = {"value": CPU_SAMPLE_SEQS / secs, "unit": UNIT, "cores": threads, "kind": "port",
                   "host_cpu": host_cpu(),
                   "sample": f"{CPU_SAMPLE_SEQS} sequences x {SEQ} tokens of the same workload, oracle "
                             "float32 mode (the reference's arithmetic, packed AVX-512 GEMM), one pass; "
                             "CPU restatement, not the reference binary"}
        if strong:
            workload = (f"global batch {args.global_batch} sequences x {SEQ} tokens, all full length, "
                        f"split over {world} GPU(s): {nb} per GPU")
        else:
            workload = f"config 2: {BATCH} sequences x {SEQ} tokens per GPU, all full length"
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "strong" if strong else "weak", "vs_baseline": None,
            "dtype": "f32",
            "data": ("synthetic: random-init EmbeddingGemma-300m-shaped weights (seed 0, "
                     + ("fp32, not bf16-exact" if args.checkpoint == "f32" else "bf16 widened to fp32")
                     + "), ids uniform in [3, 262144) seed 1, BOS first"),
            "config": {"workload": workload,
                       "global_batch": total_seqs, "seq_len": SEQ,
                       "parallelism": (f"{world} GPUs, contiguous slices of the batch + NCCL gather of "
                                       "embeddings onto rank 0" if strong else
                                       f"replicas x{world} + NCCL gather of embeddings onto rank 0")
                       if world > 1 else "single GPU",
                       "precision": arith,
                       "precision_requested": args.precision,
                       "checkpoint": args.checkpoint,
                       "weights_resident": args.weights,
                       "norm_std": args.norm_std,
                       "weight_bytes": model.weight_bytes(),
                       "l2_flush": "none: inputs larger than L2 (weights 0.7-1.2 GB, activations > 1 GB per step)"},
            "tokens_per_s": value * SEQ,
            "windows": {"steps_per_window": win_steps, "values": [round(v, 1) for v in windows],
                        "median": statistics.median(windows) if windows else None,
                        "rule": "3+ warm-ups, windows of >= 1 s, median of 5 (device time, max over ranks)"},
            "per_rank_ms": {"forward_and_gather": per_rank_all,
                            "note": "per GPU: [forward ms, gather ms] per step, CUDA events on the step's stream"},
            "attention_tflops": (attn * nb * args.steps / (attn_ms / 1e3) / 1e12) if attn_ms else None,
            "clocks": clocks,
            "e2e": {"value": e2e_value, "unit": UNIT,
                    "h2d_bytes_per_step": int(ids_np.nbytes + len_np.nbytes),
                    "d2h_bytes_per_step": int(nb * dim * 4)},
            "gpu_launches": int(launches_total),
            "roofline": roofline,
            "phases_ms_per_step": phases,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_ragged(args, rank, local_rank, world, cfg):
    """--workload ragged: benchmark config 3 — 8192 sequences, lengths
    uniform in [16, 2048] (seed 2) — end to end through the public API on
    host buffers: each rank embeds its cost-balanced contiguous slice of the
    length-sorted batch with Model.embed_ids (fg_embed_many: greedy batches
    under BatchTokens, packing and copies overlapped with the forward) and
    the embeddings meet on rank 0 in one NCCL gather (replicas.py). A step
    is the whole 8192-sequence batch; timed on the host around the
    synchronous calls, max over ranks."""
    import torch
    import torch.distributed as dist

    from ai_b200 import gemma, replicas
    from ai_b200 import synthetic as S

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    prec = prec_code(gemma, args.precision)
    budget = 131072
    w = S.make_weights(cfg, seed=0)
    model = gemma.from_synthetic(cfg, w, device=local_rank, max_batch_tokens=budget,
                                 options=[gemma.BatchTokens(budget)])
    seqs, lengths = S.make_ragged(8192, 16, 2048, 2)
    tokens = int(np.sum(lengths))

    def step():
        if world > 1:
            return replicas.embed_replicated(model, seqs, group=None, device=dev)
        return np.stack(model.embed_ids(seqs))

    def timed():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        r = step()
        torch.cuda.synchronize(dev)
        el = time.perf_counter() - t0
        per_rank = [el]
        if world > 1:
            t = torch.tensor([el], device=dev)
            parts = [torch.zeros_like(t) for _ in range(world)]
            dist.all_gather(parts, t)
            per_rank = [float(p.item()) for p in parts]
            el = max(per_rank)
        rank_times.append(per_rank)
        return r, el

    rank_times = []
    for _ in range(max(args.warmup, 1)):
        step()
    times = []
    sampler = ClockSampler(list(range(world)) if rank == 0 else [])
    if rank == 0:
        sampler.start()
    res = None
    for _ in range(max(args.steps, 1)):
        res, el = timed()
        times.append(el)
    clk = sampler.stop() if rank == 0 else None
    if rank == 0:
        sec = statistics.median(times)
        ok = res is not None and res.shape == (8192, model.Dim()) and bool(np.all(np.isfinite(res)))
        line = {
            "metric": "EmbeddingGemma embeddings/s, config 3 ragged (8192 seqs, lengths 16..2048)",
            "value": 8192 / sec, "unit": "embeddings/s", "n_gpus": world, "steps": len(times),
            "warmup": max(args.warmup, 1), "ms_per_step": sec * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: random-init weights (seed 0), ragged ids seed 2",
            "config": {"workload": "config 3: 8192 sequences, lengths uniform in [16, 2048], right-padded",
                       "batch_tokens": budget, "valid_tokens": tokens,
                       "parallelism": f"replicas x{world} on cost-balanced slices + NCCL gather onto rank 0"
                       if world > 1 else "single GPU",
                       "timing": "host wall clock around the synchronous public calls (ids on the host "
                                 "to embeddings on rank 0's host), median of steps, max over ranks"},
            "tokens_per_s": tokens / sec, "all_finite": ok, "clocks": clk,
            "rank_ms_last_step": [round(x * 1e3, 1) for x in rank_times[-1]],
            "step_ms": [round(x * 1e3, 1) for x in times],
        }
        print(json.dumps(line))
    model.close()
    if world > 1:
        dist.destroy_process_group()


def run_ragged_multi(args, cfg):
    """--workload ragged --multi: benchmark config 3 (8192 sequences, lengths
    uniform in [16, 2048], seed 2) through the one-process multi-GPU entry
    point fg_embed_many_multi — one model per GPU in this process, the
    length-sorted sequences cut into cost-balanced contiguous slices, one
    host thread per GPU, every embedding written into the host result in
    the caller's order (the call a Go host makes; no torchrun, no NCCL). A
    step is the whole batch; host wall clock around the synchronous call."""
    import torch

    from ai_b200 import gemma
    from ai_b200 import synthetic as S

    n = max(1, min(args.gpus, torch.cuda.device_count()))
    budget = 131072
    w = S.make_weights(cfg, seed=0)
    models = [gemma.from_synthetic(cfg, w, device=d, max_batch_tokens=budget, options=[gemma.BatchTokens(budget)])
              for d in range(n)]
    seqs, lengths = S.make_ragged(8192, 16, 2048, 2)
    tokens = int(np.sum(lengths))
    for _ in range(max(args.warmup, 1)):
        gemma.embed_ids_multi(models, seqs)
    clk = ClockSampler(list(range(n)))
    clk.start()
    times = []
    res = None
    for _ in range(max(args.steps, 1)):
        t0 = time.perf_counter()
        res = gemma.embed_ids_multi(models, seqs)
        times.append(time.perf_counter() - t0)
    clocks = clk.stop()
    sec = statistics.median(times)
    ok = res is not None and res.shape == (8192, models[0].Dim()) and bool(np.all(np.isfinite(res)))
    line = {
        "metric": "EmbeddingGemma embeddings/s, config 3 ragged (8192 seqs, lengths 16..2048), one process",
        "value": 8192 / sec, "unit": "embeddings/s", "n_gpus": n, "steps": len(times),
        "warmup": max(args.warmup, 1), "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: random-init weights (seed 0), ragged ids seed 2",
        "config": {"workload": "config 3: 8192 sequences, lengths uniform in [16, 2048], right-padded",
                   "batch_tokens": budget, "valid_tokens": tokens,
                   "parallelism": f"fg_embed_many_multi: {n} model(s), one host thread per GPU, no collective",
                   "timing": "host wall clock around the synchronous call (ids on the host to embeddings on "
                             "the host, caller's order), median of steps"},
        "tokens_per_s": tokens / sec, "all_finite": ok, "clocks": clocks,
        "step_ms": [round(x * 1e3, 1) for x in times],
    }
    print(json.dumps(line), flush=True)
    for m in models:
        m.close()


def eg2_work(t: dict, T: int):
    """Algorithmic FLOPs of one EmbeddingGemma 2 sequence of T valid tokens:
    the projections (Q/K/V/O, GeGLU, the PLE projection and each layer's PLE
    gate and projection) and the attention's allowed (query, key) pairs."""
    H, F, Hq, L, P = (t["hidden_size"], t["intermediate_size"], t["num_attention_heads"],
                      t["num_hidden_layers"], t["hidden_size_per_layer_input"])
    from ai_b200.gemma import config_from_dict

    c = config_from_dict({"model_type": "embedding_gemma2", "text_config": t})
    w = c.window()
    i = np.arange(T)
    local = int(np.sum(np.minimum(T - 1, i + w - 1) - np.maximum(0, i - w + 1) + 1)) if T > w else T * T
    linear = 2 * H * L * P * T  # per-layer-embedding projection
    attn = 0
    for l in range(L):
        D, kv = c.head_dim_of(l), c.kv_heads_of(l)
        linear += 2 * T * (H * (Hq + 2 * kv) * D + Hq * D * H + 3 * H * F + 2 * H * P)
        attn += 4 * Hq * D * (local if c.is_sliding(l) else T * T)
    return linear, attn


def run_eg2(args):
    """--workload eg2: EmbeddingGemma 2's text tower (the 12-layer shape of
    the reference's config test, random-init weights seed 0) at 256 × 512
    tokens on one GPU, inputs resident, device-timed with CUDA events."""
    import torch

    from ai_b200 import gemma
    from ai_b200 import synthetic as S

    dev = torch.device("cuda", 0)
    cfg = S.eg2_config()
    w = S.make_weights_eg2(cfg, seed=0)
    model = gemma.from_synthetic(cfg, w, device=0, max_batch_tokens=BATCH * SEQ)
    dim = model.Dim()
    ids = torch.from_numpy(S.make_ids(BATCH, SEQ, 1)).to(dev)
    lens = torch.from_numpy(np.full(BATCH, SEQ, np.int32)).to(dev)
    out = torch.empty((BATCH, dim), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(args.warmup, 3)):
        model.embed_device(ids, lens, BATCH, SEQ, dim, out, stream)
    model.check()
    model.read_profile()
    torch.cuda.synchronize()
    clocks = ClockSampler([0])
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        model.embed_device(ids, lens, BATCH, SEQ, dim, out, stream)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    model.check()
    # the phase split from another K steps with an event pair around every
    # launch (eager launches)
    model.set_profiling(True)
    for _ in range(args.steps):
        model.embed_device(ids, lens, BATCH, SEQ, dim, out, stream)
    torch.cuda.synchronize()
    model.set_profiling(False)
    prof = model.read_profile()
    linear, attn = eg2_work(cfg["text_config"], SEQ)
    flops = (linear + attn) * BATCH
    line = {
        "metric": "EmbeddingGemma 2 (text tower) embeddings/s at 256x512 tok, 1 B200", "value": BATCH / (ms / 1e3),
        "unit": "embeddings/s", "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: random-init EmbeddingGemma 2-shaped weights (seed 0), ids seed 1",
        "config": {"workload": "EmbeddingGemma 2 text tower: 12 layers, hidden 512, 4 heads; sliding layers "
                               "256-wide heads x2 KV, global layers 5/11 512-wide x1 KV; PLE 512; out 768; "
                               "256 x 512 tokens", "l2_flush": "none: activations exceed L2"},
        "tflops_algorithmic": flops / (ms / 1e3) / 1e12,
        "phases_ms_per_step": {p: round(v["ms"] / args.steps, 3) for p, v in prof.items()},
        "clocks": clk,
    }
    print(json.dumps(line))
    model.close()


def run_cluster(args):
    """--workload cluster: the consumer of the embeddings on one GPU —
    cluster.Nearest at the reference's TestNearestSpeed size (50 000 unit
    rows × 768 against 40 centres, cluster_test.go:65-79) timed on the
    device with CUDA events, and cluster.KMeans (k = 40, 20 rounds) timed
    end to end through its host call; the CPU restatement (oracle/cluster.py,
    numpy float64 products on all host threads) beside both."""
    import torch

    from ai_b200 import cluster as CL
    from oracle import cluster as OC

    dev = torch.device("cuda:0")
    n, d, k = 50000, 768, 40
    rng = np.random.default_rng(12)
    groups = OC.normalize(rng.standard_normal((k, d)).astype(np.float32))
    xs = OC.normalize((groups[np.arange(n) % k] + 0.1 * rng.standard_normal((n, d))).astype(np.float32))
    cs = OC.normalize(rng.standard_normal((k, d)).astype(np.float32))
    x = torch.from_numpy(xs).to(dev)
    c = torch.from_numpy(cs).to(dev)
    idx = torch.empty(n, dtype=torch.int32, device=dev)
    sim = torch.empty(n, dtype=torch.float32, device=dev)
    lib = __import__("ai_b200._lib", fromlist=["lib"]).lib()
    stream = torch.cuda.current_stream(dev)

    def nearest():
        rc = lib.fg_nearest(n, k, d, x.data_ptr(), d, c.data_ptr(), d, idx.data_ptr(), sim.data_ptr(),
                            0, stream.cuda_stream)
        assert rc == 0
    for _ in range(max(args.warmup, 3)):
        nearest()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(args.steps, 20)
    clocks = ClockSampler([0])
    clocks.start()
    e0.record(stream)
    for _ in range(reps):
        nearest()
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / reps
    algo_bytes = n * d * 4 + k * d * 4 + n * 8  # rows read once, centres, index + similarity written
    pk = peaks()
    gbs = algo_bytes / (ms / 1e3) / 1e9
    t0 = time.perf_counter()
    want_i, _ = OC.nearest(xs, cs)
    cpu_nearest_ms = (time.perf_counter() - t0) * 1e3
    agree = float(np.mean(idx.cpu().numpy() == want_i))

    t0 = time.perf_counter()
    res = CL.KMeans(x, k, 20, 1)
    torch.cuda.synchronize()
    km_ms = (time.perf_counter() - t0) * 1e3
    t0 = time.perf_counter()
    ref = OC.kmeans(xs, k, 20, 1)
    cpu_km_ms = (time.perf_counter() - t0) * 1e3
    line = {
        "metric": "cluster.Nearest rows/s, 50000 x 768 against 40 centres", "value": n / (ms / 1e3),
        "unit": "rows/s", "n_gpus": 1, "steps": reps, "warmup": max(args.warmup, 3), "ms_per_step": ms,
        "higher_is_better": True, "dtype": "f32 (split-TF32 product)", "data": "synthetic: 40 noisy groups of unit rows, seed 12",
        "config": {"workload": "cluster: Nearest 50000 x 768 vs 40 centres; KMeans k=40, 20 rounds, seed 1",
                   "l2_flush": "none: the rows (154 MB) exceed L2"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / pk["hbm_gbs"], "traffic": None,
                     "note": f"algorithmic bytes {algo_bytes} per call ({pk['source']} peak)"},
        "nearest_index_agreement_with_oracle": agree,
        "kmeans": {"ms": km_ms, "iterations": res.Iterations, "inertia": res.Inertia(),
                   "oracle_iterations": ref.iterations, "oracle_inertia": ref.inertia(),
                   "assignment_equal": bool(np.array_equal(np.asarray(res.Assignment), ref.assignment))},
        "cpu_baseline": {"nearest_ms": cpu_nearest_ms, "kmeans_ms": cpu_km_ms, "kind": "port",
                         "cores": os.cpu_count(), "sample": "the same inputs, oracle/cluster.py (numpy)"},
        "clocks": clk,
    }
    print(json.dumps(line))


MATMUL_MS = [128, 1024, 8192, 65536]
MATMUL_KN = [(768, 768), (768, 1152), (768, 2304), (768, 3072), (1152, 768)]


def run_matmul(args):
    """--workload matmul: benchmark config 4, the standalone tensor.MatMul
    sweep (tensor/matmul.go:19-72) through fg_matmul on one GPU: M ∈ {128,
    1024, 8192, 65536} × (K, N) ∈ {768} × {768, 1152, 2304, 3072} plus
    (1152, 768), as A·B and as A·Wᵀ (transposed view, no copy), in split
    precision (fp32-level) and plain TF32. N(0, 1) entries from seed 3.
    Each call (operand split / packing included) is timed with CUDA events
    on its stream, L2 flushed (a 256 MB write) before every timed call."""
    import torch

    from ai_b200 import tensor as T

    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)  # 256 MB > L2
    pk = peaks()
    tf32_peak = pk["bf16_sustained"] / 2.0
    reps = max(args.steps, 3)
    rows = []
    tot = {"split": [0.0, 0.0], "tf32": [0.0, 0.0]}
    clocks = ClockSampler([0])
    clocks.start()
    g = torch.Generator(device=dev).manual_seed(3)
    for m in MATMUL_MS:
        for k, n in MATMUL_KN:
            a = torch.randn(m, k, generator=g, device=dev)
            w_kn = torch.randn(k, n, generator=g, device=dev)
            w_nk = torch.randn(n, k, generator=g, device=dev)
            for form, w in (("A.B", w_kn), ("A.Wt", w_nk.t())):
                for prec_name, prec in (("split", T.PREC_SPLIT), ("tf32", T.PREC_TF32)):
                    for _ in range(max(args.warmup, 2)):
                        T.MatMul(a, w, precision=prec)
                    ms = 0.0
                    for _ in range(reps):
                        flush.zero_()
                        e0 = torch.cuda.Event(enable_timing=True)
                        e1 = torch.cuda.Event(enable_timing=True)
                        e0.record(stream)
                        T.MatMul(a, w, precision=prec)
                        e1.record(stream)
                        torch.cuda.synchronize()
                        ms += e0.elapsed_time(e1)
                    ms /= reps
                    flops = 2.0 * m * n * k
                    tf = flops / (ms / 1e3) / 1e12
                    tot[prec_name][0] += flops * reps
                    tot[prec_name][1] += ms * reps / 1e3
                    rows.append({"m": m, "k": k, "n": n, "form": form, "precision": prec_name,
                                 "ms": round(ms, 4), "tflops": round(tf, 2),
                                 "frac_of_tf32_peak": round(tf / tf32_peak, 4)})
    clk = clocks.stop()
    agg = {p: (f / t / 1e12 if t else None) for p, (f, t) in tot.items()}
    big = [r for r in rows if r["m"] == 65536 and r["n"] == 3072 and r["precision"] == "split"]
    top = max(big, key=lambda r: r["tflops"])
    line = {
        "metric": "tensor.MatMul fp32 sweep TFLOP/s (config 4), 1 B200", "value": agg["split"],
        "unit": "TFLOP/s", "n_gpus": 1, "steps": reps, "warmup": max(args.warmup, 2),
        "ms_per_step": None, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic: N(0, 1) entries, torch generator seed 3",
        "config": {"workload": "config 4: M in {128,1024,8192,65536} x (K,N) in {768}x{768,1152,2304,3072} "
                               "+ (1152,768), A.B and A.Wt, split and plain TF32",
                   "l2_flush": "256 MB write before every timed call"},
        "aggregate_tflops": agg,
        "roofline": {"bound": "tensor", "kernel": "fg_matmul split (operand split + gemm_pair_kernel), "
                     f"M=65536 K=768 N=3072 {top['form']}", "achieved": top["tflops"], "peak": tf32_peak,
                     "unit": "TFLOP/s", "frac": top["tflops"] / tf32_peak, "traffic": None,
                     "peak_source": f"{pk['source']} bf16 sustained / 2 (dense TF32)"},
        "shapes": rows,
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--precision", choices=["split", "split_tf32", "tf32"], default="split",
                    help="split (default): fp32-level, split-fp16 products where the weights have an exact "
                         "fp16 form, else split-TF32; split_tf32: every product split-TF32; tf32: one pass")
    ap.add_argument("--checkpoint", choices=["bf16", "f32"], default="bf16",
                    help="bf16 (the spec: random-init weights rounded to bf16) or f32 (the same draws kept "
                         "in fp32: no exact fp16 form, TF32 low parts on every projection)")
    ap.add_argument("--global-batch", type=int, default=None,
                    help="strong scaling: this many sequences in total, split over the GPUs (default: "
                         "weak scaling, --batch sequences per GPU)")
    ap.add_argument("--windows", type=int, default=5, help="timing windows of >= 1 s after the K steps")
    ap.add_argument("--multi", action="store_true",
                    help="with --workload ragged: one process drives --gpus GPUs through fg_embed_many_multi")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--norm-std", type=float, default=0.0,
                    help="RMSNorm weights ~N(0, s^2) instead of the spec's zeros (checkpoint-like: the "
                         "folded projections then carry split-TF32 low parts, a third GEMM pass)")
    ap.add_argument("--weights", choices=["f32", "bf16"], default="f32",
                    help="projection weights resident in fp32 (default) or bf16, widened per layer")
    ap.add_argument("--batch", type=int, default=BATCH,
                    help="sequences per GPU (default 256; smaller only for profiling runs)")
    ap.add_argument("--seq", type=int, default=SEQ, help="tokens per sequence (default 512)")
    ap.add_argument("--workload", choices=["encoder", "ragged", "cluster", "eg2", "matmul"], default="encoder",
                    help="encoder (config 2, the headline, default), ragged (config 3 end to end), "
                         "cluster (Nearest / KMeans on one GPU), eg2 (EmbeddingGemma 2 text tower) or "
                         "matmul (config 4, the tensor.MatMul sweep)")
    args = ap.parse_args()
    if args.workload == "cluster":
        run_cluster(args)
        return
    if args.workload == "matmul":
        run_matmul(args)
        return
    if args.workload == "eg2":
        globals().update(BATCH=args.batch, SEQ=args.seq)
        run_eg2(args)
        return
    globals().update(BATCH=args.batch, SEQ=args.seq)
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if "WORLD_SIZE" not in os.environ and args.gpus != 1:
        world = 1  # launched without torchrun: one process, one GPU
    from ai_b200 import synthetic as S

    cfg = dict(S.EMBEDDINGGEMMA_300M)
    if args.impl == "reference":
        run_reference(args, rank, world, cfg)
    elif args.workload == "ragged" and args.multi:
        run_ragged_multi(args, cfg)
    elif args.workload == "ragged":
        run_ragged(args, rank, local_rank, world, cfg)
    else:
        run_ours(args, rank, local_rank, world, cfg)


if __name__ == "__main__":
    main()
