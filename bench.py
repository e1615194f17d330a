#!/usr/bin/env python
"""KV-cached decode tokens/s at MicroChat shape on 1-8 B200 (one process per GPU).

One step = one whole CachedGenerate job per GPU: 64 independent sequences, 128-id uniform prompts,
greedy decode of 384 new ids each (prefill of the 127-id context included). Sequences are sharded by
GPU (each rank runs its own 64, seeded by global sequence index: weak scaling); nothing crosses
NVLink on the hot path — NCCL only takes the max of the timings and gathers per-rank output checksums.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

`value` is generated tokens/s of the whole job with prompts already resident in HBM, timed with CUDA
events on the launching stream (max over ranks); `e2e` is the same metric through the host-buffer C ABI
(shahd_generate: prompts copied in, ids copied out, inside the timed region). `--impl reference` times
the reference's own CPU algorithm (the oracle restatement of its TS decode, all host threads) on the same
sequences; that arm imports nothing of the GPU package.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import signal
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "KV-cached decode tokens/s at MicroChat shape, 1-8 B200; % of HBM roofline"
L2_FLUSH_BYTES = 512 << 20  # > 126 MB L2
PROMPT_SEED_BASE = 1000  # sequence g's prompt: floor(NextFloat() * vocab) from SeededRng(1000 + g)

# The decode workloads as plain data, so the reference arm runs without the GPU package. They equal
# shahd-llm-stack_b200/configs.py (tests/test_bench_contract.py checks it). `ref_sample`: sequences and
# new tokens of one reference-arm step (None: the whole job). `scaling` "strong": `seqs` is the whole job,
# split over the ranks (Phase2Modern-style: 4096 sequences over 1/2/4/8 GPUs); otherwise every rank runs
# `seqs` sequences of its own (weak scaling).
WORKLOADS = {
    "foundry": dict(name="foundry-shape E128 L4 H4 GeGlu F512 ctx256 V4096", embed_dim=128, num_layers=4, num_heads=4,
                    kv_heads=4, block_size=256, vocab_size=4096, mlp_hidden=512, position_scheme="Learned",
                    norm_kind="LayerNorm", mlp_kind="GeGlu", weight_seed=0, seqs=1, prompt_len=64, new_tokens=192,
                    ref_sample=None),
    "microchat": dict(name="MicroChat-shape E256 L6 H4 SwiGlu F1024 ctx512 V4096", embed_dim=256, num_layers=6,
                      num_heads=4, kv_heads=4, block_size=512, vocab_size=4096, mlp_hidden=1024, position_scheme="Rope",
                      norm_kind="RmsNorm", mlp_kind="SwiGlu", weight_seed=1, seqs=64, prompt_len=128, new_tokens=384,
                      ref_sample=None),
    "phase2": dict(name="Phase2Modern-style E1024 L16 H16/4 SwiGlu F2816 ctx2048 V32768", embed_dim=1024,
                   num_layers=16, num_heads=16, kv_heads=4, block_size=2048, vocab_size=32768, mlp_hidden=2816,
                   position_scheme="Rope", norm_kind="RmsNorm", mlp_kind="SwiGlu", weight_seed=4, seqs=4096,
                   prompt_len=512, new_tokens=512, ref_sample=(1, 8), scaling="strong"),
}
_SHAPE_KEYS = ("embed_dim", "num_layers", "num_heads", "kv_heads", "block_size", "vocab_size", "mlp_hidden",
               "position_scheme", "norm_kind", "mlp_kind")


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def ref_prompts(wd: dict, rank: int, n: int) -> np.ndarray:
    """The prompts of sequences rank*seqs .. rank*seqs+n-1, drawn with the oracle's SeededRng."""
    from oracle import oracle as O

    g0 = rank * wd["seqs"]
    return np.stack([O.uniform_ids(wd["prompt_len"], wd["vocab_size"], PROMPT_SEED_BASE + g0 + i) for i in range(n)])


def ref_model(wd: dict):
    """The oracle model on the reference's seeded init (bit-exact with the product's f32 master weights)."""
    from oracle import oracle as O

    shape = O.Shape(**{k: wd[k] for k in _SHAPE_KEYS}, precision="F32")
    return O.Model(shape, O.init_params(shape, wd["weight_seed"]))


def package():
    return importlib.import_module("shahd-llm-stack_b200")


def prompts_for(w, rank: int) -> np.ndarray:
    return package().sharding.shard_prompts(w, rank)


def step_roofline(w, ms_per_job: float, peaks: dict, peak_kind: str) -> dict:
    """The hot-path step roofline: algorithmic bytes of every decode step of the job (all projection
    weights once per step, each sequence's cached K/V rows read and its new K/V row written, the embedding
    row) over the timed job time (prefill included in the time, not in the bytes: a lower bound)."""
    m = w.model
    weights = 2.0 * m.matrix_params()
    kv_pos = m.num_layers * m.kv * 2 * m.head_dim * 2  # bytes of one cached position, all layers
    p0 = w.prompt_len - 1  # position of the first decode step's token
    attended = sum(p0 + k + 1 for k in range(w.new_tokens))  # cached positions read per sequence
    job = w.new_tokens * (weights + w.seqs * (kv_pos + 2 * m.embed_dim)) + w.seqs * kv_pos * attended
    achieved = job / (ms_per_job / 1000.0) / 1e9
    return {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": achieved / peaks["hbm_gbs"], "algorithmic_bytes_per_job": job, "peak_source": peak_kind,
            "scope": "all decode steps of the timed job (weights per step + KV rows read/written)"}


def load_peaks() -> tuple[dict, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None
        self.path = os.path.join("/tmp", f"shahd_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.out, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.send_signal(signal.SIGTERM)
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.out.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9 or (self.uuid and f[0] != self.uuid):
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons), "samples": len(sm)}


def cpu_baseline(wd: dict, model, threads: int, seqs: int, new_tokens: int, rank: int = 0) -> dict:
    """The reference's CPU decode (oracle restatement of CachedGenerate, f64 row math on f32 weights):
    `seqs` of the workload's sequences, one per thread."""
    prompts = ref_prompts(wd, rank, seqs)
    t0 = time.perf_counter()
    model.cached_generate_batch(prompts, new_tokens, threads=threads)
    dt = time.perf_counter() - t0
    return {"value": seqs * new_tokens / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "cpu": cpu_model(),
            "sample": f"{seqs} sequences x (prefill {wd['prompt_len'] - 1} + {new_tokens} greedy tokens), f64, "
                      f"{threads} threads (one sequence per thread), {dt:.1f} s"}


def goffi_projection_bound(wd: dict, threads: int, steps: int = 32) -> dict | None:
    """The reference's own C kernels (GoKernels/ffi/matmul_avx.c, compiled unmodified into oracle/_ref) behind
    the pthread FanOutRows twin (matmul.go:132-163), timed on every projection of a batched decode step of
    the workload's sequences (QKV, O, MLP up/down, LM head; f32). Decode in the reference never calls this
    seam (its row math is inline TS), so this is an upper bound for a GoFfi-backed decode: attention, norms
    and sampling are left out."""
    import ctypes

    from oracle import oracle as O

    R = O.ref_lib()
    if R is None:
        return None
    E, H, Hk, F, V, L = (wd["embed_dim"], wd["num_heads"], wd["kv_heads"], wd["mlp_hidden"], wd["vocab_size"],
                         wd["num_layers"])
    d = E // H
    M = wd["seqs"]
    up = 2 * F if wd["mlp_kind"] != "Relu" else F
    shapes = [(E, (H + 2 * Hk) * d), (H * d, E), (E, up), (F, E)] * L + [(E, V)]
    rng = np.random.default_rng(0)
    bufs = []
    for k, n in shapes:
        a = rng.standard_normal((M, k), dtype=np.float32)
        bt = rng.standard_normal((n, k), dtype=np.float32)
        bufs.append((a, bt, np.empty((M, n), np.float32), k, n))
    fp = ctypes.POINTER(ctypes.c_float)

    def step():
        for a, bt, out, k, n in bufs:
            R.RefMatMulNTF32(a.ctypes.data_as(fp), bt.ctypes.data_as(fp), out.ctypes.data_as(fp), M, k, n, 0, threads)

    step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = time.perf_counter() - t0
    return {"value": M * steps / dt, "unit": "tokens/s", "cores": threads, "kind": "reference", "cpu": cpu_model(),
            "avx2_fma": bool(R.RefCpuHasAvx2Fma()),
            "sample": f"{steps} decode steps of {M} rows: every projection (QKV, O, MLP up/down, LM head) through the "
                      f"reference's own AVX2 f32 kernels behind the FanOutRows twin, {threads} threads; attention, "
                      "norms and sampling excluded (an upper bound for a GoFfi-backed decode)"}


def run_reference(args, rank: int, world: int) -> None:
    """The reference's CPU decode on the host cores (rank 0 only), on the workload's own sequences."""
    if rank != 0:
        return
    wd = WORKLOADS[args.workload]
    threads = os.cpu_count() or 1
    seqs, new = (wd["seqs"], wd["new_tokens"]) if wd["ref_sample"] is None else wd["ref_sample"]
    from oracle import oracle as O

    if wd["ref_sample"] is not None:
        O.set_threads(threads)  # one long prefill: split its matmuls instead of the sequences
    model = ref_model(wd)
    warm = (min(2, seqs), min(4, new))
    for _ in range(args.warmup):  # untimed warm-up on a small sample
        cpu_baseline(wd, model, threads, *warm)
    vals = [cpu_baseline(wd, model, threads, seqs, new) for _ in range(args.steps)]
    ms = statistics.mean(seqs * new / v["value"] * 1000.0 for v in vals)
    value = seqs * new / (ms / 1000.0)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": wd.get("scaling", "weak"),
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": wd["name"], "seqs_per_gpu": seqs, "prompt_len": wd["prompt_len"], "new_tokens": new,
                   "global_batch": seqs, "seq_len": wd["prompt_len"] + new,
                   "sample_of": f"{wd['seqs']} sequences x {wd['new_tokens']} new tokens per GPU",
                   "warmup_sample": f"{warm[0]} sequences x {warm[1]} new tokens"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "cpu": cpu_model(),
                         "sample": vals[0]["sample"]},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, rank: int, world: int, local_rank: int) -> None:
    import torch

    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    pkg = package()
    import dataclasses

    w = pkg.configs.WORKLOADS[args.workload]
    strong = WORKLOADS[args.workload].get("scaling") == "strong"
    if strong:  # the job's sequences are split over the ranks
        if w.seqs % world:
            raise SystemExit(f"{w.name}: {w.seqs} sequences do not split over {world} GPUs")
        w = dataclasses.replace(w, seqs=w.seqs // world)
    if args.seqs is not None:
        w = dataclasses.replace(w, seqs=args.seqs)
    if args.new_tokens is not None:
        w = dataclasses.replace(w, new_tokens=args.new_tokens)
    if args.prompt_len is not None:
        w = dataclasses.replace(w, prompt_len=args.prompt_len)
    cfg = w.model
    params = pkg.init_params(cfg, w.weight_seed)
    lib = pkg.load()
    if args.chains:
        lib.ShahdSetDecodeChains(args.chains)
    if args.tc_min_rows:
        lib.ShahdSetTensorCoreMinRows(args.tc_min_rows)
    if args.fused_block >= 0:
        lib.ShahdSetFusedAttentionBlock(args.fused_block)
    if args.decode_attn >= 0:
        lib.ShahdSetDecodeAttentionKernel(args.decode_attn)
    # a KV pool of the job's size: every sequence's pages up to prompt + new positions (Phase2Modern-style:
    # 4096 x 16 pages of 1 MiB = 64 GiB on one GPU)
    kv_pages = w.seqs * -(-min(w.prompt_len + w.new_tokens, cfg.block_size) // 64)
    sess = pkg.Session(cfg, params, max_seqs=w.seqs, device=local_rank, kv_pages=kv_pages)
    prompts = prompts_for(w, rank)
    offs = np.arange(0, (w.seqs + 1) * w.prompt_len, w.prompt_len, dtype=np.int32)
    d_prompts = torch.from_numpy(prompts.reshape(-1).copy()).to(dev)
    d_out = torch.empty(w.seqs * w.new_tokens, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)  # a real stream handle: the library joins it with events
    torch.cuda.set_stream(stream)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def step():
        sess.generate_device(d_prompts.data_ptr(), offs, w.new_tokens, d_out.data_ptr(), stream=stream.cuda_stream)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step()
    barrier()
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid) if rank == 0 else None
    except Exception:
        uuid = None
    clocks = ClockSampler(uuid) if rank == 0 else None
    if clocks:
        clocks.start()
    launches0 = sess.kernel_launches()
    evs = []
    barrier()
    for _ in range(args.steps):
        flush.zero_()  # L2 flush between timed steps (not timed)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        step()
        e1.record(stream)
        evs.append((e0, e1))
    barrier()
    launches = sess.kernel_launches() - launches0
    clk = clocks.stop() if clocks else None
    total_ms = sum(a.elapsed_time(b) for a, b in evs)
    t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    ms_per_step = max_ms / args.steps
    tokens_per_step_all = world * w.seqs * w.new_tokens
    value = tokens_per_step_all / (ms_per_step / 1000.0)

    if args.no_extras:
        if dist is not None:
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"ms_per_step": ms_per_step, "value": value, "gpu_launches": int(launches),
                              "chains": args.chains, "tc_min_rows": args.tc_min_rows,
                              "fused_block": args.fused_block, "decode_attn": args.decode_attn}), flush=True)
        return

    # gather per-rank output checksums (the only collective, outside the timed region)
    chk = torch.tensor([int(d_out.sum().item())], dtype=torch.int64, device=dev)
    if dist is not None:
        allc = [torch.zeros_like(chk) for _ in range(world)]
        dist.all_gather(allc, chk)
        checksums = [int(c.item()) for c in allc]
    else:
        checksums = [int(chk.item())]

    # e2e through the host-buffer C ABI: prompts H2D, ids D2H inside the timed region
    e2e_ms = []
    e2e_warm = args.warmup if args.workload == "microchat" else 1  # the device leg already warmed the session
    for i in range(e2e_warm + args.steps):
        flush.zero_()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        sess.generate(prompts, w.new_tokens)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        if i >= e2e_warm:
            e2e_ms.append(e0.elapsed_time(e1))
    te = torch.tensor([sum(e2e_ms)], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = tokens_per_step_all / (float(te.item()) / len(e2e_ms) / 1000.0)

    # per-kernel-class shares over one extra job with CUDA events on the session stream around every launch.
    # Event nodes inside a replayed graph add time and break the programmatic overlap, so the bracketed run
    # gives only each class's SHARE of the job; a class's time is that share of the unbracketed ms_per_step
    # (the decode loop, when it runs, is one launch per run of steps and is timed directly).
    sess.profile(True)
    flush.zero_()
    step()
    torch.cuda.synchronize(dev)
    prof = {k: sess.profile_read(k) for k in sess.PROFILE_KINDS}
    sess.profile(False)

    if dist is not None:
        torch.cuda.synchronize(dev)
        dist.destroy_process_group()
    if rank != 0:
        return

    peaks, peak_kind = load_peaks()
    traffic_ratio = {}
    tpath = os.path.join(ROOT, "profiles", "traffic_ratio.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            traffic_ratio = json.load(f)
    bracketed_ms = sum(v["ms"] for v in prof.values())
    scale = ms_per_step / bracketed_ms if bracketed_ms > 0 else 0.0
    if prof["decode_loop"]["launches"] > 0:
        dom, kernel, scale = "decode_loop", "DecodeLoopKernel", 1.0
    else:  # per-kernel decode steps: the larger of the projection and decode-attention classes
        dom = max(("attention", "linear"), key=lambda k: prof[k]["ms"])
        kernel = {"attention": "decode attention kernels", "linear": "decode projection kernels"}[dom]
    p = prof[dom]
    nl = max(p["launches"], 1)
    class_ms = p["ms"] * scale
    achieved = p["bytes"] / (class_ms / 1000.0) / 1e9 if class_ms > 0 else 0.0
    traffic = traffic_ratio[dom] * p["bytes"] / nl if traffic_ratio.get(dom) else None
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "traffic": traffic, "kernel": kernel, "peak_source": peak_kind,
                "launches_per_job": p["launches"], "avg_launch_ms": class_ms / nl,
                "algorithmic_bytes_per_launch": p["bytes"] / nl,
                "share_of_step": class_ms / ms_per_step,
                "timing": ("one CUDA-event-timed launch per run of decode steps" if dom == "decode_loop" else
                           "the class's share of a job with CUDA events around every launch, times the unbracketed "
                           "ms_per_step"),
                "bytes": "per decode step: every weight matrix once (bf16) + each row's cached K/V rows read and its new "
                         "K/V row written (bf16); prefill not included"}
    classes = {k: {"share": v["ms"] / bracketed_ms if bracketed_ms > 0 else None, "ms_per_job": v["ms"] * scale,
                   "bracketed_ms_per_job": v["ms"], "launches": v["launches"], "algorithmic_bytes": v["bytes"]}
               for k, v in prof.items() if v["launches"] > 0}
    expected = None
    gpath = os.path.join(ROOT, "tests", "golden", "microchat_job.json")
    mc = pkg.configs.MICROCHAT
    if ((w.name, w.seqs, w.prompt_len, w.new_tokens) == (mc.name, mc.seqs, mc.prompt_len, mc.new_tokens) and rank == 0
            and os.path.exists(gpath)):
        with open(gpath) as f:
            expected = json.load(f)["checksum"]
    output_check = {"expected_checksum_per_rank": expected,
                    "match": None if expected is None else checksums[0] == expected,
                    "how": "tests/golden/microchat_job.json: the ids of rank 0's 64 sequences, every id checked against "
                           "the oracle teacher-forced on its own prefix"}
    cpu = goffi = None
    if world == 1 and not args.skip_cpu:  # the reference's CPU path on this host, rank 0 at N=1 only
        threads = os.cpu_count() or 1
        wd = WORKLOADS[args.workload]
        seqs, new = (w.seqs, w.new_tokens) if wd["ref_sample"] is None else wd["ref_sample"]
        cpu = cpu_baseline(wd, ref_model(wd), threads, seqs, new)
        goffi = goffi_projection_bound(wd, threads)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong" if strong else "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": w.name, "seqs_per_gpu": w.seqs, "prompt_len": w.prompt_len, "new_tokens": w.new_tokens,
                   "global_batch": world * w.seqs, "seq_len": w.prompt_len + w.new_tokens,
                   "parallelism": f"sequence shards x{world} (full weight replica per GPU, no collective in the step)",
                   "weights_l2_resident": 2.0 * cfg.matrix_params() < 63e6,
                   "kv_pool_bytes": int(kv_pages) * cfg.num_layers * cfg.kv * 2 * 64 * cfg.head_dim * 2,
                   "weights": f"reference init seed {w.weight_seed} (fp32 master -> bf16)",
                   "l2": "flushed (512 MiB write) before every timed step", "output_checksums": checksums},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": int(prompts.nbytes + offs.nbytes),
                "d2h_bytes_per_step": int(w.seqs * w.new_tokens * 4)},
        "roofline": roofline,
        "roofline_step": step_roofline(w, ms_per_step, peaks, peak_kind),
        "output_check": output_check,
        "cpu_baseline": cpu,
        "cpu_baseline_goffi_kernels": goffi,
        "clocks": clk,
        "gpu_launches": int(launches),
        "kernel_classes_per_job": classes,
    }
    print(json.dumps(line), flush=True)


SWEEP_M = (1, 64, 1024, 8192)
SWEEP_NK = ((768, 256), (1024, 256), (256, 1024), (4096, 256), (4096, 1024))


def run_matmul_sweep(args, rank: int) -> None:
    """The MatMulNT operator sweep (C = A·Bᵀ, A[M,K], B[N,K] ~ N(0,1), seed 2) on the two tensor-core GEMMs of
    the library with operands resident in HBM: bf16 (ShahdMatMulNTBF16Device) and fp32 through split-TF32
    (ShahdMatMulNTF32Device, three kind::tf32 passes). Each call timed alone with CUDA events after an L2 flush;
    median of --steps calls after --warmup untimed ones. One JSON line, the per-shape figures in `shapes`."""
    import torch

    if rank != 0:
        return
    pkg = package()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks, peak_kind = load_peaks()
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    g = torch.Generator(device="cpu").manual_seed(2)
    shapes = []
    launches = 0
    for n, k in SWEEP_NK:
        bt32 = torch.randn(n, k, generator=g).to(dev)
        bt16 = bt32.to(torch.bfloat16)
        for m in SWEEP_M:
            a32 = torch.randn(m, k, generator=g).to(dev)
            a16 = a32.to(torch.bfloat16)
            out = torch.empty(m, n, device=dev)
            res = {"M": m, "N": n, "K": k}
            for name, call in (
                ("bf16", lambda: pkg.backend.matmul_nt_bf16_device(a16.data_ptr(), bt16.data_ptr(), out.data_ptr(), m, k, n,
                                                                   stream=stream.cuda_stream)),
                ("tf32x3", lambda: pkg.backend.matmul_nt_f32_device(a32.data_ptr(), bt32.data_ptr(), out.data_ptr(), m, k,
                                                                    n, stream=stream.cuda_stream))):
                for _ in range(args.warmup):
                    call()
                # every timed call sits behind its own L2 flush on the stream, enqueued without waiting, so the
                # events measure the device and not the host's enqueue latency
                evs = []
                for _ in range(args.steps):
                    flush.zero_()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    call()
                    e1.record(stream)
                    evs.append((e0, e1))
                torch.cuda.synchronize(dev)
                times = [a.elapsed_time(b) for a, b in evs]
                launches += args.steps * (1 if name == "bf16" else 3)
                ms = statistics.median(times)
                tflops = 2.0 * m * n * k / (ms / 1000.0) / 1e12
                res[name] = {"ms": ms, "tflops": tflops}
            res["bf16"]["frac_of_bf16_peak"] = res["bf16"]["tflops"] / peaks["bf16_tflops"]
            # three kind::tf32 passes, each at half the bf16 tensor rate
            res["tf32x3"]["frac_of_tf32_pipe"] = 3 * res["tf32x3"]["tflops"] / (peaks["bf16_tflops"] / 2)
            shapes.append(res)
    big = [r for r in shapes if r["M"] >= 1024]
    value = statistics.mean(r["bf16"]["tflops"] for r in big)
    line = {"metric": "MatMulNT operator sweep TFLOP/s (bf16 tcgen05, M >= 1024 mean)", "value": value,
            "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": statistics.mean(r["bf16"]["ms"] for r in big), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "MatMulNT sweep M in {1,64,1024,8192} x (N,K) in 5 shapes, N(0,1) seed 2",
                       "l2": "flushed (512 MiB write) before every timed call"},
            "roofline": {"bound": "tensor", "achieved": value, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": value / peaks["bf16_tflops"], "traffic": None, "peak_source": peak_kind},
            "gpu_launches": launches, "shapes": shapes}
    print(json.dumps(line), flush=True)


FA = dict(seqs=256, heads=8, kv_heads=2, head_dim=64, prompt=512, steps=64, rope_base=10000.0, seed=3)


def fused_attention_inputs():
    """Q/K/V ~ N(0,1) (numpy default_rng(seed 3), fp32) for every prompt and decode position of every sequence."""
    n, T = FA["seqs"], FA["prompt"] + FA["steps"]
    rng = np.random.default_rng(FA["seed"])
    q = rng.standard_normal((n, T, FA["heads"], FA["head_dim"]), dtype=np.float32)
    k = rng.standard_normal((n, T, FA["kv_heads"], FA["head_dim"]), dtype=np.float32)
    v = rng.standard_normal((n, T, FA["kv_heads"], FA["head_dim"]), dtype=np.float32)
    return q, k, v


def fused_attention_cpu(q, k, v, seqs: int, threads: int) -> dict:
    """The oracle restatement of the reference's attention (RoPE, CausalSoftmax, @ V) on `seqs` sequences of
    the workload, one sequence per host thread (the C oracle releases the GIL)."""
    from concurrent.futures import ThreadPoolExecutor

    from oracle import oracle as O

    t0 = time.perf_counter()
    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(lambda i: O.fused_attention(q[i], k[i], v[i], FA["rope_base"]), range(seqs)))
    dt = time.perf_counter() - t0
    T = FA["prompt"] + FA["steps"]
    return {"value": seqs * T / dt, "unit": "positions/s", "cores": threads, "kind": "port", "cpu": cpu_model(),
            "sample": f"{seqs} sequences x {T} positions (causal attention of every position = prefill + decode "
                      f"outputs), f64, {threads} threads, {dt:.1f} s"}


def run_fused_attention(args, rank: int, world: int, local_rank: int) -> None:
    """FusedAttention with RoPE (base 10000) + GQA, 8 query heads over 2 kv heads, head_dim 64: causal prefill of
    512 positions of 256 sequences, then 64 one-token decode steps (shahd_attention_prefill / _decode). A step
    is the whole job; value = positions/s (prefill + decode). Inputs resident in HBM; e2e copies them from
    pinned host memory and the outputs back inside the timed region. Every rank runs its own 256 sequences."""
    import torch

    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    pkg = package()
    n, T, S = FA["seqs"], FA["prompt"], FA["steps"]
    H, Hk, d = FA["heads"], FA["kv_heads"], FA["head_dim"]
    q, k, v = fused_attention_inputs()
    hq, hk, hv = (torch.from_numpy(x).pin_memory() for x in (q, k, v))
    dq, dk, dv = (x.to(dev) for x in (hq, hk, hv))
    pq, pk, pv = (x[:, :T].contiguous() for x in (dq, dk, dv))  # prefill inputs
    sq, sk, sv = ([x[:, T + i].contiguous() for i in range(S)] for x in (dq, dk, dv))  # decode inputs
    out_p = torch.empty((n, T, H, d), dtype=torch.float32, device=dev)
    out_d = torch.empty((S, n, H, d), dtype=torch.float32, device=dev)
    host_out_p = torch.empty(out_p.shape, dtype=torch.float32).pin_memory()
    host_out_d = torch.empty(out_d.shape, dtype=torch.float32).pin_memory()
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    op = pkg.FusedAttention(n, H, Hk, d, T + S, FA["rope_base"], device=local_rank)
    st = stream.cuda_stream

    def job(ev=None):
        if ev:
            ev[0].record(stream)
        op.prefill(pq.data_ptr(), pk.data_ptr(), pv.data_ptr(), n, T, out_p.data_ptr(), st)
        if ev:
            ev[1].record(stream)
        for i in range(S):
            op.decode(sq[i].data_ptr(), sk[i].data_ptr(), sv[i].data_ptr(), n, out_d[i].data_ptr(), st)
        if ev:
            ev[2].record(stream)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        job()
    barrier()
    clocks = ClockSampler(None) if rank == 0 else None
    if clocks:
        clocks.start()
    evs = []
    for _ in range(args.steps):
        flush.zero_()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        job(ev)
        evs.append(ev)
    barrier()
    clk = clocks.stop() if clocks else None
    pre_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    dec_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    t = torch.tensor([pre_ms + dec_ms], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    positions = world * n * (T + S)
    # e2e: inputs from pinned host memory and outputs back to it, inside the timed region
    e2e = []
    for i in range(1 + args.steps):
        flush.zero_()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for dst, src in ((dq, hq), (dk, hk), (dv, hv)):
            dst.copy_(src, non_blocking=True)
        pq.copy_(dq[:, :T])
        pk.copy_(dk[:, :T])
        pv.copy_(dv[:, :T])
        for j in range(S):
            sq[j].copy_(dq[:, T + j])
            sk[j].copy_(dk[:, T + j])
            sv[j].copy_(dv[:, T + j])
        job()
        host_out_p.copy_(out_p, non_blocking=True)
        host_out_d.copy_(out_d, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        if i >= 1:
            e2e.append(e0.elapsed_time(e1))
    op.close()
    if dist is not None:
        dist.destroy_process_group()
    if rank != 0:
        return
    peaks, peak_kind = load_peaks()
    pre_flops = n * 4.0 * H * d * T * (T + 1) / 2  # Q.K^T and P.V over the causal triangle
    dec_bytes = sum(n * (2 * Hk * d * 2 * (T + i + 1) + 2 * Hk * d * 2 + 2 * H * d * 4) for i in range(S))
    pre_tflops = pre_flops / (pre_ms / 1000.0) / 1e12
    dec_gbs = dec_bytes / (dec_ms / 1000.0) / 1e9
    cpu = None
    if world == 1 and not args.skip_cpu:
        threads = os.cpu_count() or 1
        cpu = fused_attention_cpu(q, k, v, n, threads)
    line = {
        "metric": "FusedAttention (RoPE + GQA) positions/s: causal prefill 512 + 64 decode steps, 256 sequences",
        "value": positions / (ms / 1000.0), "unit": "positions/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "FusedAttention Hq8 Hk2 d64 RoPE10000, 256 sequences, prefill 512 + 64 decode steps",
                   "inputs": "Q/K/V ~ N(0,1), numpy default_rng(3), fp32 in HBM; K/V cached in bf16",
                   "l2": "flushed (512 MiB write) before every timed step"},
        "e2e": {"value": positions / (statistics.mean(e2e) / 1000.0), "unit": "positions/s",
                "h2d_bytes_per_step": int(q.nbytes + k.nbytes + v.nbytes),
                "d2h_bytes_per_step": int(host_out_p.numel() * 4 + host_out_d.numel() * 4)},
        "prefill": {"ms": pre_ms, "tflops": pre_tflops, "frac_of_bf16_peak": pre_tflops / peaks["bf16_tflops"],
                    "flops": pre_flops},
        "decode": {"ms_per_step": dec_ms / S, "gbs": dec_gbs, "frac_of_hbm": dec_gbs / peaks["hbm_gbs"],
                   "bytes_per_step": dec_bytes / S},
        "roofline": {"bound": "hbm", "achieved": dec_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": dec_gbs / peaks["hbm_gbs"], "traffic": None, "kernel": "decode attention (page streaming)",
                     "peak_source": peak_kind},
        "cpu_baseline": cpu, "clocks": clk, "gpu_launches": args.steps * (2 + 3 * S),
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="microchat", choices=sorted(WORKLOADS) + ["matmul_sweep", "fused_attention"])
    ap.add_argument("--no-extras", action="store_true",
                    help="time the steps only (no e2e, profile or CPU legs): the profiling command line")
    ap.add_argument("--chains", type=int, default=0, help="concurrent decode chains (0 = library default)")
    ap.add_argument("--tc-min-rows", type=int, default=0, help="rows from which projections use tensor cores (0 = default)")
    ap.add_argument("--decode-attn", type=int, default=-1, choices=[-1, 0, 1, 2, 3],
                    help="decode attention kernel (ShahdSetDecodeAttentionKernel); -1 keeps the library default")
    ap.add_argument("--prompt-len", type=int, default=None,
                    help="override the prompt length (profiling a short job at a long cached length)")
    ap.add_argument("--fused-block", type=int, default=-1, choices=[-1, 0, 1],
                    help="decode rows run the fused attention block where the model fits it (1) or the three-launch "
                         "chain (0); -1 keeps the library default")
    ap.add_argument("--new-tokens", type=int, default=None,
                    help="override the workload's new tokens per sequence (small ncu captures only)")
    ap.add_argument("--seqs", type=int, default=None,
                    help="override the sequences per GPU (1: the batch-1 decode line)")
    ap.add_argument("--skip-cpu", action="store_true", help="leave out the CPU baselines (long secondary legs)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.warmup < 3:
        args.warmup = 3
    if args.workload == "matmul_sweep":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the MatMulNT sweep has no reference arm here; the "
                              "decode workloads carry it"}), flush=True)
        else:
            run_matmul_sweep(args, rank)
    elif args.workload == "fused_attention":
        if args.impl == "reference":
            if rank == 0:
                q, k, v = fused_attention_inputs()
                threads = os.cpu_count() or 1
                vals = [fused_attention_cpu(q, k, v, FA["seqs"], threads) for _ in range(args.steps)]
                value = statistics.mean(x["value"] for x in vals)
                print(json.dumps({"impl": "reference", "metric": "FusedAttention (RoPE + GQA) positions/s: causal prefill "
                                  "512 + 64 decode steps, 256 sequences", "value": value, "unit": "positions/s",
                                  "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                                  "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
                                  "config": {"workload": "FusedAttention Hq8 Hk2 d64 RoPE10000, 256 sequences, prefill "
                                             "512 + 64 decode steps"},
                                  "cpu_baseline": {**vals[0], "value": value},
                                  "e2e": {"value": value, "unit": "positions/s", "h2d_bytes_per_step": 0,
                                          "d2h_bytes_per_step": 0}}), flush=True)
        else:
            run_fused_attention(args, rank, world, local_rank)
    elif args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
