#!/usr/bin/env python
"""KV-cached decode tokens/s at MicroChat shape on 1-8 B200 (one process per GPU).

One step = one whole CachedGenerate job per GPU: 64 independent sequences, 128-id uniform prompts,
greedy decode of 384 new ids each (prefill of the 127-id context included). Sequences are sharded by
GPU (each rank runs its own 64, seeded by global sequence index: weak scaling); nothing crosses
NVLink on the hot path — NCCL only takes the max of the timings and gathers per-rank output checksums.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

`value` is generated tokens/s of the whole job with prompts already resident in HBM, timed with CUDA
events on the launching stream (max over ranks); `e2e` is the same metric through the host-buffer C ABI
(shahd_generate: prompts copied in, ids copied out, inside the timed region). `--impl reference` times
the reference's own CPU algorithm (the oracle restatement of its TS decode, all host threads) on a
bounded sample of the same workload.
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
pkg = importlib.import_module("shahd-llm-stack_b200")

METRIC = "KV-cached decode tokens/s at MicroChat shape, 1-8 B200; % of HBM roofline"
L2_FLUSH_BYTES = 512 << 20  # > 126 MB L2


def prompts_for(w, rank: int) -> np.ndarray:
    return pkg.sharding.shard_prompts(w, rank)


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


def cpu_baseline(w, params: np.ndarray, threads: int, seqs: int, new_tokens: int) -> dict:
    """The reference's CPU decode (oracle restatement of CachedGenerate, f64) on a bounded sample."""
    from oracle import oracle as O

    cfg = w.model
    shape = O.Shape(embed_dim=cfg.embed_dim, num_layers=cfg.num_layers, num_heads=cfg.num_heads,
                    block_size=cfg.block_size, vocab_size=cfg.vocab_size, mlp_hidden=cfg.mlp_hidden, kv_heads=cfg.kv,
                    position_scheme=cfg.position_scheme, norm_kind=cfg.norm_kind, mlp_kind=cfg.mlp_kind,
                    weight_tying=cfg.weight_tying, precision="F32")
    model = O.Model(shape, params.astype(np.float64))
    prompts = prompts_for(w, 0)[:seqs]
    t0 = time.perf_counter()
    model.cached_generate_batch(prompts, new_tokens, threads=threads)
    dt = time.perf_counter() - t0
    return {"value": seqs * new_tokens / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{seqs} sequences x (prefill {w.prompt_len - 1} + {new_tokens} greedy tokens), f64, "
                      f"{threads} threads (one sequence per thread), {dt:.1f} s"}


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    w = pkg.configs.WORKLOADS[args.workload]
    params = pkg.init_params(w.model, w.weight_seed)
    threads = os.cpu_count() or 1
    seqs, new = min(threads, w.seqs), w.new_tokens
    for _ in range(args.warmup):
        cpu_baseline(w, params, threads, seqs, new)
    vals = [cpu_baseline(w, params, threads, seqs, new) for _ in range(args.steps)]
    value = statistics.mean(v["value"] for v in vals)
    ms = seqs * new / value * 1000.0
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f64", "data": "synthetic",
        "config": {"workload": w.name, "seqs": seqs, "prompt_len": w.prompt_len, "new_tokens": new,
                   "sample_of": f"{w.seqs} sequences x {w.new_tokens} new tokens per GPU"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
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
    w = pkg.configs.WORKLOADS[args.workload]
    cfg = w.model
    params = pkg.init_params(cfg, w.weight_seed)
    lib = pkg.load()
    if args.chains:
        lib.ShahdSetDecodeChains(args.chains)
    if args.tc_min_rows:
        lib.ShahdSetTensorCoreMinRows(args.tc_min_rows)
    sess = pkg.Session(cfg, params, max_seqs=w.seqs, device=local_rank)
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
                              "chains": args.chains, "tc_min_rows": args.tc_min_rows}), flush=True)
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
    for i in range(args.warmup + args.steps):
        flush.zero_()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        sess.generate(prompts, w.new_tokens)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        if i >= args.warmup:
            e2e_ms.append(e0.elapsed_time(e1))
    te = torch.tensor([sum(e2e_ms)], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = tokens_per_step_all / (float(te.item()) / len(e2e_ms) / 1000.0)

    # live per-kernel-class timing (CUDA events on the launching stream) over one extra profiled job
    sess.profile(True)
    flush.zero_()
    step()
    torch.cuda.synchronize(dev)
    prof = {k: sess.profile_read(k) for k in ("attention", "linear", "other", "prefill_attention", "prefill_linear",
                                                 "prefill_other")}
    sess.profile(False)

    if dist is not None:
        torch.cuda.synchronize(dev)
        dist.destroy_process_group()
    if rank != 0:
        return

    peaks, peak_kind = load_peaks()
    dom = max(("attention", "linear"), key=lambda k: prof[k]["ms"])
    p = prof[dom]
    achieved = p["bytes"] / (p["ms"] / 1000.0) / 1e9 if p["ms"] > 0 else 0.0
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic_ratio.json")
    if os.path.exists(tpath):
        ratio = json.load(open(tpath)).get(dom)
        if ratio:
            traffic = ratio * p["bytes"] / max(p["launches"], 1)
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "traffic": traffic, "kernel": dom, "peak_source": peak_kind,
                "avg_launch_us": p["ms"] * 1000.0 / max(p["launches"], 1), "launches_profiled": p["launches"],
                "algorithmic_bytes_per_launch": p["bytes"] / max(p["launches"], 1),
                "share_of_step": p["ms"] / max(sum(prof[k]["ms"] for k in ("attention", "linear", "other")), 1e-9),
                "scope": "decode-step launches (prefill launches are reported apart)",
                # both HBM-bound kernel classes, measured the same way (event nodes around each kernel)
                "classes": {k: {"avg_launch_us": prof[k]["ms"] * 1000.0 / max(prof[k]["launches"], 1),
                                "achieved_gbs": prof[k]["bytes"] / (prof[k]["ms"] / 1000.0) / 1e9 if prof[k]["ms"] else 0.0,
                                "frac": (prof[k]["bytes"] / (prof[k]["ms"] / 1000.0) / 1e9 / peaks["hbm_gbs"]
                                         if prof[k]["ms"] else 0.0),
                                "ms_per_job": prof[k]["ms"]}
                            for k in ("attention", "linear")}}
    cpu = None
    if world == 1:
        threads = os.cpu_count() or 1
        cpu = cpu_baseline(w, params, threads, min(threads, w.seqs), w.new_tokens)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": w.name, "seqs_per_gpu": w.seqs, "prompt_len": w.prompt_len, "new_tokens": w.new_tokens,
                   "global_batch": world * w.seqs, "seq_len": w.prompt_len + w.new_tokens,
                   "parallelism": f"sequence shards x{world} (full weight replica per GPU, no collective in the step)",
                   "weights": f"reference init seed {w.weight_seed} (fp32 master -> bf16)",
                   "l2": "flushed (512 MiB write) before every timed step", "output_checksums": checksums},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": int(prompts.nbytes + offs.nbytes),
                "d2h_bytes_per_step": int(w.seqs * w.new_tokens * 4)},
        "roofline": roofline,
        "roofline_step": step_roofline(w, ms_per_step, peaks, peak_kind),
        "cpu_baseline": cpu,
        "clocks": clk,
        "gpu_launches": int(launches),
        "kernel_classes_ms_per_job": {k: v["ms"] for k, v in prof.items()},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="microchat", choices=sorted(pkg.configs.WORKLOADS))
    ap.add_argument("--no-extras", action="store_true",
                    help="time the steps only (no e2e, profile or CPU legs): the profiling command line")
    ap.add_argument("--chains", type=int, default=0, help="concurrent decode chains (0 = library default)")
    ap.add_argument("--tc-min-rows", type=int, default=0, help="rows from which projections use tensor cores (0 = default)")
    ap.add_argument("--new-tokens", type=int, default=None,
                    help="override the workload's new tokens per sequence (small ncu captures only)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.warmup < 3:
        args.warmup = 3
    if args.new_tokens is not None:
        import dataclasses
        w = pkg.configs.WORKLOADS[args.workload]
        pkg.configs.WORKLOADS[args.workload] = dataclasses.replace(w, new_tokens=args.new_tokens)
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
