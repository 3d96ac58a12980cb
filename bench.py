#!/usr/bin/env python
"""Throughput of the compiled RV32IM stack on B200: trace tokens/s of free-running machines.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (one rank per GPU)

Workload: the bignum-heavy mix of seeded RV32IM programs (40% MUL/MULH/DIVU chains, 20% loads /
stores over a 16 KB range, the rest like the base generator): ``--machines`` (4,096) independent
machines of the whole job, split evenly over the ranks ("scaling": "strong": 4,096 on one GPU,
512 on each of eight), started from their program images.  ``--weak`` instead runs
``--machines`` on every rank (programs seeded per rank), so the job grows with the GPUs.
A step is one launch of the persistent token kernel: ``--tokens-per-step`` free-running tokens
for every local machine (each token is decoded into the next input on the device).  With fewer
machines per GPU a CTA runs a smaller group of machines (16, 8 or 4, its warps running 2, 4 or 8
stream records side by side), so the SMs stay busy with independent CTAs.  Ranks exchange nothing per step; one NCCL all-gather of the per-machine state
checksums closes the run.  The head states (12.5 MB per machine, 51 GB on one GPU) are far larger
than L2, so no flush is needed between steps.

The JSON line also carries the gated delta-rule decode-step microbenchmark (1,024 sequences x 48
heads, dk = dv = 128) with its HBM roofline.

``--impl reference`` times the reference algorithm on the host cores instead: the C restatement
of the reference executor's step and decode (oracle/), all threads, on a bounded sample of the
same workload (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "rv32im_trace_tokens_per_s"
# DRAM bytes per machine-token of the token kernel: ncu captures of 256 machines x 4 tokens
# (dram__bytes_read.sum + dram__bytes_write.sum), per machine-token: groups of 32 machines
# (11.37 MB + 0 B) and bundled groups of 4 (11.84 MB + 16.9 KB; used for every bundled group)
DRAM_BYTES_PER_MACHINE_TOKEN = {32: 11.368192e6 / 1024, 4: (11.840512e6 + 16896) / 1024}
WORKLOAD = "rv32im free-run, bignum mix (40% MUL/MULH/DIVU chains, 20% LW/SW over 16 KB)"
UNIT = "tokens/s"
GO_TOKEN = 230322  # the run-start control (families then controls: NT .. HALT, GO, SC)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--machines", type=int, default=4096,
                    help="machines of the whole job (with --weak: on every GPU)")
    ap.add_argument("--weak", action="store_true",
                    help="run --machines on every rank instead of splitting them over the ranks")
    ap.add_argument("--cluster", type=int, default=None,
                    help="CTAs (a thread-block cluster) per group of 32 machines")
    ap.add_argument("--group", type=int, default=None, choices=[4, 8, 16, 32],
                    help="machines a CTA runs (default: the executor's choice by machines per GPU)")
    ap.add_argument("--tc", type=int, default=0, choices=[0, 1],
                    help="1: linear forms on the tensor cores (tcgen05), 0: on the CUDA cores")
    ap.add_argument("--tokens-per-step", type=int, default=200)
    ap.add_argument("--no-gdn", action="store_true")
    ap.add_argument("--gdn-sequences", type=int, default=1024,
                    help="sequences of the gated delta-rule microbenchmark (48 heads each)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--seed", type=int, default=1000)
    return ap.parse_args()


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                       "-i", str(gpu_index), "-lms", "200"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        rows = [r.split(",") for r in Path(self.f.name).read_text().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for nm, v in zip(names, r[5:9]):
                    if v.strip() == "Active":
                        reasons.add(nm)
            except (ValueError, IndexError):
                continue
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_baseline(programs, seconds: float = 12.0) -> dict:
    """The oracle (C restatement of the reference executor) on the host cores: teacher-free
    generation of a bounded sample of the same machines."""
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle
    from qwenputer_b200.graphfile import default_graph_path, load_graph

    g = load_graph(default_graph_path())
    o = oracle.Oracle(g)
    B = min(len(programs), 32)
    st = o.new_state(B)
    for r in range(B):
        o.snapshot(st, r, oracle.Machine.from_program(programs[r]))
    x = g.embed([GO_TOKEN] * B)
    cores = os.cpu_count() or 1
    o.step(st, x, nthreads=cores)
    x = o.decode(x)[1]
    n = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        o.step(st, x, nthreads=cores)
        x = o.decode(x)[1]
        n += 1
    dt = time.perf_counter() - t0
    return {"value": B * n / dt, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{B} machines x {n} free-running tokens of the same workload ({dt:.1f} s)"}


def gdn_bench(torch, steps: int, warmup: int, peak_gbs: float, B: int = 1024) -> dict:
    """One gated delta-rule decode step over B x 48 heads; bytes from the realised draws."""
    from qwenputer_b200.executor import gdn_step

    from qwenputer_b200 import workload

    H, D = 48, 128
    BH = B * H
    inp = workload.gdn_inputs(B, H, seed=7)
    bytes_ = workload.gdn_algorithmic_bytes(inp)
    S = inp["S"].to("cuda").float()
    q, k, v, alpha, beta = (inp[n] for n in ("q", "k", "v", "alpha", "beta"))
    q, k, v, alpha, beta = (t.cuda() for t in (q, k, v, alpha, beta))
    o = torch.empty(BH, D, device="cuda")
    from qwenputer_b200.executor import lib

    work = torch.empty(int(lib().qx_gdn_work_bytes(BH)), dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        gdn_step(S, q, k, v, alpha, beta, o, work)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        gdn_step(S, q, k, v, alpha, beta, o, work)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    gbs = bytes_ / (ms * 1e-3) / 1e9
    return {"config": {"sequences": B, "heads": H, "dk": D, "dv": D, "one_hot_keys": 0.95,
                       "alpha": {"1": 0.9, "0.5": 0.05, "0": 0.05}},
            "ms_per_step": ms, "bytes_per_step": bytes_, "achieved_gbs": gbs,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak_gbs, "unit": "GB/s",
                         "frac": gbs / peak_gbs},
            "launches_per_step": 2}


def job_config(args, world: int) -> dict:
    """The workload a run measures (both arms print the same): machines of the job and per GPU,
    tokens per step, how the job splits, and why no L2 flush is needed."""
    per_gpu = args.machines if args.weak else -(-args.machines // world)
    return {"workload": WORKLOAD, "machines_per_gpu": per_gpu,
            "machines_total": args.machines * (world if args.weak else 1),
            "tokens_per_step": args.tokens_per_step,
            "parallelism": f"machines sharded over {world} GPU(s)",
            "l2": f"no flush: {per_gpu * 12.5e6 / 1e9:.0f} GB of head states per GPU, far above L2"}


def reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from qwenputer_b200 import workload

    sys.path.insert(0, str(REPO / "oracle"))
    import oracle
    from qwenputer_b200.graphfile import default_graph_path, load_graph

    B = min(args.machines, 64)
    progs = workload.workload_programs("bignum", B, args.seed)
    g = load_graph(default_graph_path())
    o = oracle.Oracle(g)
    st = o.new_state(B)
    for r in range(B):
        o.snapshot(st, r, oracle.Machine.from_program(progs[r]))
    x = g.embed([GO_TOKEN] * B)
    cores = os.cpu_count() or 1
    tps = 16  # tokens per step of the CPU sample

    def step(x):
        for _ in range(tps):
            o.step(st, x, nthreads=cores)
            x = o.decode(x)[1]
        return x

    for _ in range(args.warmup):
        x = step(x)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        x = step(x)
    dt = time.perf_counter() - t0
    val = B * tps * args.steps / dt
    sample = (f"each step: {B} of the job's machines x {tps} free-running tokens (a bounded sample of "
              f"a step's {args.machines} x {args.tokens_per_step}) on {cores} host threads")
    emit({
        "impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak" if args.weak else "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic: seeded RV32IM programs (bignum mix)",
        "config": job_config(args, args.gpus),
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })


_JSON_FD = None


def emit(line: dict) -> None:
    """The one JSON line, on the process's original stdout."""
    os.write(_JSON_FD if _JSON_FD is not None else 1, (json.dumps(line) + "\n").encode())


def main() -> None:
    global _JSON_FD
    # stdout carries only the JSON line: anything else written to fd 1 (library banners such as
    # NCCL's version line) goes to stderr
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    import numpy as np
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    from qwenputer_b200 import workload
    from qwenputer_b200.executor import Executor

    from qwenputer_b200.shard import combine, gather_checksums, shard

    B, seed0 = shard(args.machines, world, rank, args.weak, args.seed)
    progs = workload.workload_programs("bignum", B, seed0)
    ex = Executor(None, batch=B, cluster=args.cluster, tc=bool(args.tc), group=args.group)
    ex.load_machines(0, progs)
    ex.reset()
    ex.set_tokens(0, [GO_TOKEN] * B)
    tps = args.tokens_per_step
    tokens = torch.empty(tps, B, dtype=torch.int32, device="cuda")
    peak, peak_kind = peaks()

    def barrier():
        if dist:
            dist.barrier()

    for _ in range(args.warmup):
        ex.run(tps, tokens)
    torch.cuda.synchronize()
    sb0 = int(ex.state_bytes.cpu().numpy().view(np.uint64)[0])
    barrier()
    torch.cuda.synchronize()
    gpu_index = local
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            gpu_index = int(vis.split(",")[local])
        except (ValueError, IndexError):
            pass
    clk = Clocks(gpu_index)
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        ex.run(tps, tokens)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = clk.stop()
    ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    sb1 = int(ex.state_bytes.cpu().numpy().view(np.uint64)[0])
    total_tokens = B * world * tps * args.steps
    value = total_tokens / (ms * 1e-3)
    ms_per_step = ms / args.steps
    # roofline of the token kernel (one launch per step): weights read once per GPU per token
    # + the head-state rows touched (counted on the device)
    w_bytes = float(ex.plan.stats["weight_bytes"])
    state_per_launch = (sb1 - sb0) / args.steps
    alg_bytes = tps * w_bytes + state_per_launch
    achieved = alg_bytes / (ms_per_step * 1e-3) / 1e9
    macs_per_mtok = ex.plan.stats["form_nnz"] + ex.plan.stats["units"]

    # checksums of every machine's state: the one collective
    sums = ex.checksums()
    combined = combine(gather_checksums(sums, dist))
    errs = ex.errors()

    # end to end through the public API: per step, the machines' images go host -> device, the
    # device builds their states, the step runs and the generated tokens come back to pinned host
    # memory.  Two executors alternate (double buffering): while step k runs on the run stream,
    # step k + 1's machines are copied and built into the other executor on a load stream (its
    # previous run finished first); the timed region holds every step's copies in both directions,
    # the first step's load included
    e2e = None
    if not args.no_e2e:
        from qwenputer_b200.executor import Machine, lib, program_image, check
        import ctypes as C

        keep: list = []
        imgs = (Machine * B)(*[program_image(p, keep) for p in progs])
        h2d = sum(int(im.rom_words) * 4 + int(im.drom_bytes) + 8192 * 4 + 34 * 4 for im in imgs)
        go = np.full(B, GO_TOKEN, np.int32)
        exs = [ex, Executor(None, batch=B, cluster=args.cluster, tc=bool(args.tc), group=args.group)]
        run_s, load_s = torch.cuda.Stream(), torch.cuda.Stream()
        toks = [tokens, torch.empty_like(tokens)]
        host_tok = [torch.empty(tps, B, dtype=torch.int32, pin_memory=True) for _ in range(2)]
        ran = [torch.cuda.Event(), torch.cuda.Event()]

        def load(i):
            load_s.wait_event(ran[i])  # (the executor's previous run is done with its state)
            check(lib().qx_load_machines(exs[i].h, 0, B, imgs, C.c_void_p(load_s.cuda_stream)), "qx_load_machines")

        for i in range(2):  # untimed: staging buffers grow to size, both executors warm
            ran[i].record(run_s)
            load(i)
            with torch.cuda.stream(run_s):
                exs[i].reset()
                exs[i].set_tokens(0, go)
                exs[i].run(tps, toks[i])
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        n_e2e = max(2, min(args.steps, 6))
        t0 = time.perf_counter()
        load(0)
        for k in range(n_e2e):
            i = k % 2
            with torch.cuda.stream(run_s):
                exs[i].reset()
                exs[i].set_tokens(0, go)
                exs[i].run(tps, toks[i])
                host_tok[i].copy_(toks[i], non_blocking=True)
                ran[i].record(run_s)
            if k + 1 < n_e2e:
                load(1 - i)  # overlaps step k's run
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        del exs[1]
        if dist:
            t = torch.tensor([dt], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dt = float(t.item())
        e2e = {"value": B * world * tps * n_e2e / dt, "unit": UNIT, "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": tps * B * 4, "steps": n_e2e,
               "includes": "per step: machine images H2D + device snapshot build + run + tokens D2H, "
                           "wall clock; two executors alternate, the next step's images load while "
                           "a step runs"}

    gdn = None
    if not args.no_gdn and rank == 0:
        gdn = gdn_bench(torch, max(args.steps, 5), args.warmup, peak, args.gdn_sequences)
    cpu = None
    if not args.no_cpu and rank == 0 and world == 1:
        cpu = cpu_baseline(progs)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak" if args.weak else "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: seeded RV32IM programs (bignum mix), machines start from their images",
            "config": job_config(args, world),
            "launch": {"machines_per_cta_group": ex.group, "ctas_per_group": ex.cluster,
                       "groups_per_gpu": -(-B // ex.group), "ctas": ex.info(2),
                       "forms_on": "tensor cores (tcgen05)" if args.tc else "CUDA cores"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": DRAM_BYTES_PER_MACHINE_TOKEN[32 if ex.group == 32 else 4] * B * tps,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of a "
                                           f"256-machine x 4-token launch at groups of {32 if ex.group == 32 else 4}, "
                                           "scaled by machine-tokens",
                         "algorithmic_bytes_per_launch": alg_bytes,
                         "weight_bytes_per_token": w_bytes,
                         "state_bytes_per_machine_token": state_per_launch / (tps * B)},
            "compute": {"macs_per_machine_token": macs_per_mtok,
                        "tmacs_per_s": macs_per_mtok * B * tps / (ms_per_step * 1e-3) / 1e12,
                        "note": "fp32 CUDA-core FMAs over smem-resident residuals"},
            "clocks": clocks, "gpu_launches": args.steps,
            "e2e": e2e, "cpu_baseline": cpu, "gdn_step": gdn,
            "checksum_xor": f"{combined:016x}", "device_errors": errs,
        }
        emit(line)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
