"""Benchmark of the sampling path: sampled rows/s at V=128256, B=2048, bf16.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One process per GPU (torchrun for N > 1).  Every rank samples its own batch of
B=2048 rows (batch partitioning, weak scaling, no collective on the data path).
A step is one tg_sample call over one batch; inputs are resident in HBM and two
input sets (2 x 525 MB, larger than L2) alternate between steps.  Times are CUDA
events on the launching stream, barrier + synchronize on both sides, max over
ranks.  `e2e` repeats the measurement through tg_sample_host with pinned host
buffers (host->device copy of the step's inputs and device->host copy of the ids
inside the timed region).  `--impl reference` times the CPU restatement of the
reference sampler (oracle/, all host threads) on bounded samples of the same
workload.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

V = 128256
B = 2048
HIST = 512
METRIC = "sampled rows/sec at V=128256 B=2048 bf16; % of HBM roofline at 1/2/4/8 GPU"
BYTES_PER_ROW = V * 2 + HIST * 4  # logits once + history ids (258,560 B)
PROFILE_SUMMARY = os.path.join(ROOT, "profiles", "stream_kernel_config4.json")


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def make_inputs_gpu(torch, dev, seed, B=B):
    """Config-4 inputs built on the device: N(0,3^2) + Zipf(1.1) bias over a
    per-row affine permutation, k~U{1..1024}, p~U[0.5,1], T~U[0.3,1.2],
    repetition 1.05 over 512 Zipf history ids."""
    from tinygpt_b200 import workloads as W
    g = torch.Generator(device=dev).manual_seed(seed)
    hg = W.rng(seed)
    perm = W._AffinePerm(hg, B, V)
    x = torch.randn((B, V), generator=g, device=dev, dtype=torch.float32) * 3.0
    rank_bias = (-1.1 * torch.log(torch.arange(1, V + 1, device=dev, dtype=torch.float64))).float()
    v = torch.arange(V, device=dev, dtype=torch.int64)[None, :]
    c = torch.from_numpy(perm.c).to(dev)[:, None]
    ai = torch.from_numpy(perm.ainv).to(dev)[:, None]
    for i in range(0, B, 256):
        x[i:i + 256] += rank_bias[((v - c[i:i + 256]) % V * ai[i:i + 256]) % V]
    logits = x.to(torch.bfloat16)
    del x
    p = np.zeros(B, W.ROW_PARAMS_DTYPE)
    p["top_k"] = hg.integers(1, 1025, size=B)
    p["top_p"] = hg.uniform(0.5, 1.0, size=B)
    p["temperature"] = hg.uniform(0.3, 1.2, size=B)
    p["repetition_penalty"] = 1.05
    hist = perm.token(W._zipf_ranks(hg, (B, HIST), V))
    u = hg.random(B, dtype=np.float32)
    return dict(logits=logits, params=p, history=hist, history_len=np.full(B, HIST, np.int32),
                uniforms=u)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms in the background."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.rows = []
        self.proc = None

    def __enter__(self):
        if not self.gpus:
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={','.join(map(str, self.gpus))}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([time.time()] + [f.strip() for f in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            self.proc.wait()

    def summary(self, t0=0.0, t1=float("inf")):
        rows = [r[1:] for r in self.rows if t0 <= r[0] <= t1 and len(r) >= 10]
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(sm)}


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def profile_traffic():
    try:
        with open(PROFILE_SUMMARY) as f:
            return json.load(f).get("dram_bytes_per_launch")
    except (OSError, ValueError):
        return None


def use_all_host_threads() -> int:
    """The oracle's OpenMP pool sized to every host core (torchrun sets
    OMP_NUM_THREADS=1 per rank); must run before the oracle library loads."""
    n = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(n)
    return n


def cpu_baseline(rows_logits_bf16: np.ndarray, p, hist, hlen, u, budget_s=10.0):
    """The oracle on the host cores over repeated bounded samples of the workload."""
    use_all_host_threads()
    from oracle import oracle
    oracle.build()
    n = rows_logits_bf16.shape[0]
    oracle.sample(rows_logits_bf16[:8], p[:8], hist[:8], hlen[:8], None, None, u[:8])  # warm
    done = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        oracle.sample(rows_logits_bf16, p, hist, hlen, None, None, u)
        done += n
    dt = time.perf_counter() - t0
    return done / dt, done, dt


def run_reference(args, rank, world):
    if rank != 0:
        return
    cores = use_all_host_threads()
    from tinygpt_b200 import workloads as W
    w = W.make(4, seed=1, batch=512)
    from oracle import oracle
    oracle.build()
    step = lambda: oracle.sample(w["logits"], w["params"], w["history"], w["history_len"], None,  # noqa: E731
                                 None, w["uniforms"])
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    rows = args.steps * 512
    val = rows / dt
    line = {"impl": "reference", "metric": METRIC, "value": val, "unit": "rows/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config 4: large-batch serving, V=128256, bf16 logits, 512 rows per step sample of B=2048",
                       "vocab": V, "rows_per_step": 512, "logits_dtype": "bf16"},
            "cpu_baseline": {"value": val, "unit": "rows/s", "cores": cores, "kind": "port",
                             "sample": f"{args.steps} steps x 512 rows of config 4, oracle/tgs_oracle.c "
                                       "(C restatement of python_ref/model.py:213-224 + wasm/src/model.cpp:489-517), "
                                       f"OpenMP over {cores} threads"},
            "e2e": {"value": val, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_config(args):
    """One JSON line for one of the five workloads (`--config N`, one GPU): the
    device time of a tg_sample / tg_spec_verify call on resident inputs, CUDA
    events over `--steps` calls (configs 1 and 2: calls replayed from a CUDA graph, the
    latency of one call).  Inputs come from tinygpt_b200.workloads (the
    oracle-checked workloads); configs 3-5 exceed L2 (two sets alternate for 3
    and 4; config 5 is 722 MB per call), configs 1-2 are L2-resident."""
    import torch
    from tinygpt_b200 import workloads as W
    from tinygpt_b200.sampler import Sampler, params_to_device
    cfg = args.config
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    c = W.CONFIGS[cfg]
    Vc, Bc = c["vocab"], c["batch"]
    s = Sampler(Vc, Bc, 0)
    sets = [W.make(cfg, seed=1 + i) for i in range(2 if cfg in (3, 4) else 1)]
    if args.variant != "none":  # the same rows without top-k (top-p only, or plain temperature)
        for w in sets:
            w["params"]["top_k"] = 0
            if args.variant == "temp":
                w["params"]["top_p"] = 1.0

    def to_dev(w):
        d = {}
        if cfg == 5:
            d["t"] = torch.from_numpy(w["target"].astype(np.float32)).to(dev)
            d["d"] = torch.from_numpy(w["draft"].astype(np.float32)).to(dev)
            for k in ("draft_ids", "temperature", "u_accept", "u_draw"):
                d[k] = torch.from_numpy(np.ascontiguousarray(w[k])).to(dev)
            return d
        x = w["logits"]
        t = torch.from_numpy(np.ascontiguousarray(x))
        if x.dtype == np.uint16:
            t = t.view(torch.int16).view(torch.bfloat16)
        opt = lambda k: torch.from_numpy(w[k]).to(dev) if w.get(k) is not None else None  # noqa: E731
        d.update(x=t.to(dev), p=params_to_device(w["params"], dev), u=opt("uniforms"),
                 h=opt("history"), hl=opt("history_len"), sid=opt("state_id"),
                 m=torch.from_numpy(w["mask_table"].view(np.int32)).to(dev) if w.get("mask_table") is not None else None)
        return d

    ds = [to_dev(w) for w in sets]
    out = torch.empty(Bc, dtype=torch.int32, device=dev)

    def call(i):
        d = ds[i % len(ds)]
        st = torch.cuda.current_stream()
        if cfg == 5:
            s.spec_verify(d["t"], d["d"], d["draft_ids"], d["temperature"], d["u_accept"], d["u_draw"], stream=st)
        else:
            s.sample(d["x"], d["p"], history=d["h"], history_len=d["hl"], mask_table=d["m"],
                     state_id=d["sid"], uniforms=d["u"], out=out, stream=st)

    for i in range(max(args.warmup, 3)):
        call(i)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    loop_us = None
    if cfg == 2:  # the same calls issued from the host one by one (bound by the host loop)
        e0.record(stream)
        for i in range(args.steps):
            call(i)
        e1.record(stream)
        torch.cuda.synchronize()
        loop_us = e0.elapsed_time(e1) * 1e3 / args.steps
    if cfg in (1, 2):  # latency-bound sizes: a graph of G calls, replayed (no host launch gaps)
        G = 100
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(G):
                call(i)
        g.replay()
        torch.cuda.synchronize()
        reps = max(1, args.steps // G)
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
        calls = reps * G
    else:
        e0.record(stream)
        for i in range(args.steps):
            call(i)
        e1.record(stream)
        calls = args.steps
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / calls
    peak, peak_kind = measured_peak()
    bytes_call = W.bytes_per_row(cfg) * Bc
    achieved = bytes_call / (us * 1e-6) / 1e9
    name = c["name"] + ("" if args.variant == "none" else f", {args.variant} variant (top_k = 0"
                        + (", top_p = 1" if args.variant == "temp" else "") + ")")
    line = {"metric": f"config {cfg} ({name}): device time per call", "value": us, "unit": "us",
            "higher_is_better": False, "n_gpus": 1, "steps": calls, "warmup": args.warmup,
            "rows_per_s": Bc / (us * 1e-6), "dtype": c["dtype"],
            "data": "synthetic (tinygpt_b200.workloads, seeded Philox)",
            "config": {"workload": f"config {cfg}", "vocab": Vc, "batch": Bc,
                       "l2": "inputs larger than L2, two sets alternate" if cfg in (3, 4) else
                             ("722 MB per call, larger than L2" if cfg == 5 else "L2-resident (latency-bound size)"),
                       "timing": "CUDA graph of 100 calls, replayed" if cfg in (1, 2) else "CUDA events over back-to-back calls"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "algorithmic_bytes_per_call": bytes_call,
                         "peak_source": peak_kind}}
    if loop_us is not None:
        line["host_loop_us_per_call"] = loop_us
    if cfg == 3:  # the 64 mask rows are read from L2 after the first touch: count the table once per call
        once = Vc * 4 * Bc + sets[0]["mask_table"].nbytes
        a1 = once / (us * 1e-6) / 1e9
        line["roofline_mask_table_once"] = {"achieved": a1, "frac": a1 / peak, "algorithmic_bytes_per_call": once,
                                            "note": "logits per row + the whole mask table once"}
    print(json.dumps(line), flush=True)
    s.close()


def vocab_sharded_leg(torch, dist, s_full, dev, rank, world, local, args, steps=20):
    """tg_sample_sharded over the job's ranks: every rank holds a 1/world slice of
    the SAME config-4 rows, one NCCL all-gather of per-row records, identical
    merge on every rank.  Returns rows/s of the whole job (B rows per call), and
    whether the ids equal tg_sample on the whole rows on every rank."""
    from tinygpt_b200.dist import NcclComm
    from tinygpt_b200.sampler import Sampler, params_to_device
    if V % world:
        return {"skipped": f"vocab {V} not divisible by {world}"}
    w = make_inputs_gpu(torch, dev, 4242)  # the same seed on every rank: the same rows
    width = V // world
    v0 = rank * width
    shard = w["logits"][:, v0:v0 + width].contiguous()
    p = params_to_device(w["params"], dev)
    hist = torch.from_numpy(w["history"]).to(dev)
    hlen = torch.from_numpy(w["history_len"]).to(dev)
    u = torch.from_numpy(w["uniforms"]).to(dev)
    ref, _ = s_full.sample(w["logits"], p, history=hist, history_len=hlen, uniforms=u)
    comm = NcclComm(rank, world, local)
    ss = Sampler(width, B, local)
    ss.reserve(max_ranks=world)
    out = torch.empty(B, dtype=torch.int32, device=dev)
    call = lambda: ss.sample_sharded(comm.ptr, world, shard, p, v0, V, history=hist, history_len=hlen,  # noqa: E731
                                     uniforms=u, out=out)
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    same = torch.tensor([int(torch.equal(out, ref))], device=dev)
    dist.all_reduce(same, op=dist.ReduceOp.MIN)
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        call()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item()) / steps
    ss.close()
    comm.close()
    return {"rows_per_s": B / (ms / 1e3), "ms_per_call": ms, "rows_per_call": B, "shards": world,
            "ids_equal_batch_mode": bool(same.item()),
            "note": "each rank holds V/N ids of the same rows; local top-k records, one ncclAllGather, merge"}


def batch_8192_leg(torch, dev, local, args, steps=20):
    """Config 4 at its larger batch (8192 rows: four launch pairs of 2048)."""
    from tinygpt_b200.sampler import Sampler, params_to_device
    Bb = 8192
    w = make_inputs_gpu(torch, dev, 8192, B=Bb)
    s = Sampler(V, Bb, local)
    p = params_to_device(w["params"], dev)
    hist = torch.from_numpy(w["history"]).to(dev)
    hlen = torch.from_numpy(w["history_len"]).to(dev)
    u = torch.from_numpy(w["uniforms"]).to(dev)
    out = torch.empty(Bb, dtype=torch.int32, device=dev)
    call = lambda: s.sample(w["logits"], p, history=hist, history_len=hlen, uniforms=u, out=out)  # noqa: E731
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        call()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    s.close()
    del w
    peak, _ = measured_peak()
    gbs = Bb * BYTES_PER_ROW / (ms / 1e3) / 1e9
    return {"rows_per_s": Bb / (ms / 1e3), "ms_per_call": ms, "steps": steps,
            "step_frac_of_peak": gbs / peak, "note": "2.1 GB of logits per call, the L2 holds none of it"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--profile-steps", type=int, default=50,
                    help="untimed steps whose per-kernel CUDA-event times give the roofline")
    ap.add_argument("--config", type=int, default=0, choices=[0, 1, 2, 3, 4, 5],
                    help="1-5: one line for that workload's call time (one GPU) instead of the headline")
    ap.add_argument("--variant", default="none", choices=["none", "topp", "temp"],
                    help="with --config 1-4: the same rows without top-k (topp) or with temperature only (temp)")
    args = ap.parse_args()
    if args.config:
        run_config(args)
        return
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist
    from tinygpt_b200 import _lib
    from tinygpt_b200.sampler import Sampler, params_to_device

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    L = _lib.load()
    s = Sampler(V, B, local)

    sets = [make_inputs_gpu(torch, dev, 1000 + 17 * rank + i) for i in range(2)]
    dsets = []
    for w in sets:
        dsets.append(dict(
            logits=w["logits"], params=params_to_device(w["params"], dev),
            hist=torch.from_numpy(w["history"]).to(dev), hlen=torch.from_numpy(w["history_len"]).to(dev),
            u=torch.from_numpy(w["uniforms"]).to(dev)))
    out = torch.empty(B, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    sptr = ctypes.c_void_p(stream.cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    argsets = [(P(d["logits"]), _lib.TG_DTYPE_BF16, V, B, P(d["params"]), P(d["hist"]), P(d["hlen"]),
                HIST, None, 0, None, P(d["u"]), P(out), None, sptr) for d in dsets]

    def step(i):
        rc = L.tg_sample(s.handle, *argsets[i & 1])
        if rc != 0:
            _lib.check(rc)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(args.warmup):
        step(i)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # one nvidia-smi sampler per node (rank 0, every GPU of the job); the clock
    # record spans the timed steps and 0.5 s of the same steps right after them,
    # so it holds samples even when the timed region is a few milliseconds
    sampler_gpus = list(range(world)) if rank == 0 else []
    with ClockSampler(sampler_gpus) as clk:
        if sampler_gpus:
            time.sleep(0.5)  # let the sampler start
        barrier()
        tw0 = time.time()
        e0.record(stream)
        for i in range(args.steps):
            step(i)
        e1.record(stream)
        barrier()
        ms = e0.elapsed_time(e1)
        t_end = time.time() + 0.5
        i = 0
        while time.time() < t_end:
            for _ in range(20):
                step(i)
                i += 1
            torch.cuda.synchronize()
        barrier()
        tw1 = time.time()
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    rows = B * args.steps * world
    value = rows / (ms_max / 1e3)
    peak, peak_kind = measured_peak()
    # per-kernel device times of the same steps (untimed pass, CUDA events
    # recorded by the library around its kernels on the launching stream)
    ktimes = []
    s.profile(True)
    for i in range(args.profile_steps):
        step(i)
        ktimes.append(s.profile(True))
    s.profile(False)
    nk = len(ktimes[-1])
    kms = [float(np.mean([k[j] for k in ktimes])) for j in range(nk)]
    if nk == 2:  # two-kernel mode: the streaming kernel reads the logits once
        dom_ms, dom_bytes = kms[0], B * V * 2
        dom_name, dom_share = "tg::sample_kernel<1, true> (streaming half)", kms[0] / (kms[0] + kms[1])
    else:
        dom_ms, dom_bytes = kms[0], B * BYTES_PER_ROW
        dom_name, dom_share = "tg::sample_kernel<1>", 1.0
    achieved = dom_bytes / (dom_ms / 1e3) / 1e9
    step_achieved = B * BYTES_PER_ROW / (ms / args.steps / 1e3) / 1e9

    # ---- e2e through the host-buffer entry point (pinned host memory) -------
    w = sets[0]
    h_logits = torch.empty((B, V), dtype=torch.bfloat16, pin_memory=True)
    h_logits.copy_(w["logits"])
    hl = h_logits.view(torch.int16).numpy().view(np.uint16)
    pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory().numpy()  # noqa: E731
    hp = pin(w["params"].view(np.int32)).view(w["params"].dtype)
    hh, hn, hu = pin(w["history"]), pin(w["history_len"]), pin(w["uniforms"])
    hout = pin(np.zeros(B, np.int32))
    for _ in range(2):
        s.sample_host(hl, hp, history=hh, history_len=hn, uniforms=hu)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        o, _ = s.sample_host(hl, hp, history=hh, history_len=hn, uniforms=hu)
    e2e_local_s = time.perf_counter() - t0
    dt = torch.tensor([e2e_local_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(dt, op=dist.ReduceOp.MAX)
    e2e_val = B * args.e2e_steps * world / float(dt.item())
    h2d = B * V * 2 + B * 32 + B * HIST * 4 + B * 4 + B * 4
    d2h = B * 4
    del hout

    # per-rank figures (the max over ranks decides `value`; these name the slow rank)
    mine = torch.tensor([ms / args.steps] + kms + [h2d * args.e2e_steps / e2e_local_s / 1e9],
                        dtype=torch.float64, device=dev)
    if world > 1:
        allr = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allr, mine)
    else:
        allr = [mine]
    per_rank = [{"rank": r, "ms_per_step": float(x[0]), "kernel_ms": [float(v) for v in x[1:-1]],
                 "e2e_h2d_gbs": float(x[-1])} for r, x in enumerate(allr)]
    vsh = vocab_sharded_leg(torch, dist, s, dev, rank, world, local, args) if world > 1 else None
    b8192 = batch_8192_leg(torch, dev, local, args) if world == 1 else None

    cpu = None
    if rank == 0 and world == 1:
        from tinygpt_b200 import workloads as W
        sub = slice(0, 512)
        lg = w["logits"][sub].contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
        val, done, secs = cpu_baseline(lg, w["params"][sub], w["history"][sub], w["history_len"][sub],
                                       w["uniforms"][sub], args.cpu_budget)
        cpu = {"value": val, "unit": "rows/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"{done} rows of config 4 in {secs:.1f} s (512-row slices of the bench batch), "
                         "oracle/tgs_oracle.c with OpenMP over all host threads"}

    if rank == 0:
        clocks = clk.summary(tw0, tw1)
        line = {
            "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,3^2) + Zipf(1.1) bias, built on device)",
            "config": {"workload": "config 4: large-batch serving, V=128256, B=2048 rows per GPU, bf16 logits, "
                                   "per-row top-k U{1..1024}, top-p U[0.5,1], T U[0.3,1.2], repetition 1.05 over 512 ids",
                       "vocab": V, "rows_per_gpu": B, "logits_dtype": "bf16", "parallelism": f"batch-sharded x{world}",
                       "l2": "two 525 MB input sets alternate (each larger than the 126 MB L2)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": profile_traffic(),
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
                         "kernel": dom_name, "kernel_ms": dom_ms, "kernel_share_of_step": dom_share,
                         "algorithmic_bytes_per_launch": dom_bytes,
                         "kernel_ms_all": kms,
                         "step": {"achieved": step_achieved, "frac": step_achieved / peak,
                                  "bytes_per_row": BYTES_PER_ROW,
                                  "note": "whole step (every kernel) against the logits, history and id bytes"}},
            "e2e": {"value": e2e_val, "unit": "rows/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": args.e2e_steps,
                    "path": "tg_sample_host, pinned host buffers"},
            "gpu_launches": args.steps * (3 if nk == 2 else 1),
            "clocks": dict(clocks, window="the timed steps + 0.5 s of the same steps right after them"),
            "per_rank": per_rank,
        }
        if vsh:
            line["vocab_sharded"] = vsh
        if b8192:
            line["b8192"] = b8192
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    s.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
