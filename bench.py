"""Benchmark: one optimizer step of AdamW_adv(state_precision='int8_sr',
factored_2nd=True, nesterov=True) over Llama-3-8B parameter shapes in bf16
(8.03e9 parameters, 291 tensors), synthetic params ~N(0, 0.02^2) and grads
~N(0, 1e-3^2) with 1% of entries x100.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  With N > 1 (torchrun) every rank owns a
time-balanced share of the tensors (per-tensor sharding) and steps only
those, then every rank pulls the others' updated bf16 parameters with its
copy engines over NVLink (CUDA IPC mappings; NCCL fences order the pulls);
the timed step includes that gather.  `--impl reference` times the CPU
restatement of the reference's step (oracle/) on this host's cores.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOAD = "adamw_adv int8_sr+factored_2nd+nesterov, llama-3-8b shapes, bf16"
# DRAM bytes (read + write) of adam_fast_kernel per algorithmic byte, from one ncu
# capture of the 2-layer subset:
# 3.476 GB measured / 3.493 GB algorithmic.  Traffic grows with the elements processed,
# so the full launch's traffic is reported as this ratio times its algorithmic bytes.
TRAFFIC_PER_ALG_BYTE = 3.476247e9 / 3.492700320e9


def llama3_8b_shapes(layers=32, embed=True):
    d, kv, ffn, V = 4096, 1024, 14336, 128256
    s = [(V, d), (V, d)] if embed else []
    for _ in range(layers):
        s += [(d, d), (kv, d), (kv, d), (d, d), (ffn, d), (ffn, d), (d, ffn), (d,), (d,)]
    return s + [(d,)]


def algorithmic_bytes(shapes):
    """Mandatory HBM bytes of one step: bf16 p read+write, bf16 g read, int8 m
    read+write (+ fp32 block scale read+write); 1-D tensors also uint8 v
    read+write (+ scale); 2-D tensors read and write their fp32 row/column
    factors."""
    from advanced_optimizers_b200._plan import effective_shape
    tot = 0
    for sh in shapes:
        n = math.prod(sh)
        nb = (n + 2047) // 2048
        tot += n * (2 + 2 + 2 + 1 + 1) + nb * 8
        if len(sh) == 1:
            tot += n * 2 + nb * 8
        else:
            d1, d2 = effective_shape(n)
            tot += (d1 + d2) * 8
    return tot


def sample_clocks_start(path):
    """nvidia-smi sampling every 50 ms, started before the warm-up so that it
    is running when the timed region begins; each sample carries its time."""
    try:
        f = open(path, "w")
        p = subprocess.Popen(
            ["nvidia-smi", "--query-gpu=timestamp,index,clocks.sm,clocks.max.sm,power.draw,"
             "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
             "--format=csv,noheader,nounits", "-lms", "50"], stdout=f, stderr=subprocess.DEVNULL)
        return p, f
    except Exception:
        return None, None


def sample_clocks_stop(proc, f, path, gpu_index, t0=None, t1=None):
    """Median SM clock and the throttle reasons seen between host times t0 and
    t1 (the timed region); a region shorter than the sampling period takes
    the sample nearest to it."""
    import datetime
    if proc is None:
        return None
    proc.terminate()
    try:
        proc.wait(timeout=5)
    except Exception:
        proc.kill()
    f.close()
    rows = []
    for line in open(path):
        parts = [x.strip() for x in line.split(",")]
        if len(parts) < 10 or parts[1] != str(gpu_index):
            continue
        try:
            ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
        except ValueError:
            ts = None
        try:
            rows.append((ts, float(parts[2]), float(parts[3]), parts[6:10]))
        except ValueError:
            continue
    if not rows:
        return None
    timed = [r for r in rows if r[0] is not None]
    if t0 is None or len(timed) < len(rows):
        inside = rows
    else:
        inside = [r for r in timed if t0 - 0.05 <= r[0] <= t1 + 0.05]
        if not inside:
            mid = 0.5 * (t0 + t1)
            inside = [min(timed, key=lambda r: abs(r[0] - mid))]
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    reasons = set()
    for r in inside:
        for nm, val in zip(names, r[3]):
            if val.lower() == "active":
                reasons.add(nm)
    return {"sm_mhz": float(np.median([r[1] for r in inside])), "sm_max_mhz": float(max(r[2] for r in inside)),
            "reasons": sorted(reasons), "samples": len(inside)}


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return float(m["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# CPU baseline: the oracle (CPU restatement of the reference's step)
# ---------------------------------------------------------------------------

def llama3_8b_distinct():
    """The distinct Llama-3-8B tensor shapes and how many of the 291 tensors
    have each (embed/lm_head, q/o, k/v, gate/up, down, RMSNorm weights)."""
    d, kv, ffn, V = 4096, 1024, 14336, 128256
    return [((V, d), 2), ((d, d), 64), ((kv, d), 64), ((ffn, d), 64), ((d, ffn), 32), ((d,), 65)]


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


class OracleSample:
    """One oracle step per distinct Llama-3-8B shape, the way the reference
    runs its step: tensor after tensor, each op using every host core (the
    oracle's C primitives are OpenMP loops; its numpy parts run on one).  A
    full step's time is the sum over the 291 tensors of the measured time of
    their shape.  Shapes above 64M elements (the 525M-element embedding) are
    timed on a slab of whole rows and scaled by the element count (said in
    `describe()`), which keeps a sample to seconds."""

    def __init__(self, seed=0, cores=None, max_elems=64 << 20):
        from oracle import oracle as O
        self.O = O
        self.cores = int(cores or host_cores())
        O.set_num_threads(self.cores)
        try:
            import psutil
            avail = psutil.virtual_memory().available
        except Exception:
            avail = 64 << 30
        rng = np.random.default_rng(seed)
        self.hp = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, nesterov=True, precision="int8_sr")
        self.items = []
        self.slabbed = []
        for sh, mult in llama3_8b_distinct():
            n = math.prod(sh)
            scale = 1.0
            # at most max_elems per timed item (and what host memory holds:
            # float32 inputs, draws and the step's temporaries, ~64 B/element):
            # larger shapes are timed on a slab of whole rows
            cap = min(max_elems, int(0.5 * avail) // 64)
            if n > cap:
                k = math.ceil(n / cap)
                sh = (max(1, sh[0] // k),) + tuple(sh[1:])
                scale = n / math.prod(sh)
                self.slabbed.append((sh, scale))
                n = math.prod(sh)
            p = O.round_bf16((rng.standard_normal(n, dtype=np.float32) * 0.02).reshape(sh))
            g = rng.standard_normal(n, dtype=np.float32) * 1e-3
            g = np.where(rng.random(n, dtype=np.float32) < 0.01, g * 100, g).astype(np.float32)
            g = O.round_bf16(g.reshape(sh))
            st = O.adamw_init_state(sh, "bf16", "int8_sr", True, 0.9)
            pad = ((n + 2047) // 2048) * 2048
            nz = {"exp_avg": rng.integers(0, 65536, pad, dtype=np.int32),
                  "exp_avg_sq": rng.integers(0, 65536, pad, dtype=np.int32),
                  "param": rng.integers(0, 65536, n, dtype=np.int32)}
            self.items.append((sh, mult, scale, p, g, st, nz))

    def run(self):
        """One sample: (wall seconds of the sample, seconds of one full step)."""
        full = 0.0
        t_all = time.perf_counter()
        for sh, mult, scale, p, g, st, nz in self.items:
            t0 = time.perf_counter()
            self.O.adam_family_step(p, "bf16", g, st, self.hp, nz, algo="adamw")
            full += (time.perf_counter() - t0) * scale * mult
        return time.perf_counter() - t_all, full

    def describe(self, sample_s):
        s = (f"each sample: one oracle step per distinct Llama-3-8B shape (embed 128256x4096, q/o 4096x4096, "
             f"k/v 1024x4096, gate/up 14336x4096, down 4096x14336, norm 4096), in sequence, {self.cores} OpenMP "
             f"threads in the C primitives; full step = sum over the 291 tensors of their shape's time "
             f"(sample {sample_s:.1f} s)")
        if self.slabbed:
            s += "; timed on row slabs scaled by element count: " + ", ".join(
                f"{list(sh)} x{sc:.0f}" for sh, sc in self.slabbed)
        return s


def cpu_baseline():
    """The oracle's step on this host (one warm-up sample, one timed)."""
    smp = OracleSample()
    smp.run()
    wall, full = smp.run()
    return {"value": 1.0 / full, "unit": "optimizer steps/s", "cores": smp.cores, "kind": "port",
            "sample": smp.describe(wall), "full_step_s": full}


def run_reference(args):
    """The reference's CPU step on this host's cores (the oracle port: the
    reference is a Python package that does not travel), rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    shapes = llama3_8b_shapes()
    total = sum(math.prod(s) for s in shapes)
    smp = OracleSample()
    for _ in range(args.warmup):
        smp.run()
    walls, fulls = [], []
    for _ in range(args.steps):
        w, f = smp.run()
        walls.append(w)
        fulls.append(f)
    full = float(np.mean(fulls))
    value = 1.0 / full
    out = {"impl": "reference", "metric": "optimizer steps/s at Llama-3-8B shapes", "value": value,
           "unit": "optimizer steps/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
           # the timed samples' own wall time; full_step_ms is the whole step they stand for
           "ms_per_step": float(np.mean(walls)) * 1000, "full_step_ms": full * 1000,
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
           "dtype": "f32", "data": "synthetic",
           "config": {"workload": WORKLOAD, "params": total, "tensors": len(shapes),
                      "parallelism": f"per-tensor sharding x{args.gpus}",
                      "l2": "inputs larger than L2 (about 40 GB resident per step)"},
           "cpu_baseline": {"value": value, "unit": "optimizer steps/s", "cores": smp.cores, "kind": "port",
                            "sample": smp.describe(float(np.mean(walls)))},
           "e2e": {"value": value, "unit": "optimizer steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def run_ours(args):
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    import advanced_optimizers_b200 as A

    shapes = llama3_8b_shapes(args.layers, not args.no_embed)
    total = sum(math.prod(s) for s in shapes)
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    # every rank holds all bf16 params (they are all-gathered each step), but
    # grads and optimizer states only for the tensors it owns
    params = [torch.nn.Parameter(torch.empty(sh, dtype=torch.bfloat16, device=dev)) for sh in shapes]
    kw = dict(state_precision="int8_sr", factored_2nd=True, nesterov=True)
    if world > 1:
        # per-tensor sharding: parameters become views of rank-ordered flat
        # buffers (gather buckets), each refreshed by one asynchronous
        # all_gather_into_tensor while the next bucket is stepped
        sharded = A.ShardedOptimizer(A.AdamW_adv, params, **kw)
        owner = sharded.owner
    else:
        sharded = None
        owner = [0] * len(shapes)
    mine = [i for i in range(len(shapes)) if owner[i] == rank]
    owned = [params[i] for i in mine]
    with torch.no_grad():
        for p in owned:
            p.copy_(torch.randn(p.shape, generator=gen, device=dev) * 0.02)
    for p in owned:
        g = torch.randn(p.shape, generator=gen, device=dev, dtype=torch.float32).mul_(1e-3)
        mask = torch.rand(p.shape, generator=gen, device=dev) < 0.01
        g = torch.where(mask, g * 100, g)
        p.grad = g.to(torch.bfloat16)
        del g, mask
    torch.cuda.empty_cache()
    opts = [o for o in sharded.optimizers if o is not None] if sharded is not None else [A.AdamW_adv(owned, **kw)]
    opt = opts[0]

    def step():
        if sharded is not None:
            sharded.step()
        else:
            opt.step()

    clock_path = os.path.join(tempfile.gettempdir(), f"advopt_clocks_{rank}.csv")
    proc, fh = sample_clocks_start(clock_path)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    for o in opts:
        o._runner.kernel_events = []
    launches0 = sum(o._runner.launch_count for o in opts)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_clock0 = time.time()
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    t_clock1 = time.time()
    if world > 1:
        dist.barrier()
    clocks = sample_clocks_stop(proc, fh, clock_path, torch.cuda.get_device_properties(dev).index
                                if hasattr(torch.cuda.get_device_properties(dev), "index") else local,
                                t_clock0, t_clock1)
    elapsed_ms = e0.elapsed_time(e1)
    kev = [e for o in opts for e in o._runner.kernel_events]
    for o in opts:
        o._runner.kernel_events = None
    launches = sum(o._runner.launch_count for o in opts) - launches0
    kernel_ms = [a.elapsed_time(b) for a, b, _ in kev]
    kernel_avg_ms = float(np.sum(kernel_ms) / max(1, args.steps))
    if world > 1:
        t = torch.tensor([elapsed_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    ms_per_step = elapsed_ms / args.steps
    value = 1000.0 / ms_per_step   # whole-job optimizer steps/s (every rank takes part in each step)

    # sharded: the same step without the parameter all-gather (each rank's
    # kernels only), and the all-gather alone, beside the full step above
    split = None
    if world > 1:
        def timed(fn, n):
            torch.cuda.synchronize()
            dist.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(n):
                fn()
            b.record()
            torch.cuda.synchronize()
            t = torch.tensor([a.elapsed_time(b) / n], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())

        def step_only():
            for o in opts:
                o.step()

        only = timed(step_only, args.steps)
        gather = timed(sharded.gather, args.steps)
        moved = sum(fl.numel() * fl.element_size() for f in sharded.flats for fl, _ in f.buffers)
        recv = moved * (world - 1) / world
        # each rank's own Adam kernel time in the full step (partition balance)
        mine_k = torch.tensor([kernel_avg_ms], device=dev, dtype=torch.float64)
        all_k = [torch.zeros_like(mine_k) for _ in range(world)]
        dist.all_gather(all_k, mine_k)
        split = {"per_rank_kernel_ms": [float(x.item()) for x in all_k],
                 "step_only_ms": only, "step_only_value": 1000.0 / only, "step_plus_gather_ms": ms_per_step,
                 "gather_only_ms": gather, "gather_bytes_received_per_rank": recv,
                 "gather_gbs_per_rank": recv / (gather * 1e-3) / 1e9 if gather > 0 else 0.0,
                 "nvlink_peer_copy_gbs": 770.0}

    # ---- e2e: grads copied host->device every step, one result read back ----
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, owned, step, world, dev, opt if world == 1 else None, sharded)
    ns = prodigy = None
    modes = world == 1 and not args.no_modes
    if not (args.no_ns and args.no_prodigy and (world < 4 or args.no_70b) and not modes):
        # the other legs need the memory of the AdamW leg
        del opt, opts, owned, params, step, sharded
        torch.cuda.empty_cache()
    if not args.no_ns:
        ns = run_ns_leg(args, world, rank, dev)
    if not args.no_prodigy:
        prodigy = run_prodigy_leg(args, world, rank, dev)
    adamuon70 = None
    if world >= 4 and not args.no_70b:
        adamuon70 = run_adamuon70b_leg(args, world, rank, dev)
    mode_legs = {}
    if modes:
        mode_legs["factored_step"] = run_mode_leg(args, dev, "factored")
        mode_legs["spectral_step"] = run_mode_leg(args, dev, "spectral")
    if rank == 0:
        emit(args, shapes, mine, total, world, value, ms_per_step, kernel_avg_ms, launches, clocks, e2e, ns,
             prodigy, adamuon70, split, mode_legs)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def muon_shapes(layers=32):
    """Every 2-D hidden weight of Llama-3-8B (the Muon matrices)."""
    d, kv, ffn = 4096, 1024, 14336
    return [(d, d), (kv, d), (kv, d), (d, d), (ffn, d), (ffn, d), (d, ffn)] * layers


def run_ns_leg(args, world, rank, dev):
    """The Muon_adv step of the Llama-3-8B configuration: Muon (momentum 0.95,
    5 quintic Newton-Schulz iterations, bf16 'auto' states) on every hidden
    matrix, and Muon's auxiliary AdamW with fp32 states
    (adam_state_precision='fp32') on the two 128256x4096 embeddings and the 65
    RMSNorm weights, all in one optimizer step.  With N ranks the tensors are
    split by Newton-Schulz FLOPs / bytes (ShardedOptimizer) and the updated
    params all-gathered."""
    import torch.distributed as dist
    import advanced_optimizers_b200 as A
    from advanced_optimizers_b200.optim._muon_family import ns_flops
    shapes = muon_shapes(args.layers)
    flops = [ns_flops(min(s), max(s), 5, False) for s in shapes]
    d, V = 4096, 128256
    adam_shapes = ([(V, d), (V, d)] if not args.no_embed else []) + [(d,)] * (2 * args.layers + 1)
    gen = torch.Generator(device=dev).manual_seed(4321 + rank)
    params = [torch.nn.Parameter(torch.empty(sh, dtype=torch.bfloat16, device=dev)) for sh in shapes]
    aparams = [torch.nn.Parameter(torch.empty(sh, dtype=torch.bfloat16, device=dev)) for sh in adam_shapes]
    groups = [dict(params=params, optim_type="muon"), dict(params=aparams, optim_type="adam")]
    kw = dict(lr=1e-3, beta1=0.95, adam_state_precision="fp32")
    if world > 1:
        sharded = A.ShardedOptimizer(A.Muon_adv, groups, **kw)
        owner = sharded.owner
    else:
        sharded = None
        owner = [0] * (len(shapes) + len(adam_shapes))
    allp = params + aparams
    owned = [allp[i] for i in range(len(allp)) if owner[i] == rank]
    with torch.no_grad():
        for p in owned:
            p.normal_(0, 0.02, generator=gen)
    for p in owned:
        p.grad = torch.empty_like(p).normal_(0, 1e-3, generator=gen)
    if sharded is not None:
        opts = [o for o in sharded.optimizers if o is not None]
    else:
        opts = [A.Muon_adv([dict(params=params, optim_type="muon"), dict(params=aparams, optim_type="adam")], **kw)]
    opt = opts[0]

    def step():
        if sharded is not None:
            sharded.step()
        else:
            opt.step()

    warm = 2
    steps = 5
    for _ in range(warm):
        step()
    torch.cuda.synchronize()
    for o in opts:
        o.check_errors()
    if world > 1:
        dist.barrier()
    for o in opts:
        o._muon_runner.gemm_events = []
        o._adam_runner.kernel_events = []
    l0 = sum(o.launch_count for o in opts)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    gev = [e for o in opts for e in o._muon_runner.gemm_events]
    gemm_ms = sum(e[0].elapsed_time(e[1]) for e in gev) / steps
    fl = sum(e[2] for e in gev) / steps      # the reference's FLOP count of the chains
    fx = sum(e[3] for e in gev) / steps      # FLOPs the tensor cores execute (symmetric products halved)
    aux_ms = sum(a.elapsed_time(b) for o in opts for a, b, _ in o._adam_runner.kernel_events) / steps
    for o in opts:
        o._muon_runner.gemm_events = None
        o._adam_runner.kernel_events = None
    launches = sum(o.launch_count for o in opts) - l0
    per_rank = [[gemm_ms, aux_ms]]
    if world > 1:
        # each rank's own chain and auxiliary-Adam kernel time: the balance of
        # the partition (the step waits for the slowest rank)
        mine = torch.tensor([gemm_ms, aux_ms], device=dev, dtype=torch.float64)
        allr = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(allr, mine)
        per_rank = [x.tolist() for x in allr]
        t = torch.tensor([ms, gemm_ms, aux_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, gemm_ms, aux_ms = (float(x) for x in t.tolist())
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak, kind = float(json.load(f)["bf16_tflops_sustained"]), "measured sustained"
    except Exception:
        peak, kind = 1400.0, "fallback sustained"
    total_flops = sum(flops)
    n_aux = sum(math.prod(s) for s in adam_shapes)
    del opt, opts, owned, params, aparams, allp, sharded
    torch.cuda.empty_cache()
    return {"workload": f"Muon_adv step: Muon over {len(shapes)} Llama-3-8B hidden matrices (q/o 4096x4096, "
                        "k/v 1024x4096, gate/up 14336x4096, down 4096x14336), momentum 0.95, 5 quintic "
                        f"Newton-Schulz iterations, bf16 'auto' states; auxiliary AdamW (fp32 states) over "
                        f"{len(adam_shapes)} embedding / RMSNorm tensors ({n_aux} elements)",
            "steps": steps, "warmup": warm,
            "ms_per_step": ms, "value": 1000.0 / ms, "unit": "optimizer steps/s",
            "ns_ms_per_step": gemm_ms, "aux_adam_ms_per_step": aux_ms,
            "per_rank_ns_aux_ms": per_rank,
            "roofline": {"bound": "tensor", "achieved": (fx / (gemm_ms * 1e-3)) / 1e12 if gemm_ms > 0 else 0.0,
                         "peak": peak, "unit": "TFLOP/s",
                         "frac": ((fx / (gemm_ms * 1e-3)) / 1e12) / peak if gemm_ms > 0 else 0.0,
                         "peak_kind": kind, "kernel": "ns_gemm_kernel (tcgen05, 128x256 tiles)",
                         "algorithmic_flops_per_step": total_flops,
                         "executed_flops_per_step": fx,
                         "algorithmic_tflops": (fl / (gemm_ms * 1e-3)) / 1e12 if gemm_ms > 0 else 0.0,
                         "note": "achieved = FLOPs this rank's tensor cores execute (padded workspace; X X^T and "
                                 "b A + c A A on the blocks on or above the diagonal) / its chain time; "
                                 "algorithmic_tflops = the reference's FLOP count 5(4m^2n+2m^3) / the same time"},
            "gpu_launches": launches}


def gpt_1p3b_shapes(layers=24):
    """A 1.3B GPT-style shape list (d_model 2048, ffn 8192, vocab 50304,
    tied embeddings): embedding, per layer fused qkv 6144x2048, out 2048x2048,
    fc 8192x2048, proj 2048x8192 and two LayerNorm weights, then the final
    LayerNorm; 1.311e9 elements in 146 tensors."""
    d, ffn, V = 2048, 8192, 50304
    s = [(V, d)]
    for _ in range(layers):
        s += [(3 * d, d), (d, d), (ffn, d), (d, ffn), (d,), (d,)]
    return s + [(d,)]


def prodigy_bytes(shapes, slice_p=11):
    """Mandatory HBM bytes of one Prodigy_adv bf16_sr step: bf16 p read+write,
    bf16 g read, bf16 m and v read+write (14 B/element), plus every
    slice_p-th element's bf16 s read+write and bf16 p0 read."""
    tot = 0
    for sh in shapes:
        n = math.prod(sh)
        tot += 14 * n + 6 * ((n + slice_p - 1) // slice_p)
    return tot


def run_prodigy_leg(args, world, rank, dev):
    """Prodigy_adv(state_precision='bf16_sr', d0=1e-6) over the 1.3B GPT
    shapes; bf16 params ~N(0, 0.02^2), grads ~N(0, 1e-3^2) times a per-step
    scale drawn log-uniform in [1e-4, 1e-2].  Each step ends in the d
    estimate: with N ranks the owners' two sums are all-reduced (one 2-float
    NCCL all-reduce) and the updated params all-gathered."""
    import torch.distributed as dist
    import advanced_optimizers_b200 as A
    shapes = gpt_1p3b_shapes(args.prodigy_layers)
    gen = torch.Generator(device=dev).manual_seed(777 + rank)
    params = [torch.nn.Parameter(torch.empty(sh, dtype=torch.bfloat16, device=dev)) for sh in shapes]
    kw = dict(state_precision="bf16_sr", d0=1e-6)
    if world > 1:
        sharded = A.ShardedOptimizer(A.Prodigy_adv, params, **kw)
        owner = sharded.owner
    else:
        sharded = None
        owner = [0] * len(shapes)
    owned = [params[i] for i in range(len(shapes)) if owner[i] == rank]
    with torch.no_grad():
        for p in owned:
            p.normal_(0, 0.02, generator=gen)
    base = [torch.empty_like(p).normal_(0, 1e-3, generator=gen) for p in owned]
    opts = [o for o in sharded.optimizers if o is not None] if sharded is not None else [A.Prodigy_adv(owned, **kw)]
    rng = np.random.default_rng(99)
    scales = [float(10 ** rng.uniform(-4, -2)) for _ in range(64)]

    def step(k):
        with torch.no_grad():
            for p, b in zip(owned, base):
                p.grad = b * scales[k % len(scales)]
        if sharded is not None:
            sharded.step()
        else:
            opts[0].step()

    warm, steps = 3, 10
    for k in range(warm):
        step(k)
    torch.cuda.synchronize()
    for o in opts:
        o.check_errors()
    if world > 1:
        dist.barrier()
    # the grads of each step are set before its clock starts
    tot = 0.0
    kms = 0.0
    for k in range(steps):
        with torch.no_grad():
            for p, b in zip(owned, base):
                p.grad = b * scales[(warm + k) % len(scales)]
        for o in opts:
            o._runner.kernel_events = []
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        if sharded is not None:
            sharded.step()
        else:
            opts[0].step()
        e1.record()
        torch.cuda.synchronize()
        tot += e0.elapsed_time(e1)
        kms += sum(a.elapsed_time(b) for o in opts for a, b, _ in o._runner.kernel_events)
        for o in opts:
            o._runner.kernel_events = None
    ms, kernel_ms = tot / steps, kms / steps
    if world > 1:
        t = torch.tensor([ms, kernel_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, kernel_ms = (float(x) for x in t.tolist())
    d_val = float(opts[0].param_groups[0]["d"]) if opts else 0.0
    mine = [shapes[i] for i in range(len(shapes)) if owner[i] == rank]
    alg = prodigy_bytes(mine)
    peak, peak_kind = measured_peaks()
    achieved = alg / (kernel_ms * 1e-3) / 1e9 if kernel_ms > 0 else 0.0
    del opts, owned, params, base, sharded
    torch.cuda.empty_cache()
    return {"workload": "Prodigy_adv(state_precision='bf16_sr', d0=1e-6), 1.3B GPT shapes (d_model 2048, "
                        f"{args.prodigy_layers} layers, ffn 8192, vocab 50304, tied embedding), bf16, "
                        "grads x log-uniform[1e-4, 1e-2] per step",
            "params": sum(math.prod(s) for s in shapes), "tensors": len(shapes),
            "steps": steps, "warmup": warm, "ms_per_step": ms, "value": 1000.0 / ms, "unit": "optimizer steps/s",
            "d_after": d_val,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind, "kernel": "adam_fast_kernel<BF16_SR, bf16, Prodigy>",
                         "kernel_ms": kernel_ms, "algorithmic_bytes": alg}}


# algorithmic HBM bytes per element of the two optional-mode AdamW steps
# (bf16 params and grads):
#  factored: grad 2 + param 2 + 2 + sign bits 1/8 + 1/8 (factors and column
#            partials are per row / column, below 0.1%)
#  spectral ('auto' bf16 states): step kernel grad 2 + param 2 + m 2+2 +
#            v 2+2 + update written 2; U^T u and U v read the update twice
#            (2 + 2); the apply pass reads update 2 and param 2, writes param 2
MODE_BYTES_PER_ELEMENT = {"factored": 6.25, "spectral": 24.0}


def run_mode_leg(args, dev, mode):
    """AdamW_adv(state_precision='factored', nesterov=True) or
    AdamW_adv(state_precision='auto', spectral_normalization=True,
    nesterov=True) over the hidden weights and norms of args.mode_layers
    Llama-3-8B decoder layers (no embeddings), bf16; params ~N(0, 0.02^2),
    grads ~N(0, 1e-3^2).  Timed with CUDA events around whole steps (every
    launch of the step)."""
    import advanced_optimizers_b200 as A
    shapes = llama3_8b_shapes(args.mode_layers, embed=False)
    gen = torch.Generator(device=dev).manual_seed(4242)
    params = [torch.nn.Parameter(torch.empty(sh, dtype=torch.bfloat16, device=dev)) for sh in shapes]
    with torch.no_grad():
        for p in params:
            p.normal_(0, 0.02, generator=gen)
            p.grad = torch.empty_like(p).normal_(0, 1e-3, generator=gen)
    if mode == "factored":
        kw = dict(state_precision="factored", nesterov=True, weight_decay=0.01)
        kernel = "adam_kernel<FP32, bf16, AdamW, factored momentum> + factored finish"
    else:
        kw = dict(state_precision="auto", spectral_normalization=True, nesterov=True, weight_decay=0.01)
        kernel = "adam_kernel<AUTO, bf16, AdamW> emitting U + spec_vpart/vfinish/rows/ufinish/apply"
    opt = A.AdamW_adv(params, **kw)
    warm, steps = 3, 10
    for _ in range(warm):
        opt.step()
    torch.cuda.synchronize()
    opt.check_errors()
    l0 = opt._runner.launch_count
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        opt.step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    launches = (opt._runner.launch_count - l0) // steps
    numel = sum(math.prod(s) for s in shapes)
    alg = MODE_BYTES_PER_ELEMENT[mode] * numel
    peak, peak_kind = measured_peaks()
    achieved = alg / (ms * 1e-3) / 1e9
    del opt, params
    torch.cuda.empty_cache()
    return {"workload": f"AdamW_adv({', '.join(f'{k}={v!r}' for k, v in kw.items())}), Llama-3-8B hidden "
                        f"weights and norms of {args.mode_layers} layers, bf16 (inputs larger than L2)",
            "params": numel, "tensors": len(shapes), "steps": steps, "warmup": warm, "ms_per_step": ms,
            "value": 1000.0 / ms, "unit": "optimizer steps/s", "launches_per_step": launches,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "kernel": kernel, "algorithmic_bytes": alg,
                         "bytes_per_element": MODE_BYTES_PER_ELEMENT[mode]}}


def llama3_70b_matrices(layers=80):
    """Llama-3-70B 2-D weights: per layer q/o 8192x8192, k/v 1024x8192,
    gate/up 28672x8192, down 8192x28672, plus the 128256x8192 embedding; 561
    matrices, 6.95e10 elements."""
    d, kv, ffn, V = 8192, 1024, 28672, 128256
    s = [(V, d)]
    for _ in range(layers):
        s += [(d, d), (kv, d), (kv, d), (d, d), (ffn, d), (ffn, d), (d, ffn)]
    return s


def run_adamuon70b_leg(args, world, rank, dev):
    """AdaMuon_adv(accelerated_ns=True (CANS), state_precision='int8_sr') over
    the Llama-3-70B 2-D weights, states and Newton-Schulz work sharded per
    tensor.  The bf16 model (139 GB) does not fit replicated next to the
    states, so each rank holds only the tensors it owns
    (ShardedOptimizer(replicate_params=False)); after each bucket is stepped
    its updated params stream through one transient all-gather buffer.
    Runs with 4 or more ranks (about 105 GB per rank at 4, 55 GB at 8)."""
    import torch.distributed as dist
    import advanced_optimizers_b200 as A
    from advanced_optimizers_b200.optim._muon_family import ns_flops
    shapes = llama3_70b_matrices()
    meta = [torch.nn.Parameter(torch.empty(sh, dtype=torch.bfloat16, device="meta")) for sh in shapes]
    kw = dict(lr=1e-3, accelerated_ns=True, state_precision="int8_sr")
    sharded = A.ShardedOptimizer(A.AdaMuon_adv, [dict(params=meta, optim_type="muon")], replicate_params=False,
                                 **kw)
    gen = torch.Generator(device=dev).manual_seed(7000 + rank)
    owned = sharded.owned_params()
    with torch.no_grad():
        for p in owned:
            p.normal_(0, 0.02, generator=gen)
    for p in owned:
        p.grad = torch.empty_like(p).normal_(0, 1e-3, generator=gen)
    opts = [o for o in sharded.optimizers if o is not None]
    warm, steps = 1, 2
    for _ in range(warm):
        sharded.step()
    torch.cuda.synchronize()
    for o in opts:
        o.check_errors()
    dist.barrier()

    def timed(fn):
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / steps], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for o in opts:
        o._muon_runner.gemm_events = []
    ms = timed(sharded.step)
    gev = [e for o in opts for e in o._muon_runner.gemm_events]
    gemm_ms = sum(e[0].elapsed_time(e[1]) for e in gev) / steps
    fx = sum(e[3] for e in gev) / steps
    for o in opts:
        o._muon_runner.gemm_events = None

    def step_only():
        for o in opts:
            o.step()

    ms_step_only = timed(step_only)
    t = torch.tensor([gemm_ms, fx], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    gemm_ms_max = float(t[0])
    tf = torch.tensor([fx], device=dev, dtype=torch.float64)
    dist.all_reduce(tf, op=dist.ReduceOp.SUM)
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak, kind = float(json.load(f)["bf16_tflops_sustained"]), "measured sustained"
    except Exception:
        peak, kind = 1400.0, "fallback sustained"
    total_flops = sum(ns_flops(min(s), max(s), 5, True) for s in shapes)
    own_bytes = sum(p.numel() for p in owned) * 2
    del opts, owned, sharded, meta
    torch.cuda.empty_cache()
    return {"workload": "AdaMuon_adv(accelerated_ns=True, state_precision='int8_sr') over the 561 Llama-3-70B 2-D "
                        "weights (6.95e10 elements), bf16, states and Newton-Schulz work sharded per tensor, params "
                        "not replicated (streamed bucket all-gathers)",
            "n_gpus": world, "steps": steps, "warmup": warm,
            "ms_per_step": ms, "value": 1000.0 / ms, "unit": "optimizer steps/s",
            "step_only_ms": ms_step_only, "ns_ms_per_step_max_rank": gemm_ms_max,
            "owned_param_bytes_rank0": own_bytes,
            "roofline": {"bound": "tensor", "achieved": (tf.item() / world / (gemm_ms_max * 1e-3)) / 1e12
                         if gemm_ms_max > 0 else 0.0, "peak": peak, "unit": "TFLOP/s",
                         "frac": (tf.item() / world / (gemm_ms_max * 1e-3)) / 1e12 / peak if gemm_ms_max > 0 else 0.0,
                         "peak_kind": kind, "kernel": "ns_gemm_kernel (tcgen05, 128x256 tiles), CANS chain",
                         "algorithmic_flops_per_step": total_flops,
                         "note": "achieved = executed tensor-core FLOPs per rank (mean over ranks) / the slowest "
                                 "rank's chain time"}}


def run_e2e(args, owned, step, world, dev, opt=None, sharded=None):
    """Grads copied host->device from pinned memory every step, one result
    read back.  On one GPU the copies run on a side stream and each tensor is
    stepped through `step_parameter` (the per-parameter entry a fused back-pass
    trainer calls) as soon as its grad has landed, so the kernels overlap the
    copies of the later grads.  Sharded, the copies run bucket by bucket and
    each gather bucket is stepped (and its all-gather started) once its grads
    have landed."""
    import torch.distributed as dist
    stage_elems = max(p.numel() for p in owned)
    host = torch.empty(stage_elems, dtype=torch.bfloat16, pin_memory=True)
    host.normal_(0, 1e-3)
    readback = torch.empty(1024, dtype=torch.bfloat16, pin_memory=True)
    h2d = sum(p.grad.numel() * 2 for p in owned)
    e2e_steps = max(2, min(args.steps, 5))
    per_param = world == 1 and opt is not None
    copy_stream = torch.cuda.Stream(device=dev)
    group = opt.param_groups[0] if per_param else None

    buckets = sharded.owned_buckets() if sharded is not None else None

    def e2e_step():
        if buckets is not None:
            events = []
            with torch.cuda.stream(copy_stream):
                for ps in buckets:
                    for p in ps:
                        p.grad.view(-1).copy_(host[: p.numel()], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(copy_stream)
                    events.append(ev)
            sharded.step(bucket_events=events)
        elif per_param:
            events = []
            with torch.cuda.stream(copy_stream):
                for p in owned:
                    p.grad.view(-1).copy_(host[: p.numel()], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(copy_stream)
                    events.append(ev)
            cur = torch.cuda.current_stream()
            for p, ev in zip(owned, events):
                cur.wait_event(ev)
                opt.step_parameter(p, group)
        else:
            for p in owned:
                p.grad.view(-1).copy_(host[: p.numel()], non_blocking=True)
            step()
        readback.copy_(owned[0].detach().view(-1)[:1024], non_blocking=True)
        torch.cuda.current_stream().synchronize()

    e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    return {"value": 1.0 / e2e_s, "unit": "optimizer steps/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": readback.numel() * 2}


def emit(args, shapes, mine, total, world, value, ms_per_step, kernel_avg_ms, launches, clocks, e2e, ns=None,
         prodigy=None, adamuon70=None, split=None, mode_legs=None):
    if True:
        alg = algorithmic_bytes([shapes[i] for i in mine])
        peak, peak_kind = measured_peaks()
        achieved = alg / (kernel_avg_ms * 1e-3) / 1e9 if kernel_avg_ms > 0 else 0.0
        out = {
            "metric": "optimizer steps/s at Llama-3-8B shapes", "value": value, "unit": "optimizer steps/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": WORKLOAD if (args.layers == 32 and not args.no_embed) else
                       f"profiling subset: {args.layers} layers" + ("" if not args.no_embed else ", no embeddings"),
                       "params": total, "tensors": len(shapes),
                       "parallelism": f"per-tensor sharding x{world}" + (" + bucketed copy-engine pulls of the peers'"
                                                                 " bf16 params (NVLink)" if world > 1 else ""),
                       "l2": "inputs larger than L2 (about 40 GB resident per step)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": TRAFFIC_PER_ALG_BYTE * alg,
                         "traffic_note": "dram bytes per launch scaled from the 2-layer ncu capture",
                         "peak_kind": peak_kind,
                         "kernel": "adam_fast_kernel<INT8_SR, bf16, AdamW, Philox, flags compiled in>",
                         "kernel_ms": kernel_avg_ms,
                         "algorithmic_bytes": alg},
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clocks,
        }
        if ns is not None:
            out["muon_step"] = ns
        if prodigy is not None:
            out["prodigy_step"] = prodigy
        if adamuon70 is not None:
            out["adamuon_70b_step"] = adamuon70
        if split is not None:
            out["sharded"] = split
        for k, v in (mode_legs or {}).items():
            out[k] = v
        if world == 1 and not args.no_cpu_baseline:
            out["cpu_baseline"] = cpu_baseline()
        print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--layers", type=int, default=32, help="decoder layers (32 = the full model; fewer for profiling)")
    ap.add_argument("--no-embed", action="store_true", help="leave out embed/lm_head (profiling only)")
    ap.add_argument("--no-ns", action="store_true", help="skip the Muon_adv step leg")
    ap.add_argument("--no-prodigy", action="store_true", help="skip the Prodigy_adv step leg")
    ap.add_argument("--prodigy-layers", type=int, default=24,
                    help="layers of the 1.3B GPT shapes in the Prodigy_adv leg (24 = the full model; fewer for profiling)")
    ap.add_argument("--no-70b", action="store_true", help="skip the AdaMuon Llama-3-70B leg (4+ GPUs)")
    ap.add_argument("--no-modes", action="store_true",
                    help="skip the 'factored' state and spectral-normalisation AdamW legs (1 GPU)")
    ap.add_argument("--mode-layers", type=int, default=8, help="Llama-3-8B decoder layers of those legs")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
