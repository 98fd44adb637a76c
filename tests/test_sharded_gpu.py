"""Per-tensor sharding on 2 GPUs (NCCL): the sharded step reproduces the
single-process step.  AdamW_adv (int8_sr + factored_2nd) and Muon_adv are
bit-identical (Philox streams are keyed by the tensor's global index);
Prodigy_adv's d is within 1e-5 relative (its two sums are all-reduced in a
different order) and its params within 1 bf16 ulp.  The gather runs on the
copy engines (CUDA IPC pulls) by default; one case uses the NCCL all-gather.
Skipped with fewer than two GPUs."""
import io
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPES = [(512, 384), (384,), (256, 1024), (1024, 256), (640,), (96, 64)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _params(dev):
    g = torch.Generator().manual_seed(5)
    ps = [torch.nn.Parameter((torch.randn(s, generator=g) * 0.02).to(torch.bfloat16).to(dev)) for s in SHAPES]
    grads = [[(torch.randn(s, generator=g) * 1e-3).to(torch.bfloat16).to(dev) for s in SHAPES] for _ in range(3)]
    return ps, grads


def _make(name, params, sharded):
    import advanced_optimizers_b200 as A
    buckets = name.endswith("_buckets")
    nccl = "_nccl" in name
    name = name.replace("_buckets", "").replace("_nccl", "")
    if name == "adamw":
        cls, args, kw = A.AdamW_adv, params, dict(state_precision="int8_sr", factored_2nd=True, nesterov=True)
    elif name == "prodigy":
        cls, args, kw = A.Prodigy_adv, params, dict(state_precision="bf16_sr", d0=1e-6)
    else:
        mats = [p for p in params if p.ndim == 2]
        vecs = [p for p in params if p.ndim == 1]
        cls, args, kw = A.Muon_adv, [dict(params=mats, optim_type="muon"), dict(params=vecs, optim_type="adam")], {}
    if sharded:
        # small gather buckets: several asynchronous all-gathers per step
        extra = dict(bucket_bytes=256 << 10) if buckets else {}
        if nccl:
            # the NCCL all-gather instead of the copy-engine pulls
            extra["gather"] = "nccl"
        return A.ShardedOptimizer(cls, args, **kw, **extra)
    return cls(args, **kw)


def _run(name, params, grads, opt):
    for step in range(3):
        for p, g in zip(params, grads[step]):
            p.grad = g.clone()
        if name.endswith("_buckets"):
            # each bucket waits on an event, as a trainer copying grads on a side stream would pass
            n = len(opt.optimizers)
            assert n > 1, "expected several gather buckets"
            events = []
            for _ in range(n):
                ev = torch.cuda.Event()
                ev.record()
                events.append(ev)
            opt.step(bucket_events=events)
        else:
            opt.step()
    torch.cuda.synchronize()


def _worker(rank, world, port, name, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        ps, grads = _params(dev)
        opt = _make(name, ps, True)
        _run(name, ps, grads, opt)
        out[rank] = [p.detach().cpu() for p in ps]
        if name == "prodigy" and opt.optimizer is not None:
            out[f"d{rank}"] = opt.optimizer.param_groups[0]["d"]
        if name == "adamw_buckets":
            # the owners' states gathered into the single-process layout
            # (handed to the parent as bytes: no tensor sharing across the
            # process boundary)
            sd = opt.full_state_dict()
            if rank == 0:
                buf = io.BytesIO()
                torch.save(sd, buf)
                out["sd"] = buf.getvalue()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("name", ["adamw", "muon", "prodigy", "adamw_buckets", "muon_buckets", "adamw_nccl_buckets"])
def test_sharded_matches_single_process(name):
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), name, out), nprocs=world, join=True)
    ps, grads = _params(torch.device("cuda", 0))
    opt = _make(name, ps, False)
    _run(name.replace("_buckets", "").replace("_nccl", ""), ps, grads, opt)
    ref = [p.detach().cpu() for p in ps]
    for r in range(world):
        for i, (a, b) in enumerate(zip(out[r], ref)):
            if name == "prodigy":
                da = (a.view(torch.int16).int() - b.view(torch.int16).int()).abs()
                assert int(da.max()) <= 1, f"rank {r} tensor {i}: {int(da.max())} bf16 ulps"
            else:
                assert torch.equal(a, b), f"rank {r} tensor {i} differs"
    if name == "adamw_buckets":
        sd, want = torch.load(io.BytesIO(out["sd"]), weights_only=False), opt.state_dict()
        assert sorted(sd["state"]) == sorted(want["state"])
        assert [g["params"] for g in sd["param_groups"]] == [g["params"] for g in want["param_groups"]]
        for i, st in want["state"].items():
            for key, val in st.items():
                got = sd["state"][i][key]
                if not torch.is_tensor(val):
                    assert got == val, (i, key)
                elif key in ("mu_v_nmf", "mv_v_nmf"):
                    # float32 column sums over another piece cut
                    torch.testing.assert_close(got, val.cpu(), rtol=2e-6, atol=0)
                else:
                    assert torch.equal(got, val.cpu()), (i, key)
        # and a single-process optimizer resumes from it
        opt2 = _make("adamw", [torch.nn.Parameter(p.detach().clone()) for p in ps], False)
        opt2.load_state_dict(sd)
        assert torch.equal(opt2.state[opt2.param_groups[0]["params"][0]]["exp_avg"].cpu(),
                           want["state"][0]["exp_avg"].cpu())
    if name == "prodigy":
        d_ref = opt.param_groups[0]["d"]
        for r in range(world):
            if f"d{r}" in out:
                assert abs(out[f"d{r}"] - d_ref) <= 1e-5 * abs(d_ref)
