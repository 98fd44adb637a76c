"""Per-tensor sharding host logic on CPU: two gloo ranks (world_size 2).

The optimizer here is a stand-in (plain SGD on CPU tensors) because the B200
classes run only on CUDA; what is tested is the partition, the rank-ordered
flat parameter storage and the all-gather: after a sharded step every rank
holds exactly the parameters a single process would have."""
import copy
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from advanced_optimizers_b200.distributed import ShardedOptimizer, lpt_partition


class PlainSGD(torch.optim.Optimizer):
    def __init__(self, params, lr=0.1):
        super().__init__(params, dict(lr=lr))

    @torch.no_grad()
    def step(self, closure=None):
        for g in self.param_groups:
            for p in g["params"]:
                if p.grad is not None:
                    p.add_(p.grad, alpha=-g["lr"])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


SHAPES = [(64, 48), (10,), (33, 7), (128,), (5, 5, 3), (1,), (300,)]


def _make(seed=0):
    g = torch.Generator().manual_seed(seed)
    ps = [torch.nn.Parameter(torch.randn(s, generator=g)) for s in SHAPES]
    grads = [torch.randn(s, generator=g) for s in SHAPES]
    return ps, grads


def _worker(rank, world, port, flat, out, bucket_bytes=1 << 30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ps, grads = _make()
        opt = ShardedOptimizer(PlainSGD, ps, lr=0.5, flat=flat, bucket_bytes=bucket_bytes)
        out[f"buckets{rank}"] = len(opt.optimizers)
        for step in range(3):
            for p, g in zip(ps, grads):
                p.grad = g * (step + 1)
            opt.step()
            opt.zero_grad()
        out[rank] = [p.detach().clone() for p in ps]
        out[f"owner{rank}"] = list(opt.owner)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("flat,bucket_bytes", [(True, 1 << 30), (False, 1 << 30), (True, 512)])
def test_sharded_step_matches_single_process(flat, bucket_bytes):
    world = 2
    port = _free_port()
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, port, flat, out, bucket_bytes), nprocs=world, join=True)
    if bucket_bytes == 512:
        # small buckets: several gather buckets, each all-gathered asynchronously
        assert out["buckets0"] == out["buckets1"] > 1
    ref, grads = _make()
    opt = PlainSGD(ref, lr=0.5)
    for step in range(3):
        for p, g in zip(ref, grads):
            p.grad = g * (step + 1)
        opt.step()
    for r in range(world):
        for a, b in zip(out[r], ref):
            assert torch.equal(a, b.detach())
    assert out["owner0"] == out["owner1"]
    assert set(out["owner0"]) == {0, 1}


def test_lpt_partition_is_balanced_and_deterministic():
    costs = [100, 90, 80, 10, 10, 10, 5, 1]
    own = lpt_partition(costs, 3)
    assert own == lpt_partition(costs, 3)
    loads = [sum(c for c, r in zip(costs, own) if r == k) for k in range(3)]
    assert max(loads) - min(loads) <= max(costs)
    assert lpt_partition([5], 4) == [0]


def test_gather_buckets_keep_order_and_balance():
    """Every rank's tensors go to buckets in step order, all ranks use the
    same bucket count, and bucket k holds a similar share of every rank's bytes."""
    from advanced_optimizers_b200.distributed import gather_buckets
    import random
    rng = random.Random(3)
    sizes = [rng.choice([8 << 20, 33 << 20, 117 << 20, 8192]) for _ in range(300)]
    world = 4
    owner = lpt_partition(sizes, world)
    bucket = gather_buckets(sizes, owner, world, 1 << 30)
    k = max(bucket) + 1
    assert k > 1
    totals = [sum(s for s, o in zip(sizes, owner) if o == r) for r in range(world)]
    for r in range(world):
        mine = [b for b, o in zip(bucket, owner) if o == r]
        assert mine == sorted(mine)                      # step order
        for b in range(k):
            share = sum(s for s, o, bb in zip(sizes, owner, bucket) if o == r and bb == b) / totals[r]
            assert abs(share - 1 / k) < 0.5 / k + max(sizes) / totals[r]
    assert gather_buckets(sizes, owner, world, None) == [0] * len(sizes)


class _ProdigyScheduleStandIn(torch.optim.Optimizer):
    """CPU stand-in with Prodigy_adv's collective schedule only: calculate_d
    all-reduces the two d sums while k < prodigy_steps (always when
    prodigy_steps <= 0), then k += 1 (Prodigy_adv.py:540-576)."""

    def __init__(self, params, lr=0.1, prodigy_steps=0, fsdp_in_use=False):
        super().__init__(params, dict(lr=lr, prodigy_steps=prodigy_steps, k=0))
        self.fsdp_in_use = fsdp_in_use
        self._carry_scale = 1.0
        self._process_group = None
        self.reduces = 0

    @torch.no_grad()
    def step(self, closure=None):
        g0 = self.param_groups[0]
        if not (g0["prodigy_steps"] > 0 and g0["k"] >= g0["prodigy_steps"]):
            dist.all_reduce(torch.zeros(2), op=dist.ReduceOp.SUM, group=self._process_group)
            self.reduces += 1
        for g in self.param_groups:
            g["k"] += 1


_ProdigyScheduleStandIn.__name__ = "Prodigy_adv"


def _prodigy_worker(rank, world, port, prodigy_steps, out):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        ps = [torch.nn.Parameter(torch.ones(4)), torch.nn.Parameter(torch.ones(3))]
        opt = ShardedOptimizer(_ProdigyScheduleStandIn, ps, prodigy_steps=prodigy_steps)
        for _ in range(5):
            for p in ps:
                p.grad = torch.ones_like(p)
            opt.step()
        out[rank] = "empty" if opt.optimizer is None else opt.optimizer.reduces
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("prodigy_steps", [0, 1, 3])
def test_prodigy_rank_without_tensors_follows_the_d_schedule(prodigy_steps):
    """More ranks than tensors: the empty rank must join exactly the d
    all-reduces the owners make, also after prodigy_steps freezes d (a
    mismatch would leave the owners' next collective waiting on it)."""
    world = 3
    port = _free_port()
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_prodigy_worker, args=(world, port, prodigy_steps, out), nprocs=world, join=True)
    owners = [v for v in out.values() if v != "empty"]
    assert list(out.values()).count("empty") == 1
    expect = 5 if prodigy_steps <= 0 else min(5, prodigy_steps)
    assert owners == [expect] * 2


def _stream_worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ps, grads = _make()
        # every rank describes the whole model by shape only
        meta = [torch.nn.Parameter(torch.empty(p.shape, device="meta")) for p in ps]
        got = {}

        def consume(k, dt, buf, seg):
            got[k] = buf.clone()

        opt = ShardedOptimizer(PlainSGD, meta, lr=0.5, replicate_params=False, device="cpu", bucket_bytes=512,
                               gather_consumer=consume)
        own = opt.owned_params()
        idx = [i for i in range(len(ps)) if opt.owner[i] == rank]
        assert all(not p.is_meta for p in own)
        assert all(opt.all_params[i].is_meta for i in range(len(ps)) if opt.owner[i] != rank)
        with torch.no_grad():
            for i, p in zip(idx, own):
                p.copy_(ps[i])
        for i, p in zip(idx, own):
            p.grad = grads[i].clone()
        opt.step()
        # unpack every gathered bucket into per-tensor values (rank-ordered segments)
        vals = {}
        for k in got:
            seg = opt.local.segments[k][torch.float32][1]
            for r in range(world):
                off = 0
                for i in range(len(ps)):
                    if opt.bucket[i] == k and opt.owner[i] == r:
                        n = ps[i].numel()
                        vals[i] = got[k][r * seg + off: r * seg + off + n].view(ps[i].shape).clone()
                        off += -(-n // 64) * 64
        out[rank] = vals
        out[f"n_buckets{rank}"] = len(opt.optimizers)
    finally:
        dist.destroy_process_group()


def test_streamed_gather_without_replicated_params():
    """replicate_params=False: each rank materialises only its own tensors
    (the rest stay meta), steps them, and every bucket's all-gather streams
    the whole updated model through one transient buffer, bucket by bucket;
    the gathered values equal a single-process step."""
    world = 2
    port = _free_port()
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_stream_worker, args=(world, port, out), nprocs=world, join=True)
    assert out["n_buckets0"] == out["n_buckets1"] > 1
    ref, grads = _make()
    opt = PlainSGD(ref, lr=0.5)
    for p, g in zip(ref, grads):
        p.grad = g
    opt.step()
    for r in range(world):
        vals = out[r]
        assert sorted(vals) == list(range(len(ref)))
        for i, p in enumerate(ref):
            assert torch.equal(vals[i], p.detach()), (r, i)


class MomentumSGD(torch.optim.Optimizer):
    """Stand-in with per-param state (a buffer and a step count)."""

    def __init__(self, params, lr=0.1, momentum=0.9):
        super().__init__(params, dict(lr=lr, momentum=momentum))

    @torch.no_grad()
    def step(self, closure=None):
        for g in self.param_groups:
            for p in g["params"]:
                if p.grad is None:
                    continue
                st = self.state[p]
                if "buf" not in st:
                    st["buf"] = torch.zeros_like(p)
                    st["step"] = 0
                st["buf"].mul_(g["momentum"]).add_(p.grad)
                st["step"] += 1
                p.add_(st["buf"], alpha=-g["lr"])


def _groups(ps):
    return [dict(params=ps[:3], lr=0.3), dict(params=ps[3:])]


def _full_sd_worker(rank, world, port, single_sd, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ps, grads = _make()
        opt = ShardedOptimizer(MomentumSGD, _groups(ps), lr=0.5, bucket_bytes=512)
        for step in range(2):
            for p, g in zip(ps, grads):
                p.grad = g * (step + 1)
            opt.step()
        sd = opt.full_state_dict()
        if rank == 0:
            out["sd"] = sd
        else:
            out["other"] = sd
        # a second sharded optimizer, bucketed differently, resumes from the
        # single-process optimizer's state dict and takes the third step
        ps2, _ = _make()
        with torch.no_grad():
            for a, b in zip(ps2, single_sd["params"]):
                a.copy_(b)
        opt2 = ShardedOptimizer(MomentumSGD, _groups(ps2), lr=0.5, bucket_bytes=None)
        # (torch.optim's load_state_dict keeps same-device tensors as given:
        # load a copy, the parent's dict lives in shared memory)
        opt2.load_full_state_dict(copy.deepcopy(single_sd["sd"]))
        for p, g in zip(ps2, grads):
            p.grad = g * 3
        opt2.step()
        out[rank] = [p.detach().clone() for p in ps2]
    finally:
        dist.destroy_process_group()


def test_full_state_dict_in_the_single_process_layout():
    """full_state_dict() gathers every owner's states under global indices
    with the user's groups: equal to one unsharded optimizer's state_dict();
    load_full_state_dict() takes such a dict at another bucketing and the
    next step matches the unsharded optimizer's."""
    ref, grads = _make()
    opt = MomentumSGD(_groups(ref), lr=0.5)
    for step in range(2):
        for p, g in zip(ref, grads):
            p.grad = g * (step + 1)
        opt.step()
    single = {"sd": opt.state_dict(), "params": [p.detach().clone() for p in ref]}
    world = 2
    port = _free_port()
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_full_sd_worker, args=(world, port, single, out), nprocs=world, join=True)
    sd, want = out["sd"], single["sd"]
    assert out["other"] is None
    assert sorted(sd["state"]) == sorted(want["state"])
    for i, st in want["state"].items():
        assert sd["state"][i]["step"] == st["step"]
        assert torch.equal(sd["state"][i]["buf"], st["buf"]), i
    assert [g["params"] for g in sd["param_groups"]] == [g["params"] for g in want["param_groups"]]
    assert [g["lr"] for g in sd["param_groups"]] == [0.3, 0.5]
    for p, g in zip(ref, grads):
        p.grad = g * 3
    opt.step()
    for r in range(world):
        for a, b in zip(out[r], ref):
            assert torch.equal(a, b.detach()), r
