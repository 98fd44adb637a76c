"""Per-tensor sharding of the optimizer step across the ranks of one node
(one process per GPU, torch.distributed over NCCL).

Every parameter tensor is owned by exactly one rank, chosen by
longest-processing-time assignment of a per-tensor cost (bytes for the
elementwise optimizers, Newton–Schulz FLOPs for Muon/AdaMuon matrices).  A
rank keeps optimizer state only for the tensors it owns and steps only
those; afterwards the updated parameters are all-gathered so that every rank
holds the full model again.  Prodigy's global d estimate needs the two sums
of every rank: they are all-reduced (one 2-float NCCL all-reduce per step),
with the previous step's numerator carried by rank 0 only, so the sharded
run reproduces the single-GPU d.

With `flat=True` (default) the parameters become views into rank-ordered
flat buffers — [rank 0's tensors | rank 1's | ...], every segment padded to
the largest — so each all-gather is one in-place `all_gather_into_tensor`
with no packing copies.  Each rank's owned tensors are split, in step order,
into the same number of gather buckets of about `bucket_bytes` (one flat
buffer per bucket and dtype): bucket k is stepped, its all-gather is issued
asynchronously on NCCL's stream, and bucket k+1 is stepped while it runs.
With `flat=False` each tensor is broadcast from its owner.

This module is plumbing around the single-GPU classes (it adds no kernel);
the reference's own distributed hook is Prodigy's `fsdp_in_use`
all-reduce (Prodigy_adv.py:550-554), which the Prodigy class keeps.
"""
from __future__ import annotations

import ctypes
import math
from typing import Callable, Iterable, Optional

import torch
import torch.distributed as dist

from . import _lib as L
from .optim._muon_family import is_suitable_for_muon, ns_time_estimate

ALIGN_ELEMS = 64   # every parameter view starts on a 128-byte boundary (bf16)


def lpt_partition(costs, world: int):
    """Owner rank of each item: items in decreasing cost (ties by index) go
    to the currently least-loaded rank (ties to the lower rank)."""
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    load = [0] * world
    owner = [0] * len(costs)
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        owner[i] = r
        load[r] += costs[i]
    return owner


# The elementwise kernels' HBM rate, which turns a tensor's bytes into
# seconds on the scale of the Newton-Schulz time estimate (ns_time_estimate:
# waves of GEMM tiles, so that small matrices that fill few SMs weigh what
# they take).
HBM_BYTES_PER_S = 3.0e12


def default_cost(optimizer_cls, group: dict, p: torch.Tensor) -> float:
    """Estimated seconds of the tensor's step: HBM bytes (param and grad, plus
    about as much again of state) at the elementwise kernels' rate, plus, for
    the Muon family's matrices, the Newton–Schulz chain's estimated time."""
    elem = p.numel() * p.element_size() * 4 / HBM_BYTES_PER_S
    name = getattr(optimizer_cls, "__name__", "")
    if name in ("Muon_adv", "AdaMuon_adv") and p.ndim >= 2:
        if group.get("use_muon") is not None:
            muon = bool(group["use_muon"])
        elif group.get("optim_type") is not None:
            muon = group["optim_type"] == "muon"
        else:
            muon = is_suitable_for_muon(p)
        if muon:
            rows = p.shape[0]
            cols = p.numel() // max(1, rows)
            return elem + ns_time_estimate(min(rows, cols), max(rows, cols), group.get("ns_steps", 5),
                                           group.get("accelerated_ns", False))
    return elem


class FlatParams:
    """Rank-ordered flat storage of the parameters (one buffer per dtype and
    device); `all_gather()` refreshes every parameter in place."""

    def __init__(self, params, owner, world: int, rank: int, group=None):
        self.world, self.rank, self.group = world, rank, group
        self.buffers = []   # (flat, seg)
        by_key = {}
        for p, r in zip(params, owner):
            by_key.setdefault((p.dtype, p.device), []).append((p, r))
        for (dt, dev), items in by_key.items():
            offsets = {}
            seg_used = [0] * world
            for p, r in items:
                off = seg_used[r]
                offsets[id(p)] = (r, off)
                seg_used[r] = off + math.ceil(p.numel() / ALIGN_ELEMS) * ALIGN_ELEMS
            seg = max(max(seg_used), ALIGN_ELEMS)
            flat = torch.zeros(world * seg, dtype=dt, device=dev)
            with torch.no_grad():
                for p, _ in items:
                    r, off = offsets[id(p)]
                    view = flat[r * seg + off: r * seg + off + p.numel()].view(p.shape)
                    view.copy_(p.data)
                    p.data = view
            self.buffers.append((flat, seg))

    @torch.no_grad()
    def all_gather(self, async_op: bool = False):
        """Refresh every parameter from its owner; with async_op the work
        handles are returned (NCCL: waiting on them orders the caller's
        stream after the gather)."""
        works = []
        for flat, seg in self.buffers:
            mine = flat[self.rank * seg:(self.rank + 1) * seg]
            if dist.get_backend(self.group) == "nccl":
                w = dist.all_gather_into_tensor(flat, mine, group=self.group, async_op=async_op)
            else:
                chunks = list(flat.split(seg))
                w = dist.all_gather(chunks, mine.clone(), group=self.group, async_op=async_op)
            if async_op:
                works.append(w)
        return works


class PeerPull:
    """The parameter gather on this GPU's copy engines: each rank maps the
    other ranks' flat buffers (CUDA IPC) and pulls their segments with one
    cudaMemcpyAsync per peer segment on a side stream, so the gather takes no
    SMs from the step's kernels (an NCCL all-gather runs as kernels beside
    them and slows them by about a quarter).

    Ordering, with one 1-element NCCL all-reduce as a fence: after a bucket's
    kernels, a fence on the side stream (every rank has written its segment)
    precedes the pulls of that bucket; the caller's stream waits for the side
    stream at the end of the step; a fence on the caller's stream at the
    start of the next step (every rank has finished reading) precedes the
    next writes to this rank's segments."""

    def __init__(self, flats, world: int, rank: int, group, device):
        self.world, self.rank, self.group = world, rank, group
        lib = L.lib()
        self.bases = []
        self.peer = {}       # (bucket, buffer, rank) -> address of that rank's flat buffer
        # every step below ends in an agreement among the ranks, so that a
        # failure on one rank (no IPC for its allocations) makes all of them
        # fall back together rather than diverge in their collectives
        try:
            local = []
            for fp in flats:
                row = []
                for flat, seg in fp.buffers:
                    h = ctypes.create_string_buffer(64)
                    off = ctypes.c_uint64(0)
                    L.check(lib.advopt_ipc_get_handle(flat.data_ptr(), h, ctypes.byref(off)), "advopt_ipc_get_handle")
                    row.append((h.raw, int(off.value)))
                local.append(row)
        except Exception:
            local = None
        everyone = [None] * world
        dist.all_gather_object(everyone, local, group=group)
        if any(e is None for e in everyone):
            raise RuntimeError("a rank cannot export its parameter buffers over CUDA IPC")
        ok = True
        try:
            for q in range(world):
                if q == rank:
                    continue
                for k, row in enumerate(everyone[q]):
                    for j, (h, off) in enumerate(row):
                        base = ctypes.c_void_p(0)
                        L.check(lib.advopt_ipc_open(h, ctypes.byref(base)), "advopt_ipc_open")
                        self.bases.append(base.value)
                        self.peer[(k, j, q)] = base.value + off
        except Exception:
            ok = False
        oks = [None] * world
        dist.all_gather_object(oks, ok, group=group)
        if not all(oks):
            self.close()
            raise RuntimeError("a rank cannot map the other ranks' parameter buffers")
        self.flats = flats
        self.side = torch.cuda.Stream(device)
        self.fence = torch.zeros(1, dtype=torch.float32, device=device)

    def begin_step(self):
        """Fence on the caller's stream: every rank has finished pulling the
        previous step's segments."""
        dist.all_reduce(self.fence, group=self.group)

    def pull_bucket(self, k: int):
        """After bucket k's kernels (on the caller's stream): fence, then pull
        the other ranks' segments of its buffers on the side stream."""
        lib = L.lib()
        self.side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.side):
            dist.all_reduce(self.fence, group=self.group)
            sh = self.side.cuda_stream
            for j, (flat, seg) in enumerate(self.flats[k].buffers):
                es = flat.element_size()
                nbytes = seg * es
                # rank r pulls from r+1, r+2, ... (mod N): at each phase every
                # source GPU feeds exactly one reader, so no peer's outgoing
                # NVLink bandwidth is shared by several pulls
                for dq in range(1, self.world):
                    q = (self.rank + dq) % self.world
                    L.check(lib.advopt_copy_async(flat.data_ptr() + q * nbytes, self.peer[(k, j, q)] + q * nbytes,
                                                  nbytes, sh), "advopt_copy_async")

    def end_step(self):
        torch.cuda.current_stream().wait_stream(self.side)

    def close(self):
        if not self.bases:
            return
        torch.cuda.synchronize()
        lib = L.lib()
        for b in self.bases:
            lib.advopt_ipc_close(b)
        self.bases = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class LocalSegments:
    """Storage of this rank's tensors only, for runs whose parameters do not
    fit replicated on every rank: per gather bucket and dtype one flat
    segment holding the rank's owned tensors (views, 128-byte aligned), padded
    to the largest rank's segment so that a bucket's all-gather is one
    `all_gather_into_tensor` into a transient rank-ordered buffer.  The buffer
    is reused by every bucket: the gathered parameters stream through it (to
    `consume(bucket, dtype, buffer, segment)` when given) rather than being
    kept."""

    def __init__(self, shapes, dtypes, owner, bucket, world: int, rank: int, device, group=None):
        self.world, self.rank, self.group = world, rank, group
        self.views = {}       # tensor index -> owned view
        self.segments = []    # per bucket: {dtype: (flat, seg)}
        n_buckets = max(bucket, default=0) + 1
        recv = {}
        for k in range(n_buckets):
            per = {}
            for dt in sorted({dtypes[i] for i in range(len(shapes)) if bucket[i] == k}, key=str):
                used = [0] * world
                offs = {}
                for i in range(len(shapes)):
                    if bucket[i] != k or dtypes[i] != dt:
                        continue
                    n = math.prod(shapes[i])
                    offs[i] = used[owner[i]]
                    used[owner[i]] += math.ceil(n / ALIGN_ELEMS) * ALIGN_ELEMS
                seg = max(max(used), ALIGN_ELEMS)
                flat = torch.zeros(seg, dtype=dt, device=device)
                for i, off in offs.items():
                    if owner[i] == rank:
                        self.views[i] = flat[off: off + math.prod(shapes[i])].view(shapes[i])
                per[dt] = (flat, seg)
                recv[dt] = max(recv.get(dt, 0), world * seg)
            self.segments.append(per)
        self.recv = {dt: torch.empty(n, dtype=dt, device=device) for dt, n in recv.items()}

    @torch.no_grad()
    def all_gather(self, k: int, consume=None, async_op: bool = False):
        works = []
        for dt, (flat, seg) in self.segments[k].items():
            buf = self.recv[dt][: self.world * seg]
            if dist.get_backend(self.group) == "nccl":
                w = dist.all_gather_into_tensor(buf, flat, group=self.group, async_op=async_op)
            else:
                w = dist.all_gather(list(buf.split(seg)), flat, group=self.group, async_op=async_op)
            if async_op:
                works.append(w)
            if consume is not None:
                if async_op:
                    w.wait()
                consume(k, dt, buf, seg)
        return works


def gather_buckets(sizes, owner, world: int, bucket_bytes: Optional[int]):
    """Split every rank's owned tensors (in parameter order) into the same
    number of consecutive buckets of about `bucket_bytes` each, by byte
    fraction, so that bucket k holds a similar byte count on every rank.
    Returns the bucket index of each tensor."""
    per_rank = [[i for i in range(len(sizes)) if owner[i] == r] for r in range(world)]
    totals = [sum(sizes[i] for i in idx) for idx in per_rank]
    if not bucket_bytes or bucket_bytes <= 0:
        return [0] * len(sizes)
    k = max(1, math.ceil(max(totals, default=0) / bucket_bytes))
    bucket = [0] * len(sizes)
    for r, idx in enumerate(per_rank):
        run = 0
        for i in idx:
            # bucket of the tensor's midpoint within the rank's byte range
            mid = run + sizes[i] / 2
            bucket[i] = min(k - 1, int(mid * k / totals[r])) if totals[r] > 0 else 0
            run += sizes[i]
    return bucket


class ShardedOptimizer:
    """Wraps one of the five optimizer classes for per-tensor sharding.

        opt = ShardedOptimizer(AdamW_adv, model.parameters(), lr=1e-3,
                               state_precision="int8_sr", factored_2nd=True)
        loss.backward(); opt.step(); opt.zero_grad()

    `params` may be an iterable of tensors or of param-group dicts (the
    group options are kept for the owned tensors).  `cost(group, p)` overrides
    the partition cost.  `bucket_bytes` sizes the gather buckets (None: one
    bucket, gathered after the whole step); with more than one bucket the
    elementwise kernels leave `reserve_sms` SMs free so that the all-gather of
    the previous bucket runs beside them.  `gather`: "copy" pulls the other
    ranks' segments of the replicated flat buffers with the copy engines over
    CUDA IPC mappings (PeerPull), "nccl" all-gathers them with NCCL, "auto"
    takes "copy" where every rank can map the others' buffers.  Every rank
    must call step() (it ends in collectives)."""

    def __init__(self, optimizer_cls, params, *, process_group=None,
                 cost: Optional[Callable[[dict, torch.Tensor], float]] = None, flat: bool = True,
                 bucket_bytes: Optional[int] = 1 << 30, reserve_sms: int = 0, replicate_params: bool = True,
                 device=None, gather_consumer=None, gather: str = "auto", **kwargs):
        if not (dist.is_available() and dist.is_initialized()):
            raise RuntimeError("ShardedOptimizer needs an initialised torch.distributed process group")
        self.group = process_group
        self.world = dist.get_world_size(process_group)
        self.rank = dist.get_rank(process_group)
        groups = list(params)
        if groups and not isinstance(groups[0], dict):
            groups = [{"params": groups}]
        self.all_params = []
        costs = []
        for g in groups:
            g["params"] = list(g["params"])
            for p in g["params"]:
                self.all_params.append(p)
                merged = dict(kwargs)
                merged.update({k: v for k, v in g.items() if k != "params"})
                costs.append(cost(g, p) if cost is not None else default_cost(optimizer_cls, merged, p))
        self.owner = lpt_partition(costs, self.world)
        self.is_prodigy = getattr(optimizer_cls, "__name__", "") == "Prodigy_adv"
        # Gather buckets: each is stepped, then its all-gather is issued
        # asynchronously while the next bucket is stepped.  Prodigy keeps one
        # bucket (its d estimate couples every tensor of the step).
        sizes = [p.numel() * p.element_size() for p in self.all_params]
        overlap = (flat or not replicate_params) and self.world > 1 and not self.is_prodigy
        self.bucket = gather_buckets(sizes, self.owner, self.world, bucket_bytes if overlap else None)
        n_buckets = max(self.bucket, default=0) + 1
        self.flats = []
        self.local = None
        self.gather_consumer = gather_consumer
        if not replicate_params:
            # only the owned tensors exist on this rank (the others may be meta
            # tensors: their shapes and dtypes place them); the owned ones are
            # new Parameters, views of this rank's bucket segments
            dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
            self.local = LocalSegments([tuple(p.shape) for p in self.all_params], [p.dtype for p in self.all_params],
                                       self.owner, self.bucket, self.world, self.rank, dev, process_group)
            for g in groups:
                g["params"] = [self._materialize(p) for p in g["params"]]
            self.all_params = [p for g in groups for p in g["params"]]
        elif flat:
            for k in range(n_buckets):
                idx = [i for i in range(len(self.all_params)) if self.bucket[i] == k]
                self.flats.append(FlatParams([self.all_params[i] for i in idx], [self.owner[i] for i in idx],
                                             self.world, self.rank, process_group))
        if self.is_prodigy:
            kwargs = dict(kwargs, fsdp_in_use=self.world > 1)
            # a rank without tensors follows the owners' d-estimate schedule:
            # Prodigy_adv.calculate_d all-reduces only while k < prodigy_steps
            # (or always when prodigy_steps <= 0), then increments k
            self._empty_k = 0
            self._empty_prodigy_steps = int(dict(kwargs, **{k: v for k, v in groups[0].items()
                                                            if k != "params"}).get("prodigy_steps", 0))
        # the user's groups (global param indices, options) for the state
        # dict in the reference's layout
        self._group_meta = []
        k0 = 0
        for g in groups:
            n = len(g["params"])
            self._group_meta.append({"indices": list(range(k0, k0 + n)),
                                     "opts": dict(kwargs, **{k: v for k, v in g.items() if k != "params"})})
            k0 += n
        self._inner_src = []   # per inner optimizer: the user group of each of its groups
        self.optimizers = []
        for k in range(n_buckets):
            own = {id(p) for i, p in enumerate(self.all_params) if self.owner[i] == self.rank and self.bucket[i] == k}
            owned_groups = []
            src = []
            for gi, g in enumerate(groups):
                ps = [p for p in g["params"] if id(p) in own]
                if ps:
                    owned_groups.append(dict(g, params=ps))
                    src.append(gi)
            self._inner_src.append(src)
            opt = optimizer_cls(owned_groups, **kwargs) if owned_groups else None
            if opt is not None and hasattr(opt, "_ids"):
                # Philox streams keyed by the tensor's global index: the sharded
                # step draws the same noise as a single-process step
                for i, p in enumerate(self.all_params):
                    if id(p) in own:
                        opt._ids[id(p)] = i
            if opt is not None and len(self.flats) > 1:
                # the elementwise kernels leave SMs free for the NCCL all-gather
                # of the previous bucket, which runs beside them
                for r in ("_runner", "_adam_runner"):
                    if hasattr(opt, r):
                        getattr(opt, r).reserve_sms = reserve_sms
            if self.is_prodigy and opt is not None:
                # the carried numerator is already global: count it on one rank
                opt._carry_scale = 1.0 if self.rank == 0 else 0.0
                opt._process_group = process_group
            self.optimizers.append(opt)
        self.peer = None
        if (self.world > 1 and self.flats and gather in ("auto", "copy")
                and dist.get_backend(process_group) == "nccl"):
            try:
                self.peer = PeerPull(self.flats, self.world, self.rank, process_group,
                                     self.flats[0].buffers[0][0].device)
            except RuntimeError:
                if gather == "copy":
                    raise
                self.peer = None

    def _materialize(self, p):
        i = next(k for k, q in enumerate(self.all_params) if q is p)
        if self.owner[i] != self.rank:
            return p
        return torch.nn.Parameter(self.local.views[i], requires_grad=p.requires_grad)

    def owned_params(self):
        """This rank's parameters (with replicate_params=False, the only ones
        that hold storage)."""
        return [p for i, p in enumerate(self.all_params) if self.owner[i] == self.rank]

    @property
    def optimizer(self):
        """The inner optimizer of this rank when there is one bucket (the
        first non-empty one otherwise)."""
        return next((o for o in self.optimizers if o is not None), None)

    @property
    def param_groups(self):
        return [g for o in self.optimizers if o is not None for g in o.param_groups]

    @property
    def state(self):
        out = {}
        for o in self.optimizers:
            if o is not None:
                out.update(o.state)
        return out

    def owned(self, p) -> bool:
        return self.owner[self._index(p)] == self.rank

    def _index(self, p):
        for i, q in enumerate(self.all_params):
            if q is p:
                return i
        raise KeyError("not a parameter of this optimizer")

    @torch.no_grad()
    def gather(self):
        """Bring every rank's updated tensors to all ranks (with
        replicate_params=False: stream them through the transient buffer)."""
        if self.world == 1:
            return
        if self.local is not None:
            for k in range(len(self.optimizers)):
                for w in self.local.all_gather(k, self.gather_consumer, async_op=self.gather_consumer is None):
                    w.wait()
            return
        if self.peer is not None:
            self.peer.begin_step()
            for k in range(len(self.flats)):
                self.peer.pull_bucket(k)
            self.peer.end_step()
        elif self.flats:
            for f in self.flats:
                f.all_gather()
        else:
            for p, r in zip(self.all_params, self.owner):
                dist.broadcast(p.data, src=r, group=self.group)

    @torch.no_grad()
    def owned_buckets(self):
        """This rank's parameters per gather bucket, in step order."""
        return [[p for i, p in enumerate(self.all_params) if self.owner[i] == self.rank and self.bucket[i] == k]
                for k in range(len(self.optimizers))]

    @torch.no_grad()
    def step(self, closure=None, bucket_events=None):
        """One sharded step.  `bucket_events` (optional, one CUDA event per
        bucket): the current stream waits on event k before stepping bucket k,
        e.g. for grads of that bucket still being copied on another stream."""
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        works = []
        if self.peer is not None:
            self.peer.begin_step()
        for k, opt in enumerate(self.optimizers):
            if bucket_events is not None:
                torch.cuda.current_stream().wait_event(bucket_events[k])
            if opt is not None:
                opt.step()
            elif self.is_prodigy and self.world > 1:
                # a rank without tensors still takes part in the d all-reduce,
                # on the same steps as the owners
                ps = self._empty_prodigy_steps
                if not (ps > 0 and self._empty_k >= ps):
                    dist.all_reduce(torch.zeros(2, dtype=torch.float32, device=self.all_params[0].device),
                                    op=dist.ReduceOp.SUM, group=self.group)
                self._empty_k += 1
            if self.peer is not None:
                self.peer.pull_bucket(k)
            elif self.world > 1 and self.flats:
                works += self.flats[k].all_gather(async_op=True)
            elif self.world > 1 and self.local is not None:
                # stream the bucket's gathered parameters through the transient
                # buffer; the gathers run in order on the collective stream, so
                # the next bucket's may reuse it (a consumer reads each one
                # before the next is issued)
                works += self.local.all_gather(k, self.gather_consumer, async_op=self.gather_consumer is None)
        for w in works:
            w.wait()
        if self.peer is not None:
            self.peer.end_step()
        if self.world > 1 and not self.flats and self.local is None:
            self.gather()
        return loss

    def zero_grad(self, set_to_none: bool = True):
        for p in self.all_params:
            if set_to_none:
                p.grad = None
            elif p.grad is not None:
                p.grad.zero_()

    def full_state_dict(self, dst: int = 0):
        """The state dict one `optimizer_cls` over all the params would
        return (torch.optim's layout, which the reference's checkpoints use,
        state_util.py:181-263): global param indices, the user's groups, every
        owner's states gathered to rank `dst` as CPU tensors.  A collective:
        every rank calls it; ranks other than `dst` get None.  Loadable at any
        world size (`load_full_state_dict`) and by a single-process optimizer."""
        local_state, group_opts = {}, {}
        for opt, src in zip(self.optimizers, self._inner_src):
            if opt is None:
                continue
            sd = opt.state_dict()
            local_params = [p for g in opt.param_groups for p in g["params"]]
            for li, st in sd["state"].items():
                local_state[self._index(local_params[li])] = {
                    k: (v.detach().cpu() if torch.is_tensor(v) else v) for k, v in st.items()}
            for g, s in zip(sd["param_groups"], src):
                group_opts.setdefault(s, {k: v for k, v in g.items() if k != "params"})
        parts = [None] * self.world if self.rank == dst else None
        dist.gather_object((local_state, group_opts), parts, dst=dst, group=self._object_group())
        if self.rank != dst:
            return None
        state, opts = {}, {}
        for ls, go in parts:
            state.update(ls)
            for s, o in go.items():
                opts.setdefault(s, o)
        param_groups = []
        for s, meta in enumerate(self._group_meta):
            pg = dict(opts.get(s, meta["opts"]))
            pg["params"] = list(meta["indices"])
            param_groups.append(pg)
        return {"state": {i: state[i] for i in sorted(state)}, "param_groups": param_groups}

    def _object_group(self):
        """The group for Python-object collectives: a gloo group over the
        default group's ranks when the collectives run on NCCL (the states
        are CPU tensors by then; no device copies), else the group itself."""
        if self.group is not None or dist.get_backend(self.group) == "gloo":
            return self.group
        if getattr(self, "_cpu_group", None) is None:
            self._cpu_group = dist.new_group(backend="gloo")
        return self._cpu_group

    def load_full_state_dict(self, sd):
        """Load a state dict in torch.optim's layout (from `full_state_dict`,
        a single-process optimizer, or the reference's own `state_dict()`):
        each rank takes its owned params' entries and its groups' options."""
        for opt, src in zip(self.optimizers, self._inner_src):
            if opt is None:
                continue
            local_params = [p for g in opt.param_groups for p in g["params"]]
            state = {}
            for li, p in enumerate(local_params):
                gi = self._index(p)
                if gi in sd["state"]:
                    state[li] = sd["state"][gi]
            groups, li = [], 0
            for g, s in zip(opt.param_groups, src):
                pg = {k: v for k, v in sd["param_groups"][s].items() if k != "params"}
                pg["params"] = list(range(li, li + len(g["params"])))
                li += len(g["params"])
                groups.append(pg)
            opt.load_state_dict({"state": state, "param_groups": groups})

    def state_dict(self):
        if len(self.optimizers) == 1:
            return self.optimizers[0].state_dict() if self.optimizers[0] is not None else {}
        return {"buckets": [o.state_dict() if o is not None else {} for o in self.optimizers]}

    def load_state_dict(self, sd):
        if len(self.optimizers) == 1:
            if self.optimizers[0] is not None:
                self.optimizers[0].load_state_dict(sd)
            return
        for o, s in zip(self.optimizers, sd["buckets"]):
            if o is not None:
                o.load_state_dict(s)
