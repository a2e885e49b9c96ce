"""Sharded optimizer step over the GPUs of one node (NCCL over NVLink/NVSwitch).

The reference is single-GPU (no torch.distributed call sites); this is the
north-star's partitioned step. Placement never changes per-matrix arithmetic,
so every rank's result is bit-identical to the single-GPU engine.

  * NorMuon: whole matrices are assigned to ranks in contiguous runs of a
    shape-sorted list, cut to balance a model of each rank's launch rounds
    (assign_matrices); each rank batches its own matrices by shape. The NorMuon parameters are re-pointed into one flat bf16 arena laid
    out rank by rank, so the exchange is a single in-place all-gather.
  * AdamW: tables whose row count divides by the world size are split by rows
    (each rank updates its rows; in-place all-gather per table); the small
    scalar/gain tensors are updated redundantly by every rank (no exchange).
  * EMA: each rank folds the EMA of what it updates; shadows of other ranks'
    parameters are gathered on demand by gather_ema().

Exchange inside step(): every rank pushes the rows it updated into the same
offsets of every peer's copies with copy-engine transfers (CUDA IPC mappings),
visiting the peers in ring order so that each rank sends to one peer at a time
(all peers at once left the copy engines at ~300 GB/s on 8 GPUs). The tables
are pushed right after AdamW, so they cross NVLink while NorMuon computes: copy
engines leave every SM to the GEMMs, where an all-gather kernel would take
some and push the GEMMs' one-wave grids into a second wave. The NorMuon arena,
ready only at the end, goes by copy-engine push on two ranks ("ce", then a
one-element NCCL all-reduce as the completion barrier) and by NCCL all-gather
from four ranks on ("hybrid"; the all-gather is then also the pushes'
barrier). Where IPC export is not possible (memory from cuMemCreate, CPU
tensors) step() uses NCCL all-gathers only.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib


def gram_cost(shape) -> float:
    """Orthogonaliser FLOPs of one matrix as the engine runs it: two Gram
    products X X^T and two Q X products (6 m^2 n, symmetric outputs at half)
    and fourteen symmetric m x m products (14 m^3)."""
    r, c = shape[-2], shape[-1]
    m, n = min(r, c), max(r, c)
    return 6.0 * m * m * n + 14.0 * m ** 3


# Cost model of one rank's NorMuon share, in microseconds on one B200: GEMM
# launches run in rounds of 256 x 256 tiles over 74 CTA pairs (a launch with
# 75 tiles costs two rounds), a round costs K x 5.9 ns (a pair tile at the
# measured 1642 TFLOP/s), every launch a few microseconds of fill and drain;
# the front and apply passes stream 26 bytes per element at copy bandwidth.
_PAIRS = 74
_ROUND_NS_PER_K = 7.7
_LAUNCH_US = 4.0
_STREAM_B_PER_ELEM = 26.0
_HBM_B_PER_US = 6.5e6


def _tiles(a: int) -> int:
    return -(-a // 256)


def rank_cost_us(shapes) -> float:
    """Modelled time of the NorMuon step of one rank owning these matrices."""
    groups, classes = {}, {}
    for sh in shapes:
        groups[tuple(sh)] = groups.get(tuple(sh), 0) + 1
    us = 0.0
    for (r, c), s in groups.items():
        m, n = min(r, c), max(r, c)
        us += s * r * c * _STREAM_B_PER_ELEM / _HBM_B_PER_US
        if m <= 32:
            us += _LAUNCH_US
            continue
        classes[m] = classes.get(m, 0) + s
        sym = _tiles(m) * (_tiles(m) + 1) // 2
        syrk = -(-s * sym // _PAIRS) * n * _ROUND_NS_PER_K / 1e3
        qx = -(-s * _tiles(r) * _tiles(c) // _PAIRS) * m * _ROUND_NS_PER_K / 1e3
        us += 2 * (syrk + qx) + 4 * _LAUNCH_US
    for m, s in classes.items():
        sym = _tiles(m) * (_tiles(m) + 1) // 2
        us += 14 * (-(-s * sym // _PAIRS) * m * _ROUND_NS_PER_K / 1e3 + _LAUNCH_US)
    return us


def _shape_order_key(shape):
    r, c = shape[-2], shape[-1]
    return (min(r, c) <= 32, -max(r, c), -min(r, c), 0 if r > c else 1, (r, c))


def _contiguous_runs(shapes, parts):
    """Cuts `shapes` (in the given order) into at most `parts` contiguous runs
    minimising the largest rank_cost_us of a run (dynamic programming over cut
    points, ties towards the earlier cut). Returns [(start, end)] and costs."""
    n = len(shapes)
    cost = [[0.0] * (n + 1) for _ in range(n + 1)]
    for i in range(n):
        for j in range(i + 1, n + 1):
            cost[i][j] = rank_cost_us(shapes[i:j])
    inf = float("inf")
    k_max = max(1, min(parts, n))
    best = [[inf] * (n + 1) for _ in range(k_max + 1)]
    cut = [[0] * (n + 1) for _ in range(k_max + 1)]
    best[0][0] = 0.0
    for k in range(1, k_max + 1):
        for j in range(k, n + 1):
            for i in range(k - 1, j):
                v = max(best[k - 1][i], cost[i][j])
                if v < best[k][j] - 1e-9:
                    best[k][j], cut[k][j] = v, i
    bounds, j = [], n
    for k in range(k_max, 0, -1):
        i = cut[k][j]
        bounds.append((i, j))
        j = i
    bounds.reverse()
    return bounds, [cost[i][j] for i, j in bounds]


def assign_matrices(shapes, world, method: str = "lpt"):
    """Owner rank per matrix and each rank's load.

    "lpt": greedy longest-processing-time on gram_cost (load in FLOPs).
    "runs": matrices sorted by shape (largest n first, tall before wide, the
    one-CTA small matrices last) and cut into `world` contiguous runs that
    minimise the largest modelled rank cost (load in modelled microseconds);
    each rank then holds one or two shape batches, so its GEMM launches have
    as many tiles as its share allows. Both are deterministic, so every rank
    computes the same assignment."""
    n = len(shapes)
    if n == 0:
        return [], [0.0] * world
    if method == "lpt":
        order = sorted(range(n), key=lambda i: (-gram_cost(shapes[i]), i))
        load = [0.0] * world
        owner = [0] * n
        for i in order:
            k = min(range(world), key=lambda r: (load[r], r))
            owner[i] = k
            load[k] += gram_cost(shapes[i])
        return owner, load
    if method != "runs":
        raise ValueError("assignment must be 'lpt' or 'runs'")
    order = sorted(range(n), key=lambda i: (_shape_order_key(shapes[i]), i))
    bounds, costs = _contiguous_runs([tuple(shapes[i]) for i in order], world)
    owner = [0] * n
    load = [0.0] * world
    for rank, ((i, j), c) in enumerate(zip(bounds, costs)):
        for pos in range(i, j):
            owner[order[pos]] = rank
        load[rank] = c
    return owner, load


def split_waves(shapes, waves: int):
    """Splits one rank's matrices (indices into `shapes`) into `waves` runs of
    similar modelled cost, each run one or two shape batches."""
    n = len(shapes)
    if waves <= 1 or n <= 1:
        return [list(range(n))]
    order = sorted(range(n), key=lambda i: (_shape_order_key(shapes[i]), i))
    bounds, _ = _contiguous_runs([tuple(shapes[i]) for i in order], waves)
    return [sorted(order[i:j]) for i, j in bounds]


class ShardedStep:
    def __init__(self, model, muon, adamw, ema, world: int, rank: int, group=None, min_rows_shard: int = 1024,
                 exchange: str = "auto", push_streams: int = 1, waves: int | None = None, assignment: str = "lpt",
                 adamw_between_waves: bool = False):
        """exchange: "ce" (copy-engine pushes of the tables and the arena),
        "hybrid" (copy-engine pushes of the tables, overlapped with NorMuon;
        NCCL all-gather of the arena), "nccl" (all-gathers only) or "auto"
        ("ce" where every rank can export its buffers).
        Copy-engine modes fall back to NCCL where a rank cannot export its
        buffers ("auto") or raise. push_streams: streams the pushes are spread
        over; peers are visited in ring order rank+1, rank+2, ... so with one
        stream every rank sends to one peer at a time.
        waves: each rank steps its NorMuon matrices in this many waves and
        starts exchanging a wave's weights as soon as that wave is applied, so
        the exchange overlaps the next wave's compute (the arena is laid out
        wave by wave, each wave rank by rank). None: two waves from four ranks
        on where each rank holds at least 16 NorMuon matrices, else one.
        assignment: "lpt" or "runs" (see assign_matrices).
        adamw_between_waves: with two or more waves, run AdamW after the first
        NorMuon wave instead of before NorMuon, so the first wave's exchange
        also overlaps AdamW (the tables are then exchanged while the later
        waves compute). Measured slower on 4 GPUs (L14: 2.06 against 1.76 ms;
        the table pushes start later and share NVLink with the last wave's
        all-gather), hence off by default."""
        if exchange not in ("auto", "ce", "hybrid", "nccl"):
            raise ValueError("exchange must be 'auto', 'ce', 'hybrid' or 'nccl'")
        required = exchange != "auto"
        if exchange == "auto":
            # measured (L14 step): copy-engine pushes of the arena win at every
            # size (4 ranks, two waves: 1.50 against 1.77 ms, because a wave's
            # NCCL all-gather takes SMs from the next wave's GEMMs, 597 against
            # 741 TFLOP/s; 8 ranks, one wave: 1.52 against 1.58 ms)
            exchange = "ce"
        self.world, self.rank, self.group = world, rank, group
        self.push_streams = max(1, min(int(push_streams), max(1, world - 1)))
        self.muon, self.adamw, self.ema = muon, adamw, ema
        mparams = [p for g in muon.param_groups for p in g["params"]]
        owner, self.load = assign_matrices([tuple(p.shape) for p in mparams], world, assignment)
        self.assignment = assignment
        self.owner = {id(p): k for p, k in zip(mparams, owner)}
        muon._owned = {id(p) for p, k in zip(mparams, owner) if k == rank}
        self.owned_all = muon._owned
        # every rank's matrices split into the same number of waves
        if waves is None:
            # two waves only where each rank keeps batches large enough to fill
            # the GEMMs (measured, L14 step: 4 ranks / ~18 matrices each, 1.77
            # ms with two waves against 1.87; 8 ranks / ~9 each, 1.77 against
            # 1.57; 2 ranks, equal)
            waves = 2 if world > 2 and len(mparams) / world >= 16 else 1
        self.waves = max(1, int(waves))
        self.adamw_between_waves = bool(adamw_between_waves) and self.waves > 1
        # which optimizer reads its gradients first in step() (callers streaming gradients in)
        self.first_optimizer = "normuon" if self.adamw_between_waves else "adamw"
        per_rank = [[p for p, k in zip(mparams, owner) if k == r] for r in range(world)]
        wave_of = {}
        for r, ps in enumerate(per_rank):
            for w, idx in enumerate(split_waves([tuple(p.shape) for p in ps], self.waves)):
                for i in idx:
                    wave_of[id(ps[i])] = w
        self.wave_owned = [{id(p) for p in per_rank[rank] if wave_of[id(p)] == w} for w in range(self.waves)]
        # flat arena: wave by wave, each wave's region rank by rank (equal chunks
        # per wave, so each wave is one all-gather)
        dt = mparams[0].dtype if mparams else torch.bfloat16
        dev = mparams[0].device if mparams else torch.device("cuda")
        align = 64
        rnd = lambda n: (n + align - 1) // align * align  # noqa: E731
        self.arena_waves = []  # (base element, chunk elements, used elements per rank)
        base = 0
        for w in range(self.waves):
            used = [sum(rnd(p.numel()) for p in ps if wave_of[id(p)] == w) for ps in per_rank]
            chunk = max(used) if used else 0
            self.arena_waves.append((base, chunk, used))
            base += chunk * world
        self.arena = torch.empty(base, dtype=dt, device=dev)
        for w, (wbase, chunk, _) in enumerate(self.arena_waves):
            for r, ps in enumerate(per_rank):
                off = wbase + r * chunk
                for p in ps:
                    if wave_of[id(p)] != w:
                        continue
                    if p.dtype != dt:
                        raise ValueError("NorMuon parameters must share one dtype for the gather arena")
                    n = p.numel()
                    view = self.arena[off:off + n].view_as(p)
                    view.copy_(p.data)
                    p.data = view
                    off += rnd(n)
        self.chunk = sum(c for _, c, _ in self.arena_waves)  # elements per rank over all waves
        # AdamW row shards
        self.row_sharded = []
        slices = {}
        for g in adamw.param_groups:
            for p in g["params"]:
                rows = p.shape[0] if p.dim() >= 1 else 0
                if p.dim() >= 2 and p.numel() >= min_rows_shard * world and p.numel() % world == 0:
                    per = p.numel() // world
                    slices[id(p)] = (rank * per, per)
                    self.row_sharded.append(p)
                else:
                    slices[id(p)] = (0, p.numel())  # replicated small tensor
                del rows
        adamw._owned_slices = slices
        # EMA: skip (until gather_ema) the shadows of other ranks' NorMuon matrices
        if ema is not None:
            skip = set()
            for i, p in enumerate(ema.params):
                k = self.owner.get(id(p))
                if k is not None and k != rank:
                    skip.add(i)
            ema._skip = skip
        self.exchange = "nccl"
        self._bases = []
        self._streams = []
        self._plans = None
        self._requested = exchange
        if world > 1 and exchange != "nccl":
            self._setup_peer_exchange(required=required)

    # ------------------------------------------------------------ layout ---
    def buffers(self):
        """Tensors exchanged between ranks: the NorMuon arena, then each row-sharded table."""
        return [self.arena] + [p.data for p in self.row_sharded]

    def arena_regions(self, rank: int):
        """(wave, byte offset, bytes) of the arena parts `rank` updates."""
        es = self.arena.element_size()
        return [(w, (base + rank * chunk) * es, used[rank] * es)
                for w, (base, chunk, used) in enumerate(self.arena_waves) if used[rank]]

    def owned_regions(self, rank: int):
        """(buffer index, byte offset, bytes) of what `rank` updates in each exchanged buffer."""
        regions = [(0, off, nbytes) for _, off, nbytes in self.arena_regions(rank)]
        for i, p in enumerate(self.row_sharded):
            per = p.numel() // self.world
            regions.append((1 + i, rank * per * p.element_size(), per * p.element_size()))
        return regions

    def _setup_peer_exchange(self, required: bool):
        bufs = self.buffers()
        dev = self.arena.device
        mine = None
        if dev.type == "cuda":
            try:
                with torch.cuda.device(dev):
                    mine = [(*_lib.ipc_export(b.data_ptr()), b.numel() * b.element_size()) for b in bufs]
            except RuntimeError:
                mine = None
        every = [None] * self.world
        dist.all_gather_object(every, mine, group=self.group)
        if any(e is None for e in every):
            if required:
                raise RuntimeError("sharded step: copy-engine exchange needs CUDA IPC export on every rank")
            return  # NCCL all-gathers on every rank (all ranks saw the same list)
        for r, e in enumerate(every):
            if [n for _, _, n in e] != [n for _, _, n in mine]:
                raise RuntimeError(f"sharded step: rank {r} laid out its exchanged buffers differently")
        opened = {}
        peer_ptrs = {}
        with torch.cuda.device(dev):
            for q in range(self.world):
                if q == self.rank:
                    continue
                ptrs = []
                for handle, off, _ in every[q]:
                    if handle not in opened:
                        opened[handle] = _lib.ipc_import(handle)
                        self._bases.append(opened[handle])
                    ptrs.append(opened[handle] + off)
                peer_ptrs[q] = ptrs
            self._streams = [torch.cuda.Stream(dev) for _ in range(self.push_streams)]
        local = [b.data_ptr() for b in bufs]
        # per stream, the copies in ring order of the peers
        plans = {"tables": [[] for _ in self._streams]}
        for w in range(self.waves):
            plans[f"arena{w}"] = [[] for _ in self._streams]
        for d in range(1, self.world):
            q = (self.rank + d) % self.world
            st = (d - 1) % self.push_streams
            for w, off, nbytes in self.arena_regions(self.rank):
                plans[f"arena{w}"][st].append((peer_ptrs[q][0] + off, local[0] + off, nbytes))
            for k, off, nbytes in self.owned_regions(self.rank):
                if k > 0:
                    plans["tables"][st].append((peer_ptrs[q][k] + off, local[k] + off, nbytes))
        # ctypes argument arrays built once: the pushes reuse them every step
        self._plans = {k: [_lib.copy_args(c) if c else None for c in per_stream] for k, per_stream in plans.items()}
        self._flag = torch.zeros(1, dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            self._push_ev = torch.cuda.Event()
        self.exchange = self._requested

    def _push(self, which):
        cur = torch.cuda.current_stream()
        ev = self._push_ev  # reused: each wait takes the event as recorded at that moment
        ev.record(cur)
        for st, args in zip(self._streams, self._plans[which]):
            if args is not None:
                st.wait_event(ev)
                _lib.copy_async_args(args, st.cuda_stream)

    def _join_pushes(self):
        cur = torch.cuda.current_stream()
        for st in self._streams:
            cur.wait_stream(st)

    def close(self):
        """Unmaps the peers' buffers (call on every rank before freeing the model)."""
        if not self._bases:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for b in self._bases:
            _lib.ipc_close(b)
        self._bases = []
        self._plans = None
        self.exchange = "nccl"
        dist.barrier(group=self.group)

    def _gather_tables(self, async_op=False):
        works = []
        for p in self.row_sharded:
            flat = p.data.view(-1)
            per = flat.numel() // self.world
            w = dist.all_gather_into_tensor(flat, flat[self.rank * per:(self.rank + 1) * per], group=self.group,
                                            async_op=async_op)
            if async_op:
                works.append(w)
        return works

    def _gather_arena_wave(self, w, async_op=False):
        base, chunk, _ = self.arena_waves[w]
        if not chunk:
            return None
        region = self.arena[base:base + chunk * self.world]
        mine = region[self.rank * chunk:(self.rank + 1) * chunk]
        return dist.all_gather_into_tensor(region, mine, group=self.group, async_op=async_op)

    def _gather_arena(self, async_op=False):
        works = [self._gather_arena_wave(w, async_op) for w in range(self.waves)]
        return [x for x in works if x is not None]

    @torch.no_grad()
    def gather(self):
        """All-gathers the updated bf16 weights (in place)."""
        if self.world == 1:
            return
        self._gather_arena()
        self._gather_tables()

    @torch.no_grad()
    def step(self, mark=None, before=None):
        """One sharded optimizer step: AdamW first, so the vocabulary tables
        cross NVLink (copy-engine pushes, or NCCL all-gathers on NCCL's stream)
        while NorMuon computes; then NorMuon wave by wave, each wave's arena
        region exchanged as soon as the wave is applied (copy-engine pushes or
        an NCCL all-gather on NCCL's stream) while the next wave computes; the
        EMA update; the completion of every exchange.
        Same results as muon.step(); adamw.step(); ema.update(); gather().
        ``mark(name)``, when given, is called after each phase is enqueued
        (phase timing with events on the current stream); ``before(name)`` is
        called right before the AdamW ("adamw") and NorMuon ("normuon") steps
        (a caller streaming gradients in waits there for each optimizer's)."""
        mark = mark or (lambda name: None)
        before = before or (lambda name: None)
        push_tables = self.exchange in ("ce", "hybrid")
        works = []

        def adamw_and_tables():
            before("adamw")
            self.adamw.step()
            mark("adamw")
            if push_tables:
                self._push("tables")
            elif self.world > 1:
                works.extend(self._gather_tables(async_op=True))

        if not self.adamw_between_waves:
            adamw_and_tables()
        before("normuon")
        arena_works = []
        try:
            for w in range(self.waves):
                self.muon._owned = self.wave_owned[w]
                self.muon.step()
                if self.world > 1:
                    if self.exchange == "ce":
                        self._push(f"arena{w}")
                    elif w < self.waves - 1:
                        x = self._gather_arena_wave(w, async_op=True)
                        if x is not None:
                            arena_works.append(x)
                if w == 0 and self.adamw_between_waves:
                    self.muon._owned = self.owned_all
                    adamw_and_tables()
        finally:
            self.muon._owned = self.owned_all
        mark("normuon")
        if self.ema is not None:
            self.ema.update()
        if self.exchange == "ce":
            self._join_pushes()
            # every rank enters this collective only after its own pushes
            # landed, so its completion means every rank's pushes did
            dist.all_reduce(self._flag, group=self.group)
        elif self.world > 1:
            last = self._gather_arena_wave(self.waves - 1, async_op=True)
            if push_tables:
                # the last all-gather crosses NVLink together with the table
                # pushes still in flight; a one-element all-reduce, entered by
                # every rank after its own pushes landed and ordered after the
                # all-gathers on NCCL's stream, completes when both have
                self._join_pushes()
                dist.all_reduce(self._flag, group=self.group)
            for x in arena_works + ([last] if last is not None else []):
                x.wait()
        mark("arena_gather")
        for x in works:
            x.wait()
        mark("table_wait")

    @torch.no_grad()
    def reduce_gradients(self, average: bool = True, reduce_dtype=torch.float32):
        """Data-parallel gradient exchange before the sharded step (each rank
        computed gradients on its own data): every rank ends with the sum, or
        the mean, over ranks of the gradients it reads in step() -- its NorMuon
        matrices (one reduce-scatter over a gradient buffer laid out like the
        weight arena), its rows of the split tables (one reduce-scatter each)
        and the small replicated tensors (one all-reduce, packed). Other
        gradients keep their local values. Sums run in ``reduce_dtype``
        (fp32 by default: a bf16 sum over two ranks is rounded once) and are
        rounded to the gradient dtype after the optional division by the world
        size. Every rank must call it (collectives)."""
        if self.world == 1:
            return
        scale = (1.0 / self.world) if average else None
        mparams = [p for g in self.muon.param_groups for p in g["params"]]
        if self.chunk:
            dev = self.arena.device
            if getattr(self, "_grad_arena", None) is None or self._grad_arena.dtype != reduce_dtype:
                self._grad_arena = torch.zeros(self.arena.numel(), dtype=reduce_dtype, device=dev)
                self._grad_out = torch.empty(self.chunk, dtype=reduce_dtype, device=dev)
            base = self.arena.data_ptr()
            es = self.arena.element_size()
            offs = []
            for p in mparams:
                off = (p.data.data_ptr() - base) // es
                offs.append(off)
                if p.grad is not None:
                    self._grad_arena[off:off + p.numel()].copy_(p.grad.view(-1))
            # one reduce-scatter per wave region ([rank 0 | rank 1 | ...] each)
            out_base, ob = [], 0
            for base, chunk, _ in self.arena_waves:
                out_base.append(ob)
                if chunk:
                    dist.reduce_scatter_tensor(self._grad_out[ob:ob + chunk],
                                               self._grad_arena[base:base + chunk * self.world], group=self.group)
                ob += chunk
            if scale is not None:
                self._grad_out.mul_(scale)
            for p, off in zip(mparams, offs):
                if self.owner[id(p)] == self.rank and p.grad is not None:
                    for (base, chunk, _), o in zip(self.arena_waves, out_base):
                        lo = base + self.rank * chunk
                        if lo <= off < lo + chunk:
                            p.grad.view(-1).copy_(self._grad_out[o + off - lo:o + off - lo + p.numel()])
                            break
        for p in self.row_sharded:
            if p.grad is None:
                continue
            flat = p.grad.view(-1)
            per = flat.numel() // self.world
            out = torch.empty(per, dtype=reduce_dtype, device=flat.device)
            dist.reduce_scatter_tensor(out, flat.to(reduce_dtype), group=self.group)
            if scale is not None:
                out.mul_(scale)
            flat[self.rank * per:(self.rank + 1) * per].copy_(out)
        small = [p for g in self.adamw.param_groups for p in g["params"]
                 if p.grad is not None and not any(p is t for t in self.row_sharded)]
        if small:
            packed = torch.cat([p.grad.reshape(-1).to(reduce_dtype) for p in small])
            dist.all_reduce(packed, group=self.group)
            if scale is not None:
                packed.mul_(scale)
            off = 0
            for p in small:
                p.grad.view(-1).copy_(packed[off:off + p.numel()])
                off += p.numel()

    @torch.no_grad()
    def gather_state(self):
        """Completes every rank's optimizer state from the owners (for a
        checkpoint in the reference layout; collectives on every rank): the
        NorMuon state of each matrix from its owner, the AdamW state of the
        row-sharded tables from every rank's rows, and the EMA shadows."""
        if self.world == 1:
            return
        for g in self.muon.param_groups:
            for p in g["params"]:
                st = self.muon._init_state(p)  # zero state where this rank never stepped p
                for key in sorted(st):
                    dist.broadcast(st[key], src=self.owner[id(p)], group=self.group)
        for p in self.row_sharded:
            st = self.adamw._init_state(p)
            for key in ("exp_avg", "exp_avg_sq", "mant_rem"):
                if key in st:
                    flat = st[key].view(-1)
                    per = flat.numel() // self.world
                    dist.all_gather_into_tensor(flat, flat[self.rank * per:(self.rank + 1) * per].clone(),
                                                group=self.group)
        self.gather_ema()

    def drop_unowned_state(self):
        """Frees the NorMuon state of other ranks' matrices (after a checkpoint)."""
        if self.world == 1:
            return
        for g in self.muon.param_groups:
            for p in g["params"]:
                if self.owner[id(p)] != self.rank:
                    self.muon.state.pop(p, None)

    @torch.no_grad()
    def gather_ema(self):
        """Completes every rank's EMA shadows from their owners (for eval / checkpoints)."""
        if self.ema is None or self.world == 1:
            return
        for i, p in enumerate(self.ema.params):
            s = self.ema.shadow[i]
            k = self.owner.get(id(p))
            if k is not None:
                dist.broadcast(s, src=k, group=self.group)
            elif any(p is q for q in self.row_sharded):
                flat = s.view(-1)
                per = flat.numel() // self.world
                dist.all_gather_into_tensor(flat, flat[self.rank * per:(self.rank + 1) * per].clone(),
                                            group=self.group)
