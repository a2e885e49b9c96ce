"""Sharded optimizer step over the GPUs of one node (NCCL over NVLink/NVSwitch).

The reference is single-GPU (no torch.distributed call sites); this is the
north-star's partitioned step. Placement never changes per-matrix arithmetic,
so every rank's result is bit-identical to the single-GPU engine.

  * NorMuon: whole matrices are assigned to ranks (greedy longest-processing-time
    on the Gram Newton-Schulz FLOP count); each rank batches its own matrices by
    shape. The NorMuon parameters are re-pointed into one flat bf16 arena laid
    out rank by rank, so the exchange is a single in-place all-gather.
  * AdamW: tables whose row count divides by the world size are split by rows
    (each rank updates its rows; in-place all-gather per table); the small
    scalar/gain tensors are updated redundantly by every rank (no exchange).
  * EMA: each rank folds the EMA of what it updates; shadows of other ranks'
    parameters are gathered on demand by gather_ema().
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def gram_cost(shape) -> float:
    r, c = shape[-2], shape[-1]
    m, n = min(r, c), max(r, c)
    return 6.0 * m * m * n + 20.0 * m ** 3


def assign_matrices(shapes, world):
    """Greedy LPT: returns owner rank per matrix (ties broken by rank index)."""
    order = sorted(range(len(shapes)), key=lambda i: (-gram_cost(shapes[i]), i))
    load = [0.0] * world
    owner = [0] * len(shapes)
    for i in order:
        k = min(range(world), key=lambda r: (load[r], r))
        owner[i] = k
        load[k] += gram_cost(shapes[i])
    return owner, load


class ShardedStep:
    def __init__(self, model, muon, adamw, ema, world: int, rank: int, group=None, min_rows_shard: int = 1024):
        self.world, self.rank, self.group = world, rank, group
        self.muon, self.adamw, self.ema = muon, adamw, ema
        mparams = [p for g in muon.param_groups for p in g["params"]]
        owner, self.load = assign_matrices([tuple(p.shape) for p in mparams], world)
        self.owner = {id(p): k for p, k in zip(mparams, owner)}
        muon._owned = {id(p) for p, k in zip(mparams, owner) if k == rank}
        # flat arena laid out rank by rank
        dt = mparams[0].dtype if mparams else torch.bfloat16
        dev = mparams[0].device if mparams else torch.device("cuda")
        per_rank = [[p for p, k in zip(mparams, owner) if k == r] for r in range(world)]
        align = 64
        sizes = [sum((p.numel() + align - 1) // align * align for p in ps) for ps in per_rank]
        self.chunk = max(sizes) if sizes else 0
        self.arena = torch.empty(self.chunk * world, dtype=dt, device=dev)
        for r, ps in enumerate(per_rank):
            off = r * self.chunk
            for p in ps:
                if p.dtype != dt:
                    raise ValueError("NorMuon parameters must share one dtype for the gather arena")
                n = p.numel()
                view = self.arena[off:off + n].view_as(p)
                view.copy_(p.data)
                p.data = view
                off += (n + align - 1) // align * align
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

    def _gather_arena(self, async_op=False):
        if not self.chunk:
            return None
        mine = self.arena[self.rank * self.chunk:(self.rank + 1) * self.chunk]
        return dist.all_gather_into_tensor(self.arena, mine, group=self.group, async_op=async_op)

    @torch.no_grad()
    def gather(self):
        """All-gathers the updated bf16 weights (in place)."""
        if self.world == 1:
            return
        self._gather_arena()
        self._gather_tables()

    @torch.no_grad()
    def step(self):
        """One sharded optimizer step: AdamW first, so the all-gathers of the
        vocabulary tables run on NCCL's stream while NorMuon computes; then
        NorMuon, the EMA update and the all-gather of the NorMuon arena.
        Same results as muon.step(); adamw.step(); ema.update(); gather()."""
        self.adamw.step()
        works = self._gather_tables(async_op=True) if self.world > 1 else []
        self.muon.step()
        if self.ema is not None:
            self.ema.update()
        if self.world > 1:
            self._gather_arena()
        for w in works:
            w.wait()

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
