"""Checkpoints of the engine in the reference's file layout.

The reference saves ``{"model": model.state_dict(), "optimizer":
muon.state_dict(), "iteration": it}`` (transformer_lm/modules.py:538-560,
called at train_sol.py:538-541) and the EMA shadow as ``{param name: fp32
shadow}`` in ema_final.pt (train_sol.py:542-549, read back by
scripts/eval_canon.py:54-60). The same files come out of here, loadable by the
reference's own load_checkpoint; the engine adds the AdamW state under
"adamw" (the reference never saves it, so a resumed reference run would
restart AdamW's moments).

In a sharded step each rank holds only the optimizer state of what it
updates: save_checkpoint / ema_state_dict complete it from the owners first
(collectives on every rank), and rank 0 writes. Loading gives every rank the
full state; each uses its own part.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def _unwrap(model):
    return getattr(model, "_orig_mod", model)


def _rank0(sharded) -> bool:
    return sharded is None or sharded.world == 1 or sharded.rank == 0


def save_checkpoint(model, optimizer, iteration, out, *, adamw=None, sharded=None):
    """modules.py:538-550 layout (+ "adamw"). With ``sharded``, call on every
    rank; rank 0 writes."""
    if sharded is not None:
        sharded.gather_state()
    if _rank0(sharded):
        obj = {"model": _unwrap(model).state_dict(), "optimizer": optimizer.state_dict(), "iteration": iteration}
        if adamw is not None:
            obj["adamw"] = adamw.state_dict()
        torch.save(obj, out)
    if sharded is not None:
        sharded.drop_unowned_state()
        if sharded.world > 1:
            dist.barrier(group=sharded.group)


def load_checkpoint(src, model, optimizer, *, adamw=None, map_location=None):
    """modules.py:552-560: loads model and NorMuon state (and AdamW's when the
    file has it); returns the iteration."""
    obj = torch.load(src, map_location=map_location, weights_only=False)
    _unwrap(model).load_state_dict(obj["model"])
    optimizer.load_state_dict(obj["optimizer"])
    if adamw is not None and "adamw" in obj:
        adamw.load_state_dict(obj["adamw"])
    return obj["iteration"]


def ema_state_dict(model, ema, sharded=None):
    """{param name: fp32 shadow} as in ema_final.pt (train_sol.py:546-548)."""
    if sharded is not None:
        sharded.gather_ema()
    return {n: s for (n, _), s in zip(_unwrap(model).named_parameters(), ema.shadow)}


def save_ema(model, ema, out, sharded=None):
    sd = ema_state_dict(model, ema, sharded)
    if _rank0(sharded):
        torch.save(sd, out)


@torch.no_grad()
def load_ema(src, model, ema, map_location=None):
    """Restores EMA shadows saved by save_ema (or the reference's ema_final.pt)."""
    sd = torch.load(src, map_location=map_location, weights_only=False) if not isinstance(src, dict) else src
    for (n, _), s in zip(_unwrap(model).named_parameters(), ema.shadow):
        if n in sd:
            s.copy_(sd[n].to(device=s.device, dtype=s.dtype))
