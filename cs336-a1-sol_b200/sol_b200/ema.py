"""EMA (Polyak) weights on the B200 engine.

Drop-in for ``transformer_lm.sol_modules.EmaWeights`` (transformer_lm/sol_modules.py:1247-1280):
an fp32 ``shadow`` list aligned with ``named_parameters()`` (saved by
train_sol.py:547-549), ``update()`` and the ``averaged()`` context manager.

Folding. The reference updates the shadow with a separate pass after the
optimizer steps (train_sol.py:500-507). Here, once ``update()`` has run once
(EMA active from ``ema_start`` on, as in train_sol), the engine optimizers
apply ``shadow = lerp(shadow, p_new, 1 - decay)`` inside their own streaming
pass, and ``update()`` only lerps the parameters that no optimizer stepped
since the previous call. Callers must therefore call ``update()`` after every
step once they have started, which is what train_sol does; ``fuse=False``
keeps the separate pass.
"""
from __future__ import annotations

import weakref
from contextlib import contextmanager

import torch

from . import _lib

_OPTIMIZERS = weakref.WeakSet()


def register_optimizer(opt) -> None:
    """Engine optimizers register here so an EmaWeights can fold into them."""
    _OPTIMIZERS.add(opt)


class EmaWeights:
    def __init__(self, model, decay: float = 0.999, fuse: bool = True):
        self.decay = decay
        inner = getattr(model, "_orig_mod", model)
        self.params = [p for _, p in inner.named_parameters()]
        self.shadow = [p.detach().float().clone() for p in self.params]  # fp32 master average
        self._index = {id(p): i for i, p in enumerate(self.params)}
        self.fuse = fuse
        self._armed = False
        self._folded = set()
        self._attached = []
        self._skip = set()  # indices another rank updates in a sharded step (see sharding.py)

    @property
    def weight(self) -> float:
        return 1.0 - self.decay

    def _lookup(self, p):
        """fp32 shadow of p (or None) for an optimizer folding the EMA into its pass."""
        i = self._index.get(id(p))
        return None if i is None else self.shadow[i]

    def _mark(self, p):
        """Records that an optimizer pass has applied this step's EMA to p."""
        i = self._index.get(id(p))
        if i is not None:
            self._folded.add(i)

    def _arm(self):
        for opt in list(_OPTIMIZERS):
            owns = any(id(p) in self._index for g in opt.param_groups for p in g["params"])
            if owns:
                opt._ema = self
                opt._ema_weight = self.weight
                self._attached.append(opt)
        self._armed = True

    def disarm(self):
        for opt in self._attached:
            if opt._ema is self:
                opt._ema = None
        self._attached = []
        self._armed = False
        self._folded.clear()

    def _standalone(self, idx):
        if not idx:
            return
        lib = _lib.load()
        by = {}
        for i in idx:
            p = self.params[i]
            _lib.require_cuda(p, "EmaWeights.update")
            by.setdefault((p.device, p.dtype), []).append(i)
        for (dev, dt), ids in by.items():
            sh = _lib.ptr_array([self.shadow[i].data_ptr() for i in ids])
            pp = _lib.ptr_array([self.params[i].data_ptr() for i in ids])
            nn_ = (_lib.c_int64 * len(ids))(*[self.params[i].numel() for i in ids])
            rc = lib.b2o_ema_update(sh, pp, nn_, len(ids), _lib.dtype_code(dt), self.weight, _lib.stream_ptr(dev))
            _lib.check(rc, "ema_update")

    @torch.no_grad()
    def update(self):
        if not self._armed:
            self._standalone([i for i in range(len(self.params)) if i not in self._skip])
            if self.fuse:
                self._arm()
            return
        todo = [i for i in range(len(self.params)) if i not in self._folded and i not in self._skip]
        self._folded.clear()
        self._standalone(todo)

    @contextmanager
    def averaged(self):
        """Temporarily load the EMA weights (for eval), then restore training weights."""
        backup = [p.detach().clone() for p in self.params]
        lib = _lib.load()
        by = {}
        for i, p in enumerate(self.params):
            _lib.require_cuda(p, "EmaWeights.averaged")
            by.setdefault((p.device, p.dtype), []).append(i)
        for (dev, dt), ids in by.items():
            sh = _lib.ptr_array([self.shadow[i].data_ptr() for i in ids])
            pp = _lib.ptr_array([self.params[i].data_ptr() for i in ids])
            nn_ = (_lib.c_int64 * len(ids))(*[self.params[i].numel() for i in ids])
            _lib.check(lib.b2o_ema_copy_to_params(sh, pp, nn_, len(ids), _lib.dtype_code(dt),
                                                  _lib.stream_ptr(dev)), "ema_copy_to_params")
        try:
            yield
        finally:
            for p, b in zip(self.params, backup):
                p.data.copy_(b)
