"""Fused AdamW (+ EMA) on the B200 engine.

Drop-in for the ``torch.optim.AdamW(groups, betas=..., eps=..., fused=True)``
built by ``build_optimizers`` (transformer_lm/sol_modules.py:468-476). Same
defaults, param-group keys (lr, betas, eps, weight_decay, amsgrad, maximize,
foreach, capturable, differentiable, fused) and per-parameter state
(``step`` fp32 0-d tensor, ``exp_avg``, ``exp_avg_sq``).

Two storage modes:
  * reference (default): moments in the parameter dtype, exactly what torch's
    fused AdamW keeps for bf16 parameters; the arithmetic is torch's fused
    formula (ATen/native/cuda/fused_adam_utils.cuh, ADAMW mode) in fp32.
  * master="bf16_mt": bf16 parameter plus a bf16 low-mantissa remainder
    (``mant_rem``, the NorMuonGNS trick at sol_modules.py:406-424) and fp32
    moments (state_dtype=torch.float32); optional cautious weight decay.
One streaming kernel pass updates parameter, remainder, moments and (when an
EmaWeights object has armed folding) the fp32 EMA shadow.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from .ema import register_optimizer

MAX_GROUPS = 8
# b2o_adamw_tensor as 64-bit words (the gradient pointer is refreshed in place each step)
_DESC_WORDS = C.sizeof(_lib.AdamwTensor) // 8
_GRAD_WORD = _lib.AdamwTensor.grad.offset // 8
assert C.sizeof(_lib.AdamwTensor) % 8 == 0 and _lib.AdamwTensor.grad.offset % 8 == 0


class AdamW(torch.optim.Optimizer):
    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2, amsgrad=False, *,
                 maximize=False, foreach=None, capturable=False, differentiable=False, fused=None,
                 decoupled_weight_decay=True, master="none", state_dtype=None, cautious_wd=False):
        if amsgrad or maximize or capturable or differentiable or not decoupled_weight_decay:
            raise ValueError("the B200 AdamW implements the recipe's configuration: no amsgrad/maximize/"
                             "capturable/differentiable")
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, amsgrad=amsgrad,
                        maximize=maximize, foreach=foreach, capturable=capturable, differentiable=differentiable,
                        fused=fused, decoupled_weight_decay=True)
        super().__init__(params, defaults)
        if master not in ("none", "bf16_mt"):
            raise ValueError("master must be 'none' or 'bf16_mt'")
        self.master = master
        self.state_dtype = state_dtype
        self.cautious_wd = cautious_wd
        self._steps = {}           # id(param) -> int step count (mirrors state["step"])
        self._owned_slices = None  # id(param) -> (start_elem, numel) this rank updates
        self._ema = None           # EmaWeights folded into the pass (set when it arms)
        self._ema_weight = 0.0
        self._grad_scale = None    # device fp32 clip coefficient for the next step (clip_grad_norm_ defer_to)
        self._plan = None          # cached launch descriptors (see step)
        register_optimizer(self)

    def _init_state(self, p):
        st = self.state[p]
        if "step" not in st:
            st["step"] = torch.zeros((), dtype=torch.float32, device=p.device)
            sdt = self.state_dtype or p.dtype
            if self.master == "bf16_mt" and p.dtype == torch.bfloat16 and self.state_dtype is None:
                sdt = torch.float32
            st["exp_avg"] = torch.zeros_like(p, dtype=sdt, memory_format=torch.preserve_format)
            st["exp_avg_sq"] = torch.zeros_like(p, dtype=sdt, memory_format=torch.preserve_format)
            if self.master == "bf16_mt" and p.dtype == torch.bfloat16:
                st["mant_rem"] = torch.zeros_like(p)
            self._steps[id(p)] = int(st["step"].item()) if st["step"].device.type == "cpu" else 0
        return st


    def load_state_dict(self, state_dict):
        """Keeps each saved state tensor's dtype (fp32 moments of bf16 parameters
        in master mode; torch's loader would cast them to bf16)."""
        from .normuon import _load_state_keep_dtypes
        _load_state_keep_dtypes(self, state_dict)
        self._plan = None
        for group in self.param_groups:
            for p in group["params"]:
                st = self.state.get(p)
                if st and "step" in st:
                    self._steps[id(p)] = int(float(st["step"].item()))

    def invalidate_plan(self) -> None:
        """Drops the cached launch descriptors (rebuilt on the next step). Needed
        only after replacing a parameter's state dict or one of its state
        tensors by hand (load_state_dict does this itself); steps detect new
        parameters, moved parameter storage, gradients appearing or vanishing,
        EMA folding and shard changes themselves."""
        self._plan = None

    def _build_plan(self, ps, gis, key):
        """Launch descriptors for the parameters (with gradients) of this step:
        one b2o_adamw_tensor array per (device, param dtype, state dtype)
        bucket, with every pointer except the gradient's filled in."""
        buckets = {}
        step_of = {}
        for gi, p in zip(gis, ps):
            _lib.require_cuda(p, "AdamW.step")
            if not p.is_contiguous():
                raise ValueError("AdamW needs contiguous params and grads of the param dtype")
            st = self._init_state(p)
            if step_of.setdefault(gi, self._steps.get(id(p), 0)) != self._steps.get(id(p), 0):
                raise RuntimeError("params of one group have different step counts")
            buckets.setdefault((p.device, p.dtype, st["exp_avg"].dtype), []).append((gi, p, st))
        launches, ema_idx = [], set()
        pos = {id(p): i for i, p in enumerate(ps)}
        # (word view of a descriptor array, its rows, the items' positions in ps, byte offsets)
        refresh = []
        for (dev, pdt, sdt), members in buckets.items():
            descs, owners = [], []
            for gi, p, st in members:
                shadow = self._ema._lookup(p) if self._ema is not None else None
                rem = st.get("mant_rem")
                start, n = 0, p.numel()
                if self._owned_slices is not None:
                    sl = self._owned_slices.get(id(p))
                    if sl is None:
                        continue
                    start, n = sl
                esz = p.element_size()
                ssz = st["exp_avg"].element_size()
                descs.append(_lib.AdamwTensor(
                    p.data_ptr() + start * esz,
                    (rem.data_ptr() + start * 2) if rem is not None else None,
                    None,
                    st["exp_avg"].data_ptr() + start * ssz,
                    st["exp_avg_sq"].data_ptr() + start * ssz,
                    (shadow.data_ptr() + start * 4) if shadow is not None else None,
                    n, gi, 0, st["step"].data_ptr()))
                owners.append((p, start * esz))
                if shadow is not None:
                    ema_idx.add(self._ema._index[id(p)])
            if not descs:
                continue
            arr = (_lib.AdamwTensor * len(descs))(*descs)
            words = np.frombuffer(arr, dtype=np.uint64).reshape(len(descs), _DESC_WORDS)
            refresh.append((words, np.array([pos[id(p)] for p, _ in owners]),
                            np.array([off for _, off in owners], dtype=np.uint64)))
            launches.append((arr, len(descs), _lib.dtype_code(pdt), _lib.dtype_code(sdt), _lib.stream_ptr(dev)))
        by_group = {}
        for gi, p in zip(gis, ps):
            by_group.setdefault(gi, []).append(id(p))
        return {"key": key, "ema": self._ema, "owned": self._owned_slices, "state": self.state,
                "keep": ps, "launches": launches, "refresh": refresh, "groups": by_group,
                "ema_idx": frozenset(ema_idx)}

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        lib = _lib.load()
        ps, gs_, gis = [], [], []
        for gi, group in enumerate(self.param_groups):
            if gi >= MAX_GROUPS:
                raise ValueError("at most 8 param groups")
            for p in group["params"]:
                g = p.grad
                if g is not None:
                    if g.dtype != p.dtype or not g.is_contiguous():
                        raise ValueError("AdamW needs contiguous params and grads of the param dtype")
                    ps.append(p)
                    gs_.append(g)
                    gis.append(gi)
        # The launch descriptors depend only on which parameters step, where
        # their storage and state live, the EMA folding and the shard: cached
        # across steps; the gradient pointers are written into them each step.
        key = (tuple(gis), tuple(map(id, ps)), tuple([p.data_ptr() for p in ps]), len(self.state))
        plan = self._plan
        if (plan is None or plan["key"] != key or plan["ema"] is not self._ema or plan["owned"] is not
                self._owned_slices or plan["state"] is not self.state):
            plan = self._plan = self._build_plan(ps, gis, key)
        gptr = np.fromiter((g.data_ptr() for g in gs_), dtype=np.uint64, count=len(gs_))
        for words, where, offs in plan["refresh"]:
            words[:, _GRAD_WORD] = gptr[where] + offs
        steps_of = {}
        for gi, ids in plan["groups"].items():
            k = self._steps.get(ids[0], 0) + 1
            self._steps.update(dict.fromkeys(ids, k))
            steps_of[gi] = k
        gtab = []
        gsc = self._grad_scale.data_ptr() if self._grad_scale is not None else None
        for gi, group in enumerate(self.param_groups):
            if gi not in steps_of:
                gtab.append(None)
                continue
            b1, b2 = group["betas"]
            lr, wd = float(group["lr"]), float(group["weight_decay"])
            # torch's fused kernel multiplies fp32(lr) * fp32(weight_decay)
            lr_wd = float(C.c_float(float(C.c_float(lr).value) * float(C.c_float(wd).value)).value)
            gtab.append(_lib.AdamwGroup(lr, float(b1), float(b2), float(group["eps"]), wd, lr_wd,
                                        float(steps_of[gi]), int(bool(self.cautious_wd)), gsc))
        groups = (_lib.AdamwGroup * max(1, len(gtab)))()
        for i, g in enumerate(gtab):
            if g is not None:
                groups[i] = g
        for arr, n, pdt, sdt, stream in plan["launches"]:
            rc = lib.b2o_adamw_step(arr, n, groups, len(gtab), pdt, sdt, self._ema_weight, stream)
            _lib.check(rc, "adamw_step")
        if self._ema is not None and plan["ema_idx"]:
            self._ema._folded |= plan["ema_idx"]
        self._grad_scale = None
        return loss
