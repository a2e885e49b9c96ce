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

import torch

from . import _lib
from .ema import register_optimizer

MAX_GROUPS = 8


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
        for group in self.param_groups:
            for p in group["params"]:
                st = self.state.get(p)
                if st and "step" in st:
                    self._steps[id(p)] = int(float(st["step"].item()))

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        lib = _lib.load()
        # bucket by (device, param dtype, state dtype): one kernel launch each
        buckets = {}
        gtab = []
        for gi, group in enumerate(self.param_groups):
            if gi >= MAX_GROUPS:
                raise ValueError("at most 8 param groups")
            b1, b2 = group["betas"]
            gparams = [p for p in group["params"] if p.grad is not None]
            if not gparams:
                gtab.append(None)
                continue
            steps = set()
            for p in gparams:
                _lib.require_cuda(p, "AdamW.step")
                if p.grad.dtype != p.dtype or not p.is_contiguous() or not p.grad.is_contiguous():
                    raise ValueError("AdamW needs contiguous params and grads of the param dtype")
                st = self._init_state(p)
                self._steps[id(p)] = self._steps.get(id(p), 0) + 1
                steps.add(self._steps[id(p)])
                key = (p.device, p.dtype, st["exp_avg"].dtype)
                buckets.setdefault(key, []).append((p, st, gi))
            if len(steps) != 1:
                raise RuntimeError("params of one group have different step counts")
            lr, wd = float(group["lr"]), float(group["weight_decay"])
            # torch's fused kernel multiplies fp32(lr) * fp32(weight_decay)
            lr_wd = float(C.c_float(float(C.c_float(lr).value) * float(C.c_float(wd).value)).value)
            gs = self._grad_scale.data_ptr() if self._grad_scale is not None else None
            gtab.append(_lib.AdamwGroup(lr, float(b1), float(b2), float(group["eps"]), wd, lr_wd,
                                        float(steps.pop()), int(bool(self.cautious_wd)), gs))
        groups = (_lib.AdamwGroup * max(1, len(gtab)))()
        for i, g in enumerate(gtab):
            if g is not None:
                groups[i] = g
        for (dev, pdt, sdt), items in buckets.items():
            descs = []
            for p, st, gi in items:
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
                    p.grad.data_ptr() + start * esz,
                    st["exp_avg"].data_ptr() + start * ssz,
                    st["exp_avg_sq"].data_ptr() + start * ssz,
                    (shadow.data_ptr() + start * 4) if shadow is not None else None,
                    n, gi, 0, st["step"].data_ptr()))
            if not descs:
                continue
            if self._ema is not None:
                for p, st, gi in items:
                    if self._ema._lookup(p) is not None and (
                            self._owned_slices is None or id(p) in self._owned_slices):
                        self._ema._mark(p)
            arr = (_lib.AdamwTensor * len(descs))(*descs)
            rc = lib.b2o_adamw_step(arr, len(descs), groups, len(gtab), _lib.dtype_code(pdt),
                                    _lib.dtype_code(sdt), self._ema_weight, _lib.stream_ptr(dev))
            _lib.check(rc, "adamw_step")
        self._grad_scale = None
        return loss
