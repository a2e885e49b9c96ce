"""NorMuonGNS on the B200 engine.

Drop-in for ``transformer_lm.sol_modules.NorMuonGNS`` (transformer_lm/sol_modules.py:330-425):
same constructor arguments, param-group keys, per-parameter state
(``momentum_buffer`` param dtype (r, c), ``v_row`` fp32 (r, 1), ``mant_rem`` bf16
(r, c) when ``bf16_master`` and the param is bf16) and the overridable
``_orthogonalize_batch(U, ns_steps)`` hook (:366).

Matrices are batched by exact shape (the reference buckets by
``tuple(p.shape)``, :380-383); one step is three kinds of library calls, with
no stacking copies:
  front  (momentum lerp + Nesterov, :390-394)  -> u (S, r, c) bf16 + norm partials
  orthogonalise (:395; GEMMs on tcgen05)       -> o (S, r, c) bf16 + row sums of o^2
  finish + apply (v_row lerp, scale factors, cautious WD, update, bf16
         mantissa split, EMA; :396-424).
The front and the finish + apply passes cover every batch of a parameter group
in one call each (one launch, resp. two); the orthogonalisation of all
batches that share m = min(r, c) is one call, so their m x m products run as
single batched GEMMs.
"""
from __future__ import annotations

import ctypes as C
import math
from collections import OrderedDict

import numpy as np
import torch

from . import _lib
from .ema import register_optimizer
from .polar_express import table_for

MAX_BATCH = 64  # matrices per launch (kernel-parameter tables)


def _load_state_keep_dtypes(opt, state_dict):
    """torch.optim.Optimizer.load_state_dict without the cast of floating-point
    state to the parameter dtype: tensors move to the parameter's device only."""
    saved = state_dict["state"]
    torch.optim.Optimizer.load_state_dict(opt, {"state": {}, "param_groups": state_dict["param_groups"]})
    params = [p for g in opt.param_groups for p in g["params"]]
    for idx, st in saved.items():
        p = params[int(idx)]
        opt.state[p] = {k: (v.detach().to(device=p.device).clone() if torch.is_tensor(v) else v)
                        for k, v in st.items()}


class NorMuonGNS(torch.optim.Optimizer):
    """NorMuon (Muon + per-row second moment) with a Newton-Schulz orthogonaliser.

    Extra keyword arguments (not in the reference signature):
      orthogonalizer: "gram" (Gram Newton-Schulz, the path the reference takes when
          gram-newton-schulz is installed) or "quintic" (the reference's fallback,
          zeropower_via_newtonschulz5, restated on the same GEMM engine).
      coefficients: "polar_express" or "quintic" coefficient table for "gram".
      reset_iterations: Gram restart steps (the reference passes [2], :357).
    """

    def __init__(self, params, lr=2e-3, momentum=0.95, beta2=0.95, nesterov=True, ns_steps=5,
                 weight_decay=0.0, cautious_wd=False, bf16_master=False, *, orthogonalizer="gram",
                 coefficients="polar_express", reset_iterations=(2,), norm_eps=1e-7, norm_safety=1.0):
        super().__init__(params, dict(lr=lr, momentum=momentum, beta2=beta2, nesterov=nesterov,
                                      ns_steps=ns_steps, weight_decay=weight_decay))
        if orthogonalizer not in ("gram", "quintic"):
            raise ValueError("orthogonalizer must be 'gram' or 'quintic'")
        self.cautious_wd = cautious_wd
        self.bf16_master = bf16_master
        self.orthogonalizer = orthogonalizer
        self.coefficients = "quintic" if orthogonalizer == "quintic" else coefficients
        self.reset_iterations = tuple(int(x) for x in reset_iterations)
        self.norm_eps = float(norm_eps)
        self.norm_safety = float(norm_safety)
        self._ws = {}
        self._ows = {}
        self._tables = {}
        self._owned = None         # set of id(param) this rank updates (sharded step), None = all
        self._ema = None           # EmaWeights folded into the apply pass (set when it arms)
        self._ema_weight = 0.0
        # list -> (start event, end event, m, library launches) around each
        # orthogonaliser call (benchmark phase timing); None = off
        self._timing_events = None
        self._grad_scale = None    # device fp32 clip coefficient for the next step (clip_grad_norm_ defer_to)
        self._plans = {}           # (param-group index, owned set) -> cached launch descriptors (see step)
        register_optimizer(self)

    # ------------------------------------------------------------------ hooks
    def _orthogonalize_batch(self, U, ns_steps):
        """U: (S, r, c) bf16 CUDA tensor -> (S, r, c) bf16 (one call per shape batch)."""
        U = U.contiguous()
        _lib.require_cuda(U, "NorMuonGNS._orthogonalize_batch")
        S, r, c = U.shape
        ws = self._workspace(U.device, S, r, c)
        parts = ws["partial"].view(S, -1)
        parts.zero_()
        parts[:, 0] = U.float().pow(2).sum(dim=(1, 2))
        out = torch.empty_like(U)
        self._ortho(U, ws["partial"], S, r, c, ns_steps, out, ws)
        return out

    # -------------------------------------------------------------- internals
    def _table(self, ns_steps):
        key = (self.coefficients, ns_steps)
        if key not in self._tables:
            rows = table_for(self.coefficients, ns_steps)
            flat = [float(v) for row in rows for v in row]
            coeffs = (C.c_float * len(flat))(*flat)
            resets = (C.c_int * max(1, len(self.reset_iterations)))(*self.reset_iterations)
            self._tables[key] = (coeffs, resets, len(self.reset_iterations))
        return self._tables[key]

    def _workspace(self, device, S, r, c):
        key = (device, S, r, c)
        ws = self._ws.get(key)
        if ws is None:
            lib = _lib.load()
            rc = r * c
            nparts = lib.b2o_normuon_front_parts(rc)
            ntn = (c + 255) // 256
            wbytes = lib.b2o_ortho_workspace_bytes(S, r, c)
            ws = {
                "u": torch.empty((S, r, c), dtype=torch.bfloat16, device=device),
                "o": torch.empty((S, r, c), dtype=torch.bfloat16, device=device),
                "partial": torch.zeros(S * nparts, dtype=torch.float32, device=device),
                "rowsq": torch.zeros(S * ntn * r, dtype=torch.float32, device=device),
                "scratch": torch.empty(lib.b2o_normuon_apply_scratch_floats(S, r), dtype=torch.float32,
                                       device=device),
                "ortho_bytes": wbytes,
                # binary16 X0 written by the front: per-matrix power-of-two scale
                # (kept across steps), this step's factors, repair flags
                "prescale": torch.zeros(S, dtype=torch.float32, device=device),
                "xscale": torch.zeros(2 * S, dtype=torch.float32, device=device),
                "flags": torch.zeros(S, dtype=torch.int32, device=device),
            }
            self._ws[key] = ws
        return ws

    def _ortho_ws(self, device, key, nbytes):
        """Orthogonaliser workspace shared by the batches of one m-class (uint8, 256-byte aligned)."""
        buf = self._ows.get((device, key))
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
            self._ows[(device, key)] = buf
        return buf

    def _ortho(self, U, partial, S, r, c, ns_steps, out, ws):
        lib = _lib.load()
        coeffs, resets, nres = self._table(ns_steps)
        mode = 0 if self.orthogonalizer == "quintic" else 1
        ortho = self._ortho_ws(U.device, ("single", S, r, c), ws["ortho_bytes"])
        rc = lib.b2o_orthogonalize(U.data_ptr(), partial.data_ptr(), S, r, c, mode, coeffs, ns_steps, resets,
                                   nres, self.norm_eps, self.norm_safety, ortho.data_ptr(),
                                   ortho.numel(), out.data_ptr(), ws["rowsq"].data_ptr(),
                                   _lib.stream_ptr(U.device))
        _lib.check(rc, "orthogonalize")

    def load_state_dict(self, state_dict):
        """Loads param groups and per-parameter state keeping each saved tensor's
        dtype (torch's Optimizer.load_state_dict casts floating-point state to the
        parameter dtype, which would turn the fp32 v_row of bf16 matrices into
        bf16)."""
        _load_state_keep_dtypes(self, state_dict)
        self._plans = {}

    def _hook_overridden(self):
        return ("_orthogonalize_batch" in self.__dict__ or
                type(self)._orthogonalize_batch is not NorMuonGNS._orthogonalize_batch)

    def _init_state(self, p):
        st = self.state[p]
        if "momentum_buffer" not in st:
            st["momentum_buffer"] = torch.zeros_like(p)
            st["v_row"] = torch.zeros_like(p[..., 0:1], dtype=torch.float32)
        if self.bf16_master and p.dtype == torch.bfloat16 and "mant_rem" not in st:
            st["mant_rem"] = torch.zeros_like(p)
        return st

    def _prepare(self, params, shape, group):
        """Validates one exact-shape batch and returns its record (state, workspace)."""
        p0 = params[0]
        _lib.require_cuda(p0, "NorMuonGNS.step")
        dev = p0.device
        S = len(params)
        r, c = int(shape[-2]), int(shape[-1])
        for p in params:
            if p.dim() != 2:
                raise ValueError("NorMuonGNS handles 2-D parameters only")
            if p.grad.dtype != p.dtype or not p.is_contiguous() or not p.grad.is_contiguous():
                raise ValueError("NorMuonGNS needs contiguous params and grads of the param dtype")
        states = [self._init_state(p) for p in params]
        ws = self._workspace(dev, S, r, c)
        m, n = min(r, c), max(r, c)
        # the front writes the Gram iteration's binary16 input directly unless
        # the batch takes the one-CTA small-matrix path or another orthogonaliser
        x0 = (self.orthogonalizer == "gram" and not self._hook_overridden() and
              not (m <= 32 and m * n <= 49152))
        return dict(params=params, states=states, ws=ws, S=S, r=r, c=c, dev=dev, o=ws["o"], x0=x0)

    @staticmethod
    def _calls(recs, key):
        """Splits batch records into library calls: same key, <= 16 batches, <= 128 matrices."""
        calls = OrderedDict()
        for b in recs:
            calls.setdefault(key(b), []).append(b)
        for k, members in calls.items():
            cur, mats = [], 0
            for b in members:
                if cur and (len(cur) == 16 or mats + b["S"] > 128):
                    yield k, cur
                    cur, mats = [], 0
                cur.append(b)
                mats += b["S"]
            if cur:
                yield k, cur

    def _front_all(self, recs, group):
        """Momentum + Nesterov (sol_modules.py:390-394) for every batch: one launch per call."""
        lib = _lib.load()
        beta = float(group["momentum"])
        for (dev, dt), members in self._calls(recs, lambda b: (b["dev"], b["params"][0].dtype)):
            arr = (_lib.NormuonBatch * len(members))()
            keep = []
            for i, b in enumerate(members):
                grads = _lib.ptr_array([p.grad.data_ptr() for p in b["params"]])
                bufs = _lib.ptr_array([st["momentum_buffer"].data_ptr() for st in b["states"]])
                keep += [grads, bufs]
                ws = b["ws"]
                arr[i] = _lib.NormuonBatch(S=b["S"], r=b["r"], c=b["c"], grads=_lib.addr(grads),
                                           bufs=_lib.addr(bufs), u=ws["u"].data_ptr(),
                                           partial=ws["partial"].data_ptr(), prescale=ws["prescale"].data_ptr(),
                                           xscale=ws["xscale"].data_ptr(), flags=ws["flags"].data_ptr(),
                                           x0_half=int(b["x0"]))
            gs = self._grad_scale.data_ptr() if self._grad_scale is not None else None
            args = (arr, len(members), _lib.dtype_code(dt), 1.0 - beta, beta, int(bool(group["nesterov"])), gs)
            _lib.check(lib.b2o_normuon_front_multi(*args, _lib.stream_ptr(dev)), "normuon_front")
            if any(b["x0"] for b in members):
                _lib.check(lib.b2o_normuon_prescale(*args, self.norm_eps, self.norm_safety, _lib.stream_ptr(dev)),
                           "normuon_prescale")

    def _ortho_class(self, batches, ns_steps):
        """Orthogonalises every batch of one m = min(r, c) class with one library call."""
        lib = _lib.load()
        dev = batches[0]["dev"]
        coeffs, resets, nres = self._table(ns_steps)
        mode = 0 if self.orthogonalizer == "quintic" else 1
        groups = (_lib.OrthoGroup * len(batches))()
        for i, b in enumerate(batches):
            ws = b["ws"]
            groups[i] = _lib.OrthoGroup(ws["u"].data_ptr(), ws["partial"].data_ptr(), ws["o"].data_ptr(),
                                        ws["rowsq"].data_ptr(), b["S"], b["r"], b["c"], 0,
                                        ws["xscale"].data_ptr() if b.get("x0") else None)
        key = ("multi",) + tuple((b["S"], b["r"], b["c"]) for b in batches)
        nbytes = lib.b2o_ortho_workspace_bytes_multi(groups, len(batches))
        ortho = self._ortho_ws(dev, key, nbytes)
        ev = self._timing_events
        if ev is not None:
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record()
            n0 = _lib.launch_count()
        rc = lib.b2o_orthogonalize_multi(groups, len(batches), mode, coeffs, ns_steps, resets, nres, self.norm_eps,
                                         self.norm_safety, ortho.data_ptr(), ortho.numel(), _lib.stream_ptr(dev))
        _lib.check(rc, "orthogonalize_multi")
        if ev is not None:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record()
            ev.append((e0, e1, min(batches[0]["r"], batches[0]["c"]), _lib.launch_count() - n0))

    def _apply_all(self, recs, group):
        """v_row, normalisation, shape scale, cautious WD, update, mantissa split and
        EMA (sol_modules.py:396-424) for every batch: two launches per call."""
        lib = _lib.load()
        beta2 = float(group["beta2"])
        lr, wd = float(group["lr"]), float(group["weight_decay"])

        def key(b):
            p0 = b["params"][0]
            return (b["dev"], p0.dtype, bool(self.bf16_master and p0.dtype == torch.bfloat16))

        for (dev, dt, mt), members in self._calls(recs, key):
            arr = (_lib.NormuonBatch * len(members))()
            keep = []
            for i, b in enumerate(members):
                params, states, ws = b["params"], b["states"], b["ws"]
                pptr = _lib.ptr_array([p.data_ptr() for p in params])
                rems = _lib.ptr_array([st["mant_rem"].data_ptr() for st in states]) if mt else None
                vrows = _lib.ptr_array([st["v_row"].data_ptr() for st in states])
                emas = None
                if self._ema is not None:
                    shadows = [self._ema._lookup(p) for p in params]
                    if all(s is not None for s in shadows):
                        emas = _lib.ptr_array([s.data_ptr() for s in shadows])
                        for p in params:
                            self._ema._mark(p)
                keep += [pptr, rems, vrows, emas]
                arr[i] = _lib.NormuonBatch(S=b["S"], r=b["r"], c=b["c"],
                                           shape_scale=math.sqrt(max(1.0, b["r"] / b["c"])),
                                           o=b["o"].data_ptr(), rowsq=ws["rowsq"].data_ptr(),
                                           params=_lib.addr(pptr), rems=_lib.addr(rems), emas=_lib.addr(emas),
                                           vrows=_lib.addr(vrows), scratch=ws["scratch"].data_ptr())
            rc = lib.b2o_normuon_apply_multi(arr, len(members), _lib.dtype_code(dt), -lr, lr * wd, 1.0 - lr * wd,
                                             1 if wd else 0, int(bool(self.cautious_wd and wd)), 1.0 - beta2,
                                             self._ema_weight, _lib.stream_ptr(dev))
            _lib.check(rc, "normuon_apply")

    def _step_group(self, batches, group):
        """One parameter group through the per-step code path (used when
        _orthogonalize_batch is overridden: its output tensor changes every step)."""
        ns_steps = int(group["ns_steps"])
        recs = [self._prepare(params, shape, group) for shape, params in batches]
        self._front_all(recs, group)
        if self._hook_overridden():
            for b in recs:
                S, r, c = b["S"], b["r"], b["c"]
                o = self._orthogonalize_batch(b["ws"]["u"], ns_steps).to(torch.bfloat16).contiguous()
                ntn = (c + 255) // 256
                rs = b["ws"]["rowsq"].view(S, ntn, r)
                rs.zero_()
                rs[:, 0, :] = o.float().pow(2).sum(dim=-1)
                b["o"] = o
        else:
            classes = OrderedDict()
            for b in recs:
                classes.setdefault((b["dev"], min(b["r"], b["c"])), []).append(b)
            for members in classes.values():
                self._ortho_class(members, ns_steps)
        self._apply_all(recs, group)

    # ------------------------------------------------- cached launch plans --
    def invalidate_plan(self) -> None:
        """Drops the cached launch descriptors (rebuilt on the next step). Needed
        only after replacing a parameter's state dict or one of its state
        tensors by hand (load_state_dict does this itself); steps detect new
        parameters, moved parameter storage, gradients appearing or vanishing,
        EMA folding and shard changes themselves."""
        self._plans = {}

    def _build_plan(self, gi, params, group, key):
        """Every descriptor of one group's step except the gradient pointers:
        front calls (pointer tables of gradients and momentum buffers), one
        orthogonaliser call per m-class, finish + apply calls (parameters,
        remainders, v_row, EMA shadows)."""
        lib = _lib.load()
        by_shape = OrderedDict()  # exact-shape buckets in param order (sol_modules.py:380-383)
        for p in params:
            by_shape.setdefault(tuple(p.shape), []).append(p)
        batches = [(shape, ps[i:i + MAX_BATCH]) for shape, ps in by_shape.items()
                   for i in range(0, len(ps), MAX_BATCH)]
        recs = [self._prepare(ps, shape, group) for shape, ps in batches]
        keep = []
        # every gradient pointer table of the plan is a slice of one flat array,
        # refreshed each step with one vectorised write (gpos: slot of each param)
        gflat = (C.c_void_p * max(1, len(params)))()
        gpos_of, used = {}, 0
        front = []
        for (dev, dt), members in self._calls(recs, lambda b: (b["dev"], b["params"][0].dtype)):
            arr = (_lib.NormuonBatch * len(members))()
            for i, b in enumerate(members):
                grads = (C.c_void_p * b["S"]).from_buffer(gflat, used * C.sizeof(C.c_void_p))
                bufs = _lib.ptr_array([st["momentum_buffer"].data_ptr() for st in b["states"]])
                keep += [grads, bufs]
                for j, p in enumerate(b["params"]):
                    gpos_of[id(p)] = used + j
                used += b["S"]
                ws = b["ws"]
                arr[i] = _lib.NormuonBatch(S=b["S"], r=b["r"], c=b["c"], grads=_lib.addr(grads),
                                           bufs=_lib.addr(bufs), u=ws["u"].data_ptr(),
                                           partial=ws["partial"].data_ptr(), prescale=ws["prescale"].data_ptr(),
                                           xscale=ws["xscale"].data_ptr(), flags=ws["flags"].data_ptr(),
                                           x0_half=int(b["x0"]))
            front.append((arr, len(members), _lib.dtype_code(dt), _lib.stream_ptr(dev),
                          any(b["x0"] for b in members)))
        ortho = []
        classes = OrderedDict()
        for b in recs:
            classes.setdefault((b["dev"], min(b["r"], b["c"])), []).append(b)
        for (dev, m), members in classes.items():
            groups = (_lib.OrthoGroup * len(members))()
            for i, b in enumerate(members):
                ws = b["ws"]
                groups[i] = _lib.OrthoGroup(ws["u"].data_ptr(), ws["partial"].data_ptr(), ws["o"].data_ptr(),
                                            ws["rowsq"].data_ptr(), b["S"], b["r"], b["c"], 0,
                                            ws["xscale"].data_ptr() if b.get("x0") else None)
            okey = ("multi",) + tuple((b["S"], b["r"], b["c"]) for b in members)
            nbytes = lib.b2o_ortho_workspace_bytes_multi(groups, len(members))
            wsb = self._ortho_ws(dev, okey, nbytes)
            ortho.append((groups, len(members), wsb, _lib.stream_ptr(dev), m))
        apply, ema_idx = [], set()

        def akey(b):
            p0 = b["params"][0]
            return (b["dev"], p0.dtype, bool(self.bf16_master and p0.dtype == torch.bfloat16))

        for (dev, dt, mt), members in self._calls(recs, akey):
            arr = (_lib.NormuonBatch * len(members))()
            for i, b in enumerate(members):
                ps, states, ws = b["params"], b["states"], b["ws"]
                pptr = _lib.ptr_array([p.data_ptr() for p in ps])
                rems = _lib.ptr_array([st["mant_rem"].data_ptr() for st in states]) if mt else None
                vrows = _lib.ptr_array([st["v_row"].data_ptr() for st in states])
                emas = None
                if self._ema is not None:
                    shadows = [self._ema._lookup(p) for p in ps]
                    if all(x is not None for x in shadows):
                        emas = _lib.ptr_array([x.data_ptr() for x in shadows])
                        ema_idx.update(self._ema._index[id(p)] for p in ps)
                keep += [pptr, rems, vrows, emas]
                arr[i] = _lib.NormuonBatch(S=b["S"], r=b["r"], c=b["c"],
                                           shape_scale=math.sqrt(max(1.0, b["r"] / b["c"])),
                                           o=ws["o"].data_ptr(), rowsq=ws["rowsq"].data_ptr(),
                                           params=_lib.addr(pptr), rems=_lib.addr(rems), emas=_lib.addr(emas),
                                           vrows=_lib.addr(vrows), scratch=ws["scratch"].data_ptr())
            apply.append((arr, len(members), _lib.dtype_code(dt), _lib.stream_ptr(dev)))
        states = [self.state[p] for p in params]
        return {"key": key, "ema": self._ema, "owned": self._owned, "state": self.state,
                "keep": (keep, params, states, recs, gflat), "front": front, "ortho": ortho, "apply": apply,
                "gview": np.frombuffer(gflat, dtype=np.uint64), "gpos": np.array([gpos_of[id(p)] for p in params]),
                "ema_idx": frozenset(ema_idx)}

    def _run_plan(self, plan, params, group):
        lib = _lib.load()
        plan["gview"][plan["gpos"]] = np.fromiter((p.grad.data_ptr() for p in params), dtype=np.uint64,
                                                  count=len(params))
        beta = float(group["momentum"])
        nesterov = int(bool(group["nesterov"]))
        gs = self._grad_scale.data_ptr() if self._grad_scale is not None else None
        for arr, n, dtc, stream, x0 in plan["front"]:
            args = (arr, n, dtc, 1.0 - beta, beta, nesterov, gs)
            _lib.check(lib.b2o_normuon_front_multi(*args, stream), "normuon_front")
            if x0:
                _lib.check(lib.b2o_normuon_prescale(*args, self.norm_eps, self.norm_safety, stream),
                           "normuon_prescale")
        ns_steps = int(group["ns_steps"])
        coeffs, resets, nres = self._table(ns_steps)
        mode = 0 if self.orthogonalizer == "quintic" else 1
        ev = self._timing_events
        for groups, n, wsb, stream, m in plan["ortho"]:
            if ev is not None:
                e0 = torch.cuda.Event(enable_timing=True)
                e0.record()
                n0 = _lib.launch_count()
            rc = lib.b2o_orthogonalize_multi(groups, n, mode, coeffs, ns_steps, resets, nres, self.norm_eps,
                                             self.norm_safety, wsb.data_ptr(), wsb.numel(), stream)
            _lib.check(rc, "orthogonalize_multi")
            if ev is not None:
                e1 = torch.cuda.Event(enable_timing=True)
                e1.record()
                ev.append((e0, e1, m, _lib.launch_count() - n0))
        beta2 = float(group["beta2"])
        lr, wd = float(group["lr"]), float(group["weight_decay"])
        for arr, n, dtc, stream in plan["apply"]:
            rc = lib.b2o_normuon_apply_multi(arr, n, dtc, -lr, lr * wd, 1.0 - lr * wd, 1 if wd else 0,
                                             int(bool(self.cautious_wd and wd)), 1.0 - beta2, self._ema_weight,
                                             stream)
            _lib.check(rc, "normuon_apply")
        if self._ema is not None and plan["ema_idx"]:
            self._ema._folded |= plan["ema_idx"]

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        hooked = self._hook_overridden()
        owned = self._owned
        for gi, group in enumerate(self.param_groups):
            params = []
            for p in group["params"]:
                g = p.grad
                if g is None or (owned is not None and id(p) not in owned):
                    continue
                if g.dtype != p.dtype or not g.is_contiguous():
                    raise ValueError("NorMuonGNS needs contiguous params and grads of the param dtype")
                params.append(p)
            if not params:
                continue
            if hooked:
                by_shape = OrderedDict()  # exact-shape buckets in param order (sol_modules.py:380-383)
                for p in params:
                    by_shape.setdefault(tuple(p.shape), []).append(p)
                self._step_group([(shape, ps[i:i + MAX_BATCH]) for shape, ps in by_shape.items()
                                  for i in range(0, len(ps), MAX_BATCH)], group)
                continue
            # The launch descriptors depend only on which parameters step, where
            # their storage and state live, the EMA folding and the shard: cached
            # across steps; gradient pointers and scalars are filled in each step.
            key = (tuple(map(id, params)), tuple([p.data_ptr() for p in params]), len(self.state))
            pkey = (gi, id(owned))  # a sharded step alternates between its waves' owned sets
            plan = self._plans.get(pkey)
            if (plan is None or plan["key"] != key or plan["ema"] is not self._ema or plan["owned"] is not owned
                    or plan["state"] is not self.state):
                plan = self._plans[pkey] = self._build_plan(gi, params, group, key)
            self._run_plan(plan, params, group)
        self._grad_scale = None
        return loss
