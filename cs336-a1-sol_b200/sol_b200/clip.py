"""Gradient-norm clip on the engine.

Drop-in for ``torch.nn.utils.clip_grad_norm_(params, max_norm, foreach=True)``
as transformer_lm/train_sol.py:498-499 calls it (2-norm, the norm tensor
returned without a host sync). Same result, same dtype rules (per-tensor norms
in the gradient dtype, the total and the coefficient in the promoted dtype),
in three kernel launches (sum of squares, finalisation, in-place scaling).

``defer_to=(muon, adamw)`` skips the in-place scaling: the coefficient stays
on the device and the optimizers' next step reads every gradient as
dtype(g * coef), the value torch's in-place multiply would have left, so the
step is unchanged and one read + write pass over all gradients disappears.
``p.grad`` itself then keeps the unclipped values.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib

_DT = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16}


@torch.no_grad()
def clip_grad_norm_(parameters, max_norm, norm_type=2.0, error_if_nonfinite=False, foreach=None, *,
                    defer_to=None):
    if isinstance(parameters, torch.Tensor):
        parameters = [parameters]
    grads = [p.grad for p in parameters if p.grad is not None]
    if float(norm_type) != 2.0:
        raise ValueError("the engine's clip computes the 2-norm (the reference's call)")
    if not grads:
        return torch.tensor(0.0)
    dev = grads[0].device
    for g in grads:
        _lib.require_cuda(g, "clip_grad_norm_")
        if g.device != dev or g.dtype not in _DT or not g.is_contiguous():
            raise ValueError("clip_grad_norm_: contiguous fp32/bf16 gradients on one device")
    if len(grads) > 1024:
        raise ValueError("clip_grad_norm_: at most 1024 gradient tensors")
    lib = _lib.load()
    out = torch.empty(2, dtype=torch.float32, device=dev)  # [total norm, clip coefficient]
    stream = _lib.stream_ptr(dev)
    n = len(grads)
    ptrs = _lib.ptr_array([g.data_ptr() for g in grads])
    numels = (C.c_int64 * n)(*[g.numel() for g in grads])
    dtypes = (C.c_int * n)(*[_DT[g.dtype] for g in grads])
    scratch = torch.empty(lib.b2o_clip_scratch_floats(numels, n), dtype=torch.float32, device=dev)
    _lib.check(lib.b2o_clip_grad_norm(ptrs, numels, dtypes, n, float(max_norm), scratch.data_ptr(),
                                      out.data_ptr(), stream), "clip_grad_norm")
    if defer_to is None:
        _lib.check(lib.b2o_clip_scale(ptrs, numels, dtypes, n, out.data_ptr() + 4, stream), "clip_scale")
    if defer_to is not None:
        for opt in defer_to:
            opt._grad_scale = out[1:2]
    out_dtype = torch.float32 if any(g.dtype == torch.float32 for g in grads) else grads[0].dtype
    total = out[0].to(out_dtype)
    if error_if_nonfinite and not bool(torch.isfinite(total)):
        raise RuntimeError(f"The total norm of order {float(norm_type)} for gradients is non-finite, so it "
                           "cannot be clipped")
    return total
