"""Caller-provided gradient buffers for parameters.

A caller that wants a parameter's gradient in a particular place (the
data-parallel reducer keeps each all-reduce bucket's gradients in one flat
buffer) attaches a view of that place to the parameter. The backward of the
library's autograd functions then has its kernels write the weight and bias
gradients straight into the view, autograd takes the returned tensor as
``param.grad`` without a copy (it is the only reference), and the bucket's
all-reduce runs on the flat buffer with no gather or scatter pass.

A view is handed out at most once per arming, and only while
``param.grad`` is ``None``: when the gradient already exists (gradient
accumulation) autograd adds the new gradient into it, so the new one must not
live in the same memory; when one backward reaches the same parameter twice (a
layer applied twice), the second contribution must not overwrite the first.
The owner re-arms the views (``arm``) once it has consumed the gradients.
"""

from __future__ import annotations

import weakref

import torch

# id(param) -> [weakref to param, view, armed]
_views: dict[int, list] = {}
# callables (params, buffers) told when a backward has written gradients
_listeners: list = []


def attach(param: torch.Tensor, view: torch.Tensor) -> None:
    """Have the library's backward write ``param``'s gradient into ``view``
    (same number of elements, dtype and device as ``param``)."""
    if view.numel() != param.numel() or view.dtype != param.dtype or view.device != param.device:
        raise ValueError("a gradient view must match its parameter's size, dtype and device")
    _views[id(param)] = [weakref.ref(param), view, True]


def detach(param: torch.Tensor) -> None:
    _views.pop(id(param), None)


def arm(param: torch.Tensor) -> None:
    """Allow the view of ``param`` to be handed out again."""
    ent = _views.get(id(param))
    if ent is not None and ent[0]() is param:
        ent[2] = True


def view_of(param: torch.Tensor) -> torch.Tensor | None:
    ent = _views.get(id(param))
    if ent is not None and ent[0]() is param:
        return ent[1]
    return None


def grad_buffer(param: torch.Tensor | None, shape, dtype: torch.dtype,
                device: torch.device) -> torch.Tensor:
    """Tensor of ``shape`` for the backward to write ``param``'s gradient into:
    the attached view when one is armed and ``param.grad`` is ``None``, else a
    fresh allocation."""
    if param is not None:
        ent = _views.get(id(param))
        if ent is not None and ent[0]() is param and ent[2] and param.grad is None:
            view = ent[1]
            if view.dtype == dtype and view.device == device:
                ent[2] = False
                return view.view(shape)
    return torch.empty(shape, dtype=dtype, device=device)


def add_listener(fn) -> None:
    """Have ``fn(params, buffers)`` called whenever the library's backward has
    written the gradients of ``params`` into ``buffers`` (on the current
    stream, before the backward returns and before autograd stores them as
    ``param.grad``)."""
    _listeners.append(fn)


def remove_listener(fn) -> None:
    if fn in _listeners:
        _listeners.remove(fn)


def grads_written(params, buffers) -> None:
    """Called by a backward once the gradient kernels of ``params`` have been
    launched into ``buffers`` (the work that follows in the same backward may
    then overlap with whatever a listener starts)."""
    for fn in list(_listeners):
        fn(tuple(params), tuple(buffers))


__all__ = ["add_listener", "arm", "attach", "detach", "grad_buffer", "grads_written",
           "remove_listener", "view_of"]
