"""Edge-stream elementwise chain in one pass on B200.

``edge_chain(terms, shape, activation=None)`` evaluates
``act(sum_t coef_t * a_t * b_t)`` over an ``[E, S, C]`` edge stream in one
kernel, each factor a float32 tensor broadcastable to ``shape`` (torch
broadcasting rules: a ``[E, 1, C]`` gate, a ``[E]``-shaped per-edge scale
given as ``[E, 1, 1]``, a ``[C]`` per-channel vector ...).  It is the
term-table kernel the reference plans for the elementwise pool of its DeepMD
profile (``docs/task2-hip-fusion-plan.md:280-302``: residual adds, gates and
broadcast multiply-adds over ``[E, 9/10, 64]`` rows, one ATen pass each); the
gain is the pass count -- every operand is read once and the result written
once.  Forward only (an inference fusion); the eager composition is the
oracle (``tests/test_gpu_chain.py``).
"""
from __future__ import annotations

from typing import Sequence

import torch

from .native import _extension, require_dcu

MAX_TERMS = 8
_ACTIVATIONS = {None: 0, "none": 0, "silu": 1, "sigmoid": 2}


def edge_chain(terms: Sequence[tuple], shape: Sequence[int], activation: str | None = None):
    """``act(sum_t coef_t * a_t * b_t)`` as a new contiguous float32 ``shape`` tensor.

    ``terms``: 1 to 8 tuples ``(coef, a)`` or ``(coef, a, b)``; ``coef`` a
    Python number, ``a`` / ``b`` float32 tensors on one CUDA device,
    broadcastable to ``shape`` = ``(E, S, C)``.  ``activation``: ``None``,
    ``"silu"`` (``z * sigmoid(z)``) or ``"sigmoid"``.  Terms are summed in
    the given order (fused multiply-adds), deterministically.
    """
    if len(shape) != 3 or any(int(x) < 0 for x in shape):
        raise ValueError("edge chain shape must be (n_edges, components, channels)")
    e, s, c = (int(x) for x in shape)
    if s == 0 or c == 0:
        raise ValueError("edge chain components and channels must be positive")
    if not 1 <= len(terms) <= MAX_TERMS:
        raise ValueError(f"edge chain takes 1 to {MAX_TERMS} terms")
    if activation not in _ACTIVATIONS:
        raise ValueError("edge chain activation must be None, 'silu' or 'sigmoid'")
    first, second, coefs = [], [], []
    for term in terms:
        if len(term) not in (2, 3):
            raise ValueError("an edge chain term is (coef, a) or (coef, a, b)")
        coef, *factors = term
        for f in factors:
            if not isinstance(f, torch.Tensor):
                raise TypeError("edge chain factors must be tensors")
            if f.dtype != torch.float32:
                raise TypeError("edge chain factors must be float32")
            try:
                torch.broadcast_shapes(tuple(f.shape), (e, s, c))
            except RuntimeError as error:
                raise ValueError(f"edge chain factor of shape {tuple(f.shape)} does not "
                                 f"broadcast to {(e, s, c)}") from error
            if torch.broadcast_shapes(tuple(f.shape), (e, s, c)) != (e, s, c):
                raise ValueError("edge chain factors may not enlarge the output shape")
            if f.requires_grad:
                raise RuntimeError("edge_chain is forward-only (an inference fusion)")
        first.append(factors[0])
        second.append(factors[1] if len(factors) == 2 else None)
        coefs.append(float(coef))
    tensors = [t for t in first + second if t is not None]
    if len({t.device for t in tensors}) != 1:
        raise ValueError("all edge chain factors must share a device")
    require_dcu(*tensors)
    return _extension("edge_chain").edge_chain(first, second, coefs, e, s, c,
                                               _ACTIVATIONS[activation])


__all__ = ["MAX_TERMS", "edge_chain"]
