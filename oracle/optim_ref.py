"""CPU restatement of Sheaf's optimizer step as the nanoGPT training loop runs
it (examples/nanoGPT/train.shf:26-33): `clip-by-global-norm` then
`adamw-step`.  Test infrastructure only (the oracle for the fused device
optimizer); numpy float32 tensors with scalars evaluated in float64 first, as
Sheaf evaluates scalar expressions before they meet tensors.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

import numpy as np


def global_norm(leaves: Sequence[np.ndarray]) -> np.float32:
    """lib/optim.shf:72-75: sqrt(tree-reduce + (map (sum (** g 2)))) over the leaves."""
    total = np.float32(0.0)
    for g in leaves:
        total = np.float32(total + np.sum(np.asarray(g, np.float32) ** 2, dtype=np.float32))
    return np.float32(np.sqrt(total))


def clip_by_global_norm(leaves: Sequence[np.ndarray], max_norm: float) -> List[np.ndarray]:
    """lib/optim.shf:77-83: scale every leaf by min(1, max_norm / (norm + 1e-8))."""
    n = global_norm(leaves)
    factor = np.float32(min(np.float32(1.0), np.float32(max_norm) / np.float32(n + np.float32(1e-8))))
    return [np.asarray(g, np.float32) * factor for g in leaves]


def adamw_step(params, grads, m, v, t: int, lr, b1, b2, eps, wd) -> Tuple[list, list, list, int]:
    """lib/optim.shf:36-58: returns [new-params new-m new-v new-t]."""
    new_t = t + 1
    f = np.float32
    bcm = f(1.0 / (1.0 - b1 ** new_t))
    bcv = f(1.0 / (1.0 - b2 ** new_t))
    nm = [f(b1) * np.asarray(md, f) + f(1.0 - b1) * np.asarray(gd, f) for md, gd in zip(m, grads)]
    nv = [f(b2) * np.asarray(vd, f) + f(1.0 - b2) * (np.asarray(gd, f) * np.asarray(gd, f)) for vd, gd in zip(v, grads)]
    npar = [np.asarray(p, f) - f(lr) * (f(wd) * np.asarray(p, f) + (mh * bcm) / (np.sqrt(vh * bcv) + f(eps)))
            for p, mh, vh in zip(params, nm, nv)]
    return npar, nm, nv, new_t


def train_update(params, grads, m, v, t, lr, b1, b2, eps, wd, max_norm):
    """The optimizer half of train-step (train.shf:29-32)."""
    g = clip_by_global_norm(grads, max_norm) if max_norm > 0 else [np.asarray(x, np.float32) for x in grads]
    return adamw_step(params, g, m, v, t, lr, b1, b2, eps, wd)
