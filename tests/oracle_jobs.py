"""Oracle evaluations of the full-size benchmark graphs, run in worker
processes (spawn) while the GPU computes the same graphs.

The f32 oracle needs about a minute per graph at these sizes; running them
side by side keeps the GPU test suite short.  Test infrastructure only.
"""
import numpy as np


def inputs(cfg_name, batch, seed):
    from sheaf_lowering import models as M
    cfg = getattr(M, cfg_name)
    return M.gpt_inputs(cfg, batch=batch, seed=seed)


def evaluate(text, qualified, arg_names, cfg_name, batch, seed):
    """Outputs of function `qualified` of `text` on the seeded inputs, f32."""
    from oracle.stablehlo_ref import run
    inp = inputs(cfg_name, batch, seed)
    return run(text, qualified, [inp[n] for n in arg_names], dtype=np.float32)


def sweep_last_output(op, shape, vjp, seed):
    """Last output (the op's result, or the VJP's dx) of an op-sweep program on
    its seeded inputs, f32."""
    from oracle.stablehlo_ref import run
    from sheaf_lowering import models as M
    low = M.sweep_program(op, shape, vjp)
    inp = M.sweep_inputs(op, shape, vjp, seed=seed)
    return run(low.text, low.qualified, [inp[n] for n in low.arg_names], dtype=np.float32)[-1]


_POOL = None


def pool():
    """A process pool for oracle jobs, started with `spawn` (never forked from
    a process that holds a CUDA context)."""
    global _POOL
    if _POOL is None:
        import multiprocessing as mp
        _POOL = mp.get_context("spawn").Pool(3)
    return _POOL
