"""Data-parallel decomposition on CPU ranks (gloo, world size 2).

Each rank evaluates the value-and-grad graph on its half of the batch (the
sharding `bench.py` and `sb_session_call(..., SB_REDUCE_MEAN)` use); the mean
over ranks of the loss and of every gradient must equal the full-batch value,
because Sheaf's cross-entropy is a mean over tokens (sheaf/lib/nn.shf:50-56).
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from oracle.stablehlo_ref import run
    from sheaf_lowering import models as M
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = M.GPTConfig(n_layer=1, n_head=2, n_embd=16, block_size=8, vocab_size=11, batch=4)
        b = c.batch // world
        inp = M.gpt_inputs(c, seed=5)
        low = M.gpt_vag(c, batch=b)
        ins = [inp[n][rank * b:(rank + 1) * b] if n in ("x", "y") else inp[n] for n in low.arg_names]
        outs = run(low.text, low.qualified, ins)
        red = []
        for o in outs:
            t = torch.tensor(np.asarray(o, np.float64))
            dist.all_reduce(t)
            red.append((t / world).numpy())
        if rank == 0:
            q.put(red)
    finally:
        dist.destroy_process_group()


def test_two_rank_mean_equals_full_batch():
    from oracle.stablehlo_ref import run
    from sheaf_lowering import models as M
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    red = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    c = M.GPTConfig(n_layer=1, n_head=2, n_embd=16, block_size=8, vocab_size=11, batch=4)
    low = M.gpt_vag(c)
    inp = M.gpt_inputs(c, seed=5)
    full = run(low.text, low.qualified, [inp[n] for n in low.arg_names])
    for a, f in zip(red, full):
        np.testing.assert_allclose(a, f, rtol=1e-10, atol=1e-12)
