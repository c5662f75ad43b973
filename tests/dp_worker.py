"""One rank of the 2-GPU data-parallel check (launched by test_gpu_dp.py).

Each rank runs the GPT value-and-grad on its half of the batch through a
world-size-2 session; the session all-reduces (mean) the loss and every
gradient with NCCL.  Rank 0 compares the result with a single-GPU session on the
full batch and writes the max relative error to the file given as argv[1].
With argv[2] == "overlap" the gradients are all-reduced in buckets on a second
stream while the backward runs (SB_SESSION_FLAG_OVERLAP_ALLREDUCE).  Three calls
with different token batches cover the eager first call and the CUDA-graph
capture and replay of the call with its all-reduce.
"""
import datetime
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    import numpy as np
    import torch
    import torch.distributed as dist
    from sheaf_lowering import models as M
    from sheaf_b200.session import B200Session, nccl_unique_id

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    c = M.GPTConfig(n_layer=2, n_head=2, n_embd=64, block_size=32, vocab_size=65, batch=8)
    b = c.batch // world
    inp = M.gpt_inputs(c, seed=3)
    obj = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    overlap = len(sys.argv) > 2 and sys.argv[2] == "overlap"
    sess = B200Session(device=local, precision="fp32", rank=rank, world_size=world, nccl_id=obj[0],
                       timeout_ms=60000, overlap_allreduce=overlap)
    low = M.gpt_vag(c, batch=b)
    sess.load_stablehlo(low.text)
    # three calls: the first runs eagerly, the second is captured into a CUDA
    # graph with its all-reduce, the third replays it; each call gets a new
    # token batch (new input buffers: staged by the replay)
    batches = [M.gpt_inputs(c, seed=3 + k) for k in range(3)]
    dps = []
    for bt in batches:
        ins = [bt[n][rank * b:(rank + 1) * b] if n in ("x", "y") else inp[n] for n in low.arg_names]
        outs = sess.call_device(low.qualified, ins, reduce=["mean"] * len(low.result_types))
        dps.append([o.to_host(timeout_ms=60000) for o in outs])
        for o in outs:
            o.release()
    dist.barrier()
    if rank == 0:
        full = M.gpt_vag(c)
        single = B200Session(device=local, precision="fp32")
        single.load_stablehlo(full.text)
        errs = []
        for bt, dp in zip(batches, dps):
            ref = single.call(full.qualified, [bt[n] if n in ("x", "y") else inp[n] for n in full.arg_names])
            errs += [float(np.max(np.abs(a - r)) / max(np.max(np.abs(r)), 1e-30)) for a, r in zip(dp, ref)]
        with open(sys.argv[1], "w") as f:
            json.dump({"max_rel": max(errs), "loss_dp": float(dps[-1][0])}, f)
        single.close()
    dist.barrier()
    sess.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
