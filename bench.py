#!/usr/bin/env python
"""Value-and-grad throughput of Sheaf's nanoGPT training step on B200.

Workload (default): the nanoGPT-style model of examples/nanoGPT/model.shf
(6 layers, d_model 384, 6 heads, ctx 256, vocab 65), value-and-grad of the
cross-entropy loss on shifted tokens, global batch 64 x 256 split over the
ranks (strong scaling); lowered to StableHLO as Sheaf's JIT lowers it and run
through libsheafb200's C ABI.  Other workloads: `gpt2` (GPT-2-small value-and-
grad: 12 layers, d768, ctx 1024, vocab 50304, batch 8 per GPU, weak scaling),
`nanogpt-fwd` (the forward alone), `nanogpt-train` (value-and-grad followed by
the fused clip-by-global-norm + AdamW step of examples/nanoGPT/train.shf),
`nanogpt-generate` (one generate-token step of sample.shf on the 256-token
window: forward, top-k sort, softmax, split, choice; tokens/s),
`mlp` (the 784-512-10 MLP value-and-grad, samples/s), `matmul` (op sweep,
--size / --shape / --layout).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--workload W]

Prints one JSON line (rank 0).  Device time: CUDA events on the session's
stream around K steps, max over ranks.  Inputs (weights, activations) are far
larger than the 126 MB L2, so no flush is needed between steps.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "value-and-grad steps/s & tokens/s at 1/2/4/8 B200; % of TC/HBM roofline"

# DRAM bytes (read + write) per GEMM launch, averaged over one step's GEMM
# launches, from an ncu capture of the same workload on one GPU (the bench
# itself runs no profiler): (workload, batch per rank, precision) -> (bytes,
# capture summary)
GEMM_TRAFFIC = {
    ("nanogpt", 64, "tf32"): (84.46e6, "profiles/gemm_dram_traffic_nanogpt_vag.md"),
}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--precision", default=os.environ.get("SHEAF_B200_PRECISION", "tf32"),
                   choices=["fp32", "tf32", "bf16"])
    p.add_argument("--workload", default="nanogpt",
                   choices=["nanogpt", "nanogpt-fwd", "nanogpt-train", "nanogpt-generate", "gpt2", "mlp", "matmul",
                            "ref-vag", "ref-forward", "sweep", "nanogpt-decode"])
    p.add_argument("--op", default="softmax", choices=["softmax", "layer-norm", "gelu"],
                   help="sweep workload: the op (on [65536, --dim], gelu on 2^28 elements)")
    p.add_argument("--dim", type=int, default=768, help="sweep workload: D of [65536, D]")
    p.add_argument("--dtype", default="f32", choices=["f32", "bf16"], help="sweep workload: tensor type")
    p.add_argument("--vjp", action="store_true", help="sweep workload: the VJP (value-and-grad) instead of the op")
    p.add_argument("--size", type=int, default=4096, help="matmul workload: M = N = K")
    p.add_argument("--shape", default="", help="matmul workload: M,N,K (overrides --size)")
    p.add_argument("--layout", default="nn", choices=["nn", "nt", "tn", "tt"],
                   help="matmul workload: operands stored transposed (t) or not (n)")
    p.add_argument("--batch", type=int, default=0,
                   help="global batch override (profiling captures on a smaller case)")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-profile", action="store_true")
    p.add_argument("--no-overlap", action="store_true",
                   help="data parallel: one all-reduce after the backward instead of buckets during it")
    return p.parse_args()


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def workload(name, world, batch=0):
    """(config, global batch, per-rank batch, scaling) of a GPT workload."""
    from sheaf_lowering import models as M
    if name in ("nanogpt", "nanogpt-fwd", "nanogpt-train"):
        c = M.NANOGPT
        gb = batch or c.batch
        if gb % world:
            raise SystemExit(f"global batch {gb} is not divisible by {world} ranks")
        return c, gb, gb // world, "strong"
    c = M.GPT2_SMALL
    b = batch or c.batch
    return c, b * world, b, "weak"


def program(args, world, rank):
    """The timed program: lowered module, host inputs of this rank, the names of
    the per-step data inputs, work units per step (all ranks), unit, scaling,
    config, and whether the outputs are data-parallel means (value-and-grad)."""
    from sheaf_lowering import models as M
    if args.workload == "mlp":
        gb = args.batch or 256
        if gb % world:
            raise SystemExit(f"global batch {gb} is not divisible by {world} ranks")
        b = gb // world
        low = M.mlp_vag(batch=b)
        full = M.mlp_inputs(batch=gb, seed=0)
        inp = dict(full)
        inp["x"], inp["y"] = full["x"][rank * b:(rank + 1) * b], full["y"][rank * b:(rank + 1) * b]
        cfg = {"workload": f"mlp value-and-grad {gb}x784", "model": "784-512-10 gelu, mse",
               "global_batch": gb, "parallelism": f"dp{world}",
               "l2": "operands fit in L2 (3.4 MB), no flush: launch-latency bound by design"}
        return low, inp, ["x", "y"], gb, "samples/s", "strong", cfg, True
    if args.workload in ("ref-vag", "ref-forward"):
        # the reference's own benchmark programs, one 64-token sequence per rank
        c = M.GPT2_BENCH
        vag = args.workload == "ref-vag"
        low = M.bench_vag_program(c) if vag else M.bench_forward_program(c)
        inp = M.bench_inputs(c, seed=42 + rank)
        src = "benchmarks/bench_vag_sheaf.shf (loss = mean of the logits)" if vag else "benchmarks/bench_forward.shf"
        cfg = {"workload": f"GPT-2 124M {'value-and-grad' if vag else 'forward'} {c.batch}x{c.T} ({src})",
               "model": f"L{c.n_layer} D{c.n_embd} H{c.n_head} T{c.T} V{c.vocab_size}", "global_batch": world,
               "seq_len": c.T, "parallelism": f"dp{world}",
               "l2": "weights (0.5 GB) exceed L2; no flush"}
        return low, inp, ["idx"], world * c.T, "tokens/s", "weak", cfg, vag
    if args.workload == "nanogpt-generate":
        from sheaf_lowering import generate as G
        from sheaf_lowering import random as RG
        c = M.NANOGPT
        low = G.gpt_generate_program(c, 200, 0.8)
        inp = M.gpt_inputs(c, batch=1, seed=0)
        inp = {n: inp[n] for n in low.arg_names[:-2]} | {"idx": inp["idx"], "key": RG.key_of_seed(1337)}
        cfg = {"workload": f"nanogpt generate-token (top-k 200, temperature 0.8) 1x{c.T}",
               "model": f"L{c.n_layer} D{c.n_embd} H{c.n_head} T{c.T} V{c.vocab_size}", "global_batch": world,
               "seq_len": c.T, "parallelism": f"replicas{world}",
               "l2": "weights (43 MB) fit in L2: one token per step, latency-bound by design"}
        return low, inp, ["idx", "key"], world, "tokens/s", "weak", cfg, False
    c, gb, b, scaling = workload(args.workload, world, args.batch)
    inp = M.gpt_inputs(c, batch=gb, seed=0)
    for n in ("x", "y", "idx"):
        inp[n] = inp[n][rank * b:(rank + 1) * b]
    fwd = args.workload == "nanogpt-fwd"
    low = M.gpt_fwd(c, batch=b) if fwd else M.gpt_vag(c, batch=b)
    kind = "forward" if fwd else ("train step (value-and-grad, clip-by-global-norm 1.0, adamw)"
                                  if args.workload == "nanogpt-train" else "value-and-grad")
    name = "gpt2-small" if args.workload == "gpt2" else "nanogpt"
    cfg = {"workload": f"{name} {kind} {gb}x{c.T}",
           "model": f"L{c.n_layer} D{c.n_embd} H{c.n_head} T{c.T} V{c.vocab_size}",
           "global_batch": gb, "seq_len": c.T, "parallelism": f"dp{world}",
           "l2": "inputs and activations exceed L2; no flush"}
    return low, inp, (["idx"] if fwd else ["x", "y"]), gb * c.T, "tokens/s", scaling, cfg, not fwd


class Clocks:
    """Samples nvidia-smi during the timed region (clock and throttle reasons)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.device), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for ln in self.proc.stdout:
            self.rows.append([x.strip() for x in ln.split(",")])

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            for k, n in enumerate(names):
                if len(r) > 5 + k and r[5 + k].lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows)}


def peaks(burst=False):
    """(HBM GB/s, dense bf16 TFLOP/s, source): the driver's measured peaks;
    the burst GEMM figure for a kernel timed alone, the sustained one for a
    kernel timed inside a long step."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return d["hbm_gbs"], d["bf16_tflops" if burst else "bf16_tflops_sustained"], "measured"
    except Exception:
        return 6650.0, 1590.0 if burst else 1400.0, "fallback"


def blas_threads():
    """Threads numpy's BLAS uses (the oracle's matrix products); element-wise
    numpy ops run on one thread."""
    try:
        from threadpoolctl import threadpool_info
        n = [d["num_threads"] for d in threadpool_info() if d.get("user_api") == "blas"]
        return max(n) if n else 1
    except Exception:
        return 1


def cpu_baseline(args, steps=2):
    """The oracle port (numpy f32) timed on a bounded sample of the same workload:
    the full MLP batch, 16 of the 64 nanoGPT sequences, or one GPT-2 sequence
    of 1024 tokens; same graph (value-and-grad or forward) as the device run."""
    from oracle.stablehlo_ref import evaluate, parse_module
    from sheaf_lowering import models as M
    if args.workload == "mlp":
        low, inp, units, unit = M.mlp_vag(batch=256), M.mlp_inputs(batch=256), 256, "samples/s"
        sample = "the full 256-sample batch"
    elif args.workload == "nanogpt-generate":
        low, inp, _, units, unit, _, _, _ = program(args, 1, 0)
        sample = "one generate-token step (1 token on the 256-token window)"
    elif args.workload in ("ref-vag", "ref-forward"):
        low, inp, _, units, unit, _, _, _ = program(args, 1, 0)
        sample = "the full program (1 x 64 tokens)"
    else:
        c = workload(args.workload, 1)[0]
        b, T = (16, c.T) if c.T <= 256 else (1, c.T)
        low = M.gpt_fwd(c, batch=b) if args.workload == "nanogpt-fwd" else M.gpt_vag(c, batch=b)
        inp, units, unit = M.gpt_inputs(c, batch=b), b * T, "tokens/s"
        sample = f"{b} sequence(s) x {T} tokens of the same model"
        if c.T > 256:
            steps = 1
    f = parse_module(low.text)[low.qualified]
    ins = [inp[n] for n in low.arg_names]
    train = args.workload == "nanogpt-train"
    params = [inp[n] for n in low.arg_names if n not in ("x", "y")]
    moments = [np.zeros_like(p) for p in params]

    def one():
        outs = evaluate(f, ins, dtype=np.float32)
        if train:
            from oracle.optim_ref import train_update
            train_update(params, outs[1:], moments, moments, 0, *TRAIN_HP)
    one()
    t0 = time.time()
    for _ in range(steps):
        one()
    dt = (time.time() - t0) / steps
    if train:
        sample = sample + " plus clip-by-global-norm + AdamW over all parameters (oracle/optim_ref.py)"
    nt = blas_threads()
    return {"value": units / dt, "unit": unit, "cores": nt, "kind": "port",
            "sample": f"{sample} per step, numpy float32 interpretation of the same StableHLO "
                      f"(oracle/stablehlo_ref.py), mean of {steps} steps after one untimed step; "
                      f"matrix products on {nt} BLAS threads, element-wise ops on 1 thread "
                      f"(host has {os.cpu_count()} cores)"}


# train.shf:29-32: clip-by-global-norm 1.0, adamw-step lr b1 b2 eps wd (lr as
# nanoGPT's shakespeare-char config, before any schedule)
TRAIN_HP = (1e-3, 0.9, 0.95, 1e-8, 0.1, 1.0)


def run_reference(args):
    rank, _, world = env_rank()
    if rank != 0:
        return
    _, _, _, _, unit, scaling, cfg, _ = program(args, world, 0)
    res = cpu_baseline(args, steps=max(1, min(args.steps, 3)))
    line = {"impl": "reference", "metric": METRIC, "value": res["value"], "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
            "cpu_baseline": res,
            "e2e": {"value": res["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference's IREE llvm-cpu path cannot be built here (no Rust toolchain, no IREE); "
                    "this times the CPU restatement of the same graphs on the host cores"}
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    rank, local, world = env_rank()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    from sheaf_b200 import build
    from sheaf_lowering import models as M
    from sheaf_b200.session import B200Session, library, nccl_unique_id
    build.build()
    low, inp, data_names, units, unit, scaling, cfg, vag = program(args, world, rank)
    nid = None
    if world > 1:
        obj = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nid = obj[0]
    sess = B200Session(device=local, precision=args.precision, rank=rank, world_size=world, nccl_id=nid,
                       timeout_ms=300000, overlap_allreduce=not args.no_overlap)
    t0 = time.time()
    sess.load_stablehlo(low.text)
    load_s = time.time() - t0
    names = low.arg_names
    bufs = [sess.buffer(inp[n]) for n in names]
    q = low.qualified
    reduce = ["mean"] * len(low.result_types) if (world > 1 and vag) else None

    # training step: the fused optimizer applies the (all-reduced) gradients to
    # the resident parameters, as train.shf's train-step does after value-and-grad
    train = args.workload == "nanogpt-train"
    pidx = [i for i, n in enumerate(names) if n not in data_names]
    if train:
        moments = [[sess.buffer(np.zeros_like(inp[names[i]])) for i in pidx] for _ in range(2)]
        tstate = [0]
        lr, b1, b2, eps, wd, clip = TRAIN_HP

    def step(buffers):
        outs = sess.call_device(q, buffers, reduce)
        if train:
            tstate[0] = sess.adamw_step([buffers[i] for i in pidx], outs[1:], moments[0], moments[1], tstate[0],
                                        lr, b1, b2, eps, wd, max_grad_norm=clip)
        return outs

    def barrier():
        sess.synchronize()
        if dist:
            dist.barrier()

    for _ in range(args.warmup):
        for o in step(bufs):
            o.release()
    barrier()
    stream = torch.cuda.ExternalStream(sess.cuda_stream, device=torch.device("cuda", local))
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    lib = library()
    n_launch0 = lib.sb_kernel_launch_count()
    with Clocks(local) as clk:
        ev0.record(stream)
        h0 = time.perf_counter()
        for _ in range(args.steps):
            for o in step(bufs):
                o.release()
        # host time to enqueue the steps: when it approaches the device time
        # per step, the step is launch-bound on the host
        host_ms = (time.perf_counter() - h0) * 1e3
        ev1.record(stream)
        ev1.synchronize()
    # kernels this library launched in the timed region (counted by every
    # launch path of the library)
    timed_launches = int(lib.sb_kernel_launch_count() - n_launch0)
    ms = ev0.elapsed_time(ev1)
    barrier()
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    value = units / (ms_step / 1e3)

    # exposed communication: the same steps without the all-reduce (every
    # rank skips it, so no rank waits on a collective); the difference in
    # device time per step is what the all-reduce adds to the step
    comm_exposed = None
    if world > 1 and vag and not args.no_profile:
        def plain_step(buffers):
            return sess.call_device(q, buffers, None)
        for _ in range(2):
            for o in plain_step(bufs):
                o.release()
        barrier()
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        for _ in range(args.steps):
            for o in plain_step(bufs):
                o.release()
        p1.record(stream)
        p1.synchronize()
        t = torch.tensor([p0.elapsed_time(p1)], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        comm_exposed = {"ms_per_step": ms_step - float(t.item()) / args.steps,
                        "compute_only_ms_per_step": float(t.item()) / args.steps}

    # end to end: per step, H2D of the step's data inputs from pinned host
    # memory, the call, and the first output (the loss; the logits of a
    # forward) read back to the host (as Sheaf's VAG dispatch does for the loss)
    e2e = None
    if not args.no_e2e:
        pinned = [torch.from_numpy(inp[n]).pin_memory().numpy() for n in data_names]
        idx = [names.index(n) for n in data_names]
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        d2h = 0
        for _ in range(args.steps):
            staged = [sess.buffer(p) for p in pinned]
            bb = list(bufs)
            for i, bx in zip(idx, staged):
                bb[i] = bx
            outs = step(bb)
            first = outs[0].to_host()
            d2h = int(np.asarray(first).nbytes)
            for o in outs:
                o.release()
            for bx in staged:
                bx.release()
        e1.record(stream)
        e1.synchronize()
        ems = e0.elapsed_time(e1)
        if dist:
            t = torch.tensor([ems], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        e2e = {"value": units / (ems / args.steps / 1e3), "unit": unit,
               "h2d_bytes_per_step": int(sum(p.nbytes for p in pinned)) * world, "d2h_bytes_per_step": d2h * world,
               "steps_per_s": 1e3 / (ems / args.steps)}
        if vag:
            e2e["loss"] = float(np.asarray(first))

    # per-kernel device time (separate pass of the same steps, CUDA events per launch)
    roof, breakdown = None, None
    if not args.no_profile:
        sess.set_profiling(True)
        for _ in range(args.steps):
            for o in step(bufs):
                o.release()
        rows = sess.profile_report()
        sess.set_profiling(False)
        dump = os.environ.get("SHEAF_B200_PROFILE_CSV")
        if dump and rank == 0:
            with open(dump, "w") as fh:
                fh.write("step,kind,kernel,calls,total_ms,elements,bytes,flops\n")
                for r in rows:
                    fh.write(f"{r['step']},{r['kind']},{r['kernel']},{r['calls']},{r['total_ms']:.6f},"
                             f"{r['elements']},{r['bytes']},{r['flops']}\n")
        calls = max(1, rows[0]["calls"]) if rows else 1
        kinds = ("gemm", "attention", "loop", "reduce", "convert", "scatter", "sort")
        tot = {k: sum(r["total_ms"] for r in rows if r["kind"] == k) / calls for k in kinds}
        allms = sum(tot.values())
        breakdown = {k: {"ms_per_step": v, "share": v / allms if allms else 0} for k, v in tot.items()}
        att = [r for r in rows if r["kind"] == "attention"]
        if att and tot["attention"] > 0:
            breakdown["attention"]["tflops"] = sum(r["flops"] for r in att) / (tot["attention"] / 1e3) / 1e12
        hbm, tc, src = peaks(burst=True)
        gem = [r for r in rows if r["kind"] == "gemm"]
        gflops = sum(r["flops"] for r in gem)  # per step (static per plan step)
        gms = tot["gemm"]
        if gem and gms > 0:
            ach = gflops / (gms / 1e3) / 1e12
            roof = {"bound": "tensor", "kernel": "gemm (all dot_general launches)", "achieved": ach, "peak": tc,
                    "unit": "TFLOP/s", "frac": ach / tc, "traffic": None, "peak_source": src,
                    "flops_per_step": gflops, "launches_per_step": len(gem), "share_of_step": gms / allms}
            # GEMMs that also compute and store gelu of their result (their
            # time is counted, their elementwise work is not in flops_per_step)
            from sheaf_b200.session import plan_steps
            fused = sum(r["epi"] for r in plan_steps(low.text, q, args.precision) if r["kind"] == "gemm")
            if fused:
                roof["fused_gelu_epilogues"] = fused
                roof["note"] = (f"{fused} of the GEMM launches also compute and store gelu of their result "
                                "(fused epilogue): their time is in the achieved figure, the gelu is not in the FLOPs")
            key = (args.workload, (cfg.get("global_batch") or 0) // world, args.precision)
            if key in GEMM_TRAFFIC:
                roof["traffic"], roof["traffic_source"] = GEMM_TRAFFIC[key]
    data = ("synthetic: seeded N(0,1) inputs, Xavier-uniform weights, one-hot labels" if args.workload == "mlp"
            else "synthetic: seeded N(0,0.02) weights, uniform tokens")
    result = {"metric": METRIC, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
              "warmup": args.warmup, "ms_per_step": ms_step, "steps_per_s": 1e3 / ms_step,
              "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32",
              "contraction": args.precision, "data": data, "config": cfg,
              "clocks": clk.summary(), "e2e": e2e, "gpu_launches": timed_launches,
              "roofline": roof, "breakdown": breakdown, "module_load_s": load_s,
              "host_enqueue_ms_per_step": host_ms / args.steps, "allreduce_exposed": comm_exposed}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            result["cpu_baseline"] = cpu_baseline(args)
        except Exception as ex:  # reported, not fatal
            result["cpu_baseline"] = {"error": str(ex)[:200]}
    if rank == 0:
        print(json.dumps(result), flush=True)
    sess.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_matmul(args):
    """Op-sweep matmul: C = A @ B, M = N = K = --size or --shape M,N,K, f32 in
    memory, as Sheaf emits `(@ a b)`; --layout picks which operands are stored
    transposed (t) and read through a transpose view, as in x @ W^T ("nt") and
    X^T @ G ("tn"); contraction per --precision."""
    import torch
    from sheaf_b200 import build
    from sheaf_b200.session import B200Session
    build.build()
    m, n, k = (int(x) for x in args.shape.split(",")) if args.shape else (args.size,) * 3
    at, bt = args.layout[0] == "t", args.layout[1] == "t"
    # bf16: the operands are bf16 tensors (Sheaf's `(cast x :bf16)`), the
    # product f32, as Sheaf emits `(@ a b)` of bf16 operands
    bf = args.precision == "bf16"
    et = "bf16" if bf else "f32"
    ty = lambda r, c, e=et: f"tensor<{r}x{c}x{e}>"
    sa, sb = (ty(k, m) if at else ty(m, k)), (ty(n, k) if bt else ty(k, n))
    body, lhs, rhs = [], "%arg0", "%arg1"
    if at:
        body.append(f"    %ta = stablehlo.transpose %arg0, dims = [1, 0] : ({sa}) -> {ty(m, k)}")
        lhs = "%ta"
    if bt:
        body.append(f"    %tb = stablehlo.transpose %arg1, dims = [1, 0] : ({sb}) -> {ty(k, n)}")
        rhs = "%tb"
    body.append(f"    %0 = stablehlo.dot_general {lhs}, {rhs}, contracting_dims = [1] x [0] : "
                f"({ty(m, k)}, {ty(k, n)}) -> {ty(m, n, 'f32')}")
    name = f"matmul_{m}_{n}_{k}_{args.layout}_{et}"
    text = (f"module @{name} {{\n func.func @f(%arg0: {sa}, %arg1: {sb}) -> {ty(m, n, 'f32')} {{\n" +
            "\n".join(body) + f"\n    return %0 : {ty(m, n, 'f32')}\n }}\n}}\n")
    sess = B200Session(precision=args.precision)
    sess.load_stablehlo(text)
    rng = np.random.default_rng(0)
    a = sess.buffer(rng.standard_normal((k, m) if at else (m, k), dtype=np.float32), bf16=bf)
    b = sess.buffer(rng.standard_normal((n, k) if bt else (k, n), dtype=np.float32), bf16=bf)
    q = f"{name}.f"
    for _ in range(args.warmup):
        for o in sess.call_device(q, [a, b]):
            o.release()
    sess.synchronize()
    stream = torch.cuda.ExternalStream(sess.cuda_stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        for o in sess.call_device(q, [a, b]):
            o.release()
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    _, tc, src = peaks(burst=True)
    tf = 2 * m * n * k / (ms / 1e3) / 1e12
    print(json.dumps({"metric": "matmul TFLOP/s", "value": tf, "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
                      "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "none",
                      "vs_baseline": None, "dtype": et, "contraction": args.precision, "data": "synthetic N(0,1)",
                      "config": {"workload": f"matmul {m}x{n}x{k} {args.layout}",
                                 "l2": "operands L2-resident below ~40 MB; no flush (op sweep, not a bench line)"},
                      "roofline": {"bound": "tensor", "achieved": tf, "peak": tc, "unit": "TFLOP/s",
                                   "frac": tf / tc, "traffic": None, "peak_source": src}}), flush=True)
    sess.close()


def run_sweep(args):
    """Op sweep: softmax / layer-norm on [65536, D] or gelu on 2^28 elements,
    forward or VJP, f32 or bf16 tensors, as Sheaf lowers them.  Algorithmic
    bytes: forward reads x and writes y (2 x elements x s), VJP reads x and the
    cotangent and writes dx (3 x elements x s), s = 4 (f32) / 2 (bf16).  L2 is
    flushed (a 256 MB write) before every timed call; only the call is inside
    the CUDA events."""
    import torch
    from sheaf_b200 import build
    from sheaf_b200.session import B200Session, library
    from sheaf_lowering import models as M
    build.build()
    shape = (1 << 28,) if args.op == "gelu" else (65536, args.dim)
    low = M.sweep_program(args.op, shape, args.vjp, args.dtype)
    inp = M.sweep_inputs(args.op, shape, args.vjp)
    sess = B200Session(precision="fp32")
    sess.load_stablehlo(low.text)
    bf = args.dtype == "bf16"
    bufs = [sess.buffer(inp[n], bf16=bf) for n in low.arg_names]
    q = low.qualified
    stream = torch.cuda.ExternalStream(sess.cuda_stream)
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    for _ in range(args.warmup):
        for o in sess.call_device(q, bufs):
            o.release()
    sess.synchronize()
    lib = library()
    n0 = lib.sb_kernel_launch_count()
    total = 0.0
    with Clocks(0) as clk:
        for _ in range(args.steps):
            with torch.cuda.stream(stream):
                flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            outs = sess.call_device(q, bufs)
            e1.record(stream)
            e1.synchronize()
            total += e0.elapsed_time(e1)
            for o in outs:
                o.release()
    launches = int(lib.sb_kernel_launch_count() - n0)
    ms = total / args.steps
    elems = int(np.prod(shape))
    nbytes = (3 if args.vjp else 2) * elems * (2 if bf else 4)
    gbs = nbytes / (ms / 1e3) / 1e9
    hbm, _, src = peaks()
    what = f"{args.op} {'VJP' if args.vjp else 'forward'} {'x'.join(map(str, shape))} {args.dtype}"
    print(json.dumps({"metric": "op sweep HBM GB/s", "value": gbs, "unit": "GB/s", "n_gpus": 1,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                      "scaling": "none", "vs_baseline": None, "dtype": args.dtype, "data": "synthetic N(0,1)",
                      "config": {"workload": f"op sweep: {what}", "l2": "flushed (256 MB write) before each call"},
                      "clocks": clk.summary(), "gpu_launches": launches,
                      "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                                   "traffic": None, "peak_source": src, "algorithmic_bytes": nbytes}}), flush=True)
    sess.close()


def run_decode(args):
    """Decoding with the key/value cache: nanoGPT (6 layers, d384, T 256), one
    new token per step (forward of one position against the cached keys and
    values, top-k 200 sampling at temperature 0.8); the sampled id and the
    updated caches feed the next step on the device.  W warm-up steps feed the
    start of a random prompt; the K timed steps continue the sequence.  e2e
    adds the read-back of each step's token id to the host."""
    import torch
    from sheaf_b200 import build
    from sheaf_b200.session import B200Session, library
    from sheaf_lowering import generate as G
    from sheaf_lowering import models as M
    from sheaf_lowering import random as RG
    build.build()
    c = M.NANOGPT
    if args.warmup + args.steps > c.T:
        raise SystemExit(f"--warmup + --steps must be <= {c.T} positions")
    low = G.gpt_decode_program(c, 200, 0.8)
    inp = M.gpt_inputs(c, batch=1, seed=0)
    sess = B200Session(precision=args.precision)
    t0 = time.time()
    sess.load_stablehlo(low.text)
    load_s = time.time() - t0
    params = [sess.buffer(inp[n]) for n, _ in M.gpt_param_leaves(c)]
    caches = [sess.buffer(np.zeros(sh, np.float32)) for _, sh in G.cache_leaves(c)]
    key = sess.buffer(RG.key_of_seed(1337))
    q = low.qualified
    pos_bufs = [sess.buffer(np.float32([p])) for p in range(args.warmup + args.steps)]
    tok = sess.buffer(np.float32([[inp["idx"][0, 0]]]))
    # a [] -> [1, 1] reshape of the sampled id, as the sampling loop does
    rs = ("module @tok_reshape {\n func.func @f(%arg0: tensor<f32>) -> tensor<1x1xf32> {\n"
          "    %0 = stablehlo.reshape %arg0 : (tensor<f32>) -> tensor<1x1xf32>\n"
          "    return %0 : tensor<1x1xf32>\n }\n}\n")
    sess.load_stablehlo(rs)

    def advance(p, tok, caches, key, read_back=False):
        """One step; releases the step's inputs that earlier steps produced."""
        outs = sess.call_device(q, params + caches + [tok, pos_bufs[p], key])
        nt = sess.call_device("tok_reshape.f", [outs[0]])[0]
        if read_back:
            float(outs[0].to_host())
        outs[0].release()
        for b in [tok, key] + caches:
            b.release()
        return nt, outs[2:], outs[1]

    for p in range(args.warmup):
        tok, caches, key = advance(p, tok, caches, key)
    sess.synchronize()
    stream = torch.cuda.ExternalStream(sess.cuda_stream)
    lib = library()
    n0 = lib.sb_kernel_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(0) as clk:
        e0.record(stream)
        for p in range(args.warmup, args.warmup + args.steps):
            tok, caches, key = advance(p, tok, caches, key)
        e1.record(stream)
        e1.synchronize()
    launches = int(lib.sb_kernel_launch_count() - n0)
    ms = e0.elapsed_time(e1) / args.steps
    # end to end: the same positions again, each sampled id read back to the host
    h0 = time.perf_counter()
    for p in range(args.warmup, args.warmup + args.steps):
        tok, caches, key = advance(p, tok, caches, key, read_back=True)
    ems = (time.perf_counter() - h0) * 1e3 / args.steps
    dump = os.environ.get("SHEAF_B200_PROFILE_CSV")
    if dump:
        # per-kernel device time of the decode step (the last position again,
        # CUDA events around each launch), for the profile summary
        sess.set_profiling(True)
        for _ in range(4):
            tok, caches, key = advance(args.warmup + args.steps - 1, tok, caches, key)
        rows = sess.profile_report()
        sess.set_profiling(False)
        with open(dump, "w") as fh:
            fh.write("function,step,kind,kernel,calls,total_ms,elements,bytes,flops\n")
            for r in rows:
                fh.write(f"{r['function']},{r['step']},{r['kind']},{r['kernel']},{r['calls']},{r['total_ms']:.6f},"
                         f"{r['elements']},{r['bytes']},{r['flops']}\n")
    print(json.dumps({"metric": "KV-cache decode tokens/s", "value": 1e3 / ms, "unit": "tokens/s", "n_gpus": 1,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                      "scaling": "none", "vs_baseline": None, "dtype": "f32", "contraction": args.precision,
                      "data": "synthetic: seeded N(0,0.02) weights, random prompt",
                      "config": {"workload": f"nanogpt decode with key/value cache (top-k 200, temperature 0.8), "
                                             f"positions {args.warmup}..{args.warmup + args.steps - 1} of {c.T}",
                                 "model": f"L{c.n_layer} D{c.n_embd} H{c.n_head} T{c.T} V{c.vocab_size}",
                                 "l2": "weights and caches (48 MB) fit in L2: latency-bound by design"},
                      "clocks": clk.summary(), "gpu_launches": launches,
                      "e2e": {"value": 1e3 / ems, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                              "d2h_bytes_per_step": 4, "note": "host wall clock per step incl. the id read-back"},
                      "module_load_s": load_s}), flush=True)
    sess.close()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "matmul":
        run_matmul(args)
    elif args.workload == "sweep":
        run_sweep(args)
    elif args.workload == "nanogpt-decode":
        run_decode(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
