"""Two-GPU data parallel: NCCL mean of the sharded value-and-grad equals the
single-GPU full-batch result (fp32, 1e-5 max-relative).  Needs 2 GPUs."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode,port", [("after", 29617), ("overlap", 29619)])
def test_two_gpu_allreduce_matches_full_batch(tmp_path, mode, port):
    """after: one grouped all-reduce after the backward; overlap: 64 KB buckets
    all-reduced on a second stream while the backward continues."""
    out = tmp_path / "dp.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", SHEAF_B200_ALLREDUCE_BUCKET_BYTES="65536")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(HERE, "dp_worker.py"), str(out), mode]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["max_rel"] <= 1e-5, res
