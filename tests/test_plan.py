"""Execution plans built on the host (no GPU): what the planner's rewrites do
to the benchmark graphs."""
from sheaf_b200 import session as S
from sheaf_lowering import models as M


def _summary(text, prec="tf32"):
    line = S.inspect_module(text, prec).splitlines()[0]
    return dict(kv.split("=") for kv in line.split(": ", 1)[1].split() if "=" in kv)


def test_embedding_gradient_is_a_scatter_add():
    """GPT value-and-grad with GPT-2's vocabulary (50304): the table gradient
    is a scatter-add, not a [V, N] x [N, D] product, and the GEMM FLOPs of the step are the
    algorithmic ones, 3 passes x 2 N (12 L D^2 + V D)."""
    c = M.GPTConfig(n_layer=2, n_head=2, n_embd=128, block_size=128, vocab_size=50304, batch=2)
    low = M.gpt_vag(c)
    s = _summary(low.text)
    assert s["scatter"] == "1" and s["attention"] == "4"
    n = c.batch * c.block_size
    # one [V, N] x [N, D] product remains: lm_head's weight gradient
    big = [r for r in S.plan_steps(low.text, low.qualified, "tf32")
           if r["kind"] == "gemm" and r["M"] == c.vocab_size and r["K"] == n]
    assert len(big) == 1
    L, D, V = c.n_layer, c.n_embd, c.vocab_size
    assert float(s["gemm_flops"]) == 3 * 2 * n * (12 * L * D * D + V * D)


def test_bf16_plan_converts_gemm_operands():
    low = M.gpt_vag(M.NANOGPT, batch=2)
    s = _summary(low.text, "bf16")
    assert int(s["convert"]) > 0 and s["attention"] == "12"
