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


def test_gelu_is_fused_into_the_mlp_gemm_epilogue():
    """nanoGPT value-and-grad and forward: each layer's c_fc GEMM writes both
    its result and gelu of it (the gelu loop and its launch are gone); the
    fp32 mode (CUDA-core GEMMs) keeps the loop."""
    c = M.NANOGPT
    for low in (M.gpt_vag(c, batch=2), M.gpt_fwd(c, batch=2)):
        rows = S.plan_steps(low.text, low.qualified, "tf32")
        fused = [r for r in rows if r["kind"] == "gemm" and r["epi"] == 1]
        assert len(fused) == c.n_layer
        # the c_fc product: [B*T, D] x [D, 4D]
        assert all(r["N"] == 4 * c.n_embd and r["K"] == c.n_embd for r in fused)
    rows = S.plan_steps(M.gpt_vag(c, batch=2).text, M.gpt_vag(c, batch=2).qualified, "fp32")
    assert not [r for r in rows if r["epi"]]


def test_gelu_matcher_rejects_other_functions():
    """An erf-style or otherwise different activation after a GEMM is not
    fused (the numeric check of the element-wise cone fails)."""
    text = """module @notgelu {
 func.func @f(%arg0: tensor<256x128xf32>, %arg1: tensor<128x512xf32>) -> tensor<256x512xf32> {
    %0 = stablehlo.dot_general %arg0, %arg1, contracting_dims = [1] x [0] : (tensor<256x128xf32>, tensor<128x512xf32>) -> tensor<256x512xf32>
    %c = stablehlo.constant dense<0.7978846> : tensor<f32>
    %1 = stablehlo.broadcast_in_dim %c, dims = [] : (tensor<f32>) -> tensor<256x512xf32>
    %2 = stablehlo.multiply %0, %1 : tensor<256x512xf32>
    %3 = stablehlo.tanh %2 : tensor<256x512xf32>
    %4 = stablehlo.multiply %0, %3 : tensor<256x512xf32>
    return %4 : tensor<256x512xf32>
 }
}
"""
    rows = S.plan_steps(text, "notgelu.f", "tf32")
    assert not [r for r in rows if r["epi"]]


def test_operand_shadows_written_by_their_producers():
    """TF32: the residual-stream gradients that GEMMs and other steps both
    read get TF32-rounded copies written by the row-group kernels that
    produce them, so the plan has no separate conversion steps; bf16 mode
    still converts the parameters (and values produced outside row groups).
    Batch 8: 2048 rows (row groups start at 1024 rows)."""
    low = M.gpt_vag(M.NANOGPT, batch=8)
    assert int(_summary(low.text, "tf32").get("convert", "0")) == 0
    n_bf16 = int(_summary(low.text, "bf16").get("convert", "0"))
    assert 0 < n_bf16 < 75


def test_bf16_softmax_is_one_row_group():
    """A softmax over bf16 rows plans as one kernel, as the f32 one does."""
    for dt in ("f32", "bf16"):
        low = M.sweep_program("softmax", (4096, 768), False, dt)
        s = _summary(low.text, "tf32")
        assert s["loop"] == "1" and s["reduce"] == "0", (dt, s)


def test_layer_norm_weight_gradient_sums_are_finished_in_one_batch():
    """The 13 column sums of the nanoGPT step (LayerNorm weight gradients,
    outputs no later step reads) are marked for the runtime's batched finish."""
    low = M.gpt_vag(M.NANOGPT, batch=8)
    rows = S.plan_steps(low.text, low.qualified, "tf32")
    assert sum(r["deferred_sums"] for r in rows) == 2 * M.NANOGPT.n_layer + 1


def test_second_gemm_may_take_first_gemms_operand_memory():
    """A value's arena memory is free after its last reader, so a GEMM's result
    may be placed where the previous GEMM's operand was (here dX = G @ W takes
    the memory of X*X, read last by dW = G^T @ (X*X)).  That is why the runtime
    launches two GEMM steps together only when neither writes memory that the
    other reads (they run at the same time)."""
    T, I, O = 2048, 384, 1152
    g, w, x = f"tensor<{T}x{O}xf32>", f"tensor<{O}x{I}xf32>", f"tensor<{T}x{I}xf32>"
    dw, gt = f"tensor<{O}x{I}xf32>", f"tensor<{O}x{T}xf32>"
    text = (f"module @reuse {{\n func.func @f(%arg0: {g}, %arg1: {w}, %arg2: {x}) -> ({dw}, {x}) {{\n"
            f"    %t = stablehlo.multiply %arg2, %arg2 : {x}\n"
            f"    %gt = stablehlo.transpose %arg0, dims = [1, 0] : ({g}) -> {gt}\n"
            f"    %dw = stablehlo.dot_general %gt, %t, contracting_dims = [1] x [0] : ({gt}, {x}) -> {dw}\n"
            f"    %dx = stablehlo.dot_general %arg0, %arg1, contracting_dims = [1] x [0] : ({g}, {w}) -> {x}\n"
            f"    %y = stablehlo.add %dx, %dx : {x}\n"
            f"    return %dw, %y : {dw}, {x}\n }}\n}}\n")
    rows = S.plan_steps(text, "reuse.f", "tf32")
    assert [r["kind"] for r in rows] == ["loop", "gemm", "gemm", "loop"]
    assert rows[1]["root_offset"] == -1  # dW is returned: a buffer of its own
    assert rows[2]["root_offset"] == rows[0]["root_offset"] >= 0
