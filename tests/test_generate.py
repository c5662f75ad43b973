"""The generation path: `stablehlo.sort` (top_k) and `generate-token`
(examples/nanoGPT/model.shf:116-125) as device programs, against the oracle."""
import numpy as np
import pytest

from oracle.stablehlo_ref import run
from sheaf_lowering import generate as G
from sheaf_lowering import models as M
from sheaf_lowering import random as RG


def sort_module(rows, n, k, direction="GT"):
    t, ti = f"tensor<{rows}x{n}xf32>", f"tensor<{rows}x{n}xi32>"
    return f"""module @srt_{rows}_{n}_{k}_{direction} {{
 func.func @f(%arg0: {t}) -> (tensor<{rows}x{k}xf32>, tensor<{rows}x{k}xf32>) {{
    %0 = stablehlo.iota dim = 1 : {ti}
    %1, %2 = "stablehlo.sort"(%arg0, %0) ({{
    ^bb0(%3: tensor<f32>, %4: tensor<f32>, %5: tensor<i32>, %6: tensor<i32>):
      %7 = "stablehlo.compare"(%3, %4) {{comparison_direction = #stablehlo<comparison_direction {direction}>}} : (tensor<f32>, tensor<f32>) -> tensor<i1>
      "stablehlo.return"(%7) : (tensor<i1>) -> ()
    }}) {{dimension = 1 : i64, is_stable = true}} : ({t}, {ti}) -> ({t}, {ti})
    %8 = stablehlo.slice %1 [0:{rows}:1, 0:{k}:1] : ({t}) -> tensor<{rows}x{k}xf32>
    %9 = stablehlo.slice %2 [0:{rows}:1, 0:{k}:1] : ({ti}) -> tensor<{rows}x{k}xi32>
    %10 = stablehlo.convert %9 : (tensor<{rows}x{k}xi32>) -> tensor<{rows}x{k}xf32>
    return %8, %10 : tensor<{rows}x{k}xf32>, tensor<{rows}x{k}xf32>
 }}
}}
"""


def test_oracle_sort_is_stable_descending():
    x = np.float32([[3, 1, 3, 2, 3]])
    v, i = run(sort_module(1, 5, 5), "srt_1_5_5_GT.f", [x], dtype=np.float32)
    assert v.tolist() == [[3, 3, 3, 2, 1]] and i.tolist() == [[0, 2, 4, 3, 1]]


def test_generate_program_plans(lib):
    from sheaf_b200.session import inspect_module
    c = M.GPTConfig(2, 2, 64, 64, 65, 1, 64)
    assert "sort=1" in inspect_module(G.gpt_generate_program(c).text, "fp32")


@pytest.mark.gpu
@pytest.mark.parametrize("rows,n,k,d", [(1, 65, 65, "GT"), (3, 1000, 200, "GT"), (2, 777, 777, "LT"),
                                        (1, 50304, 200, "GT")])
def test_device_sort_topk(fp32_session, rows, n, k, d):
    rng = np.random.default_rng(n)
    x = rng.standard_normal((rows, n)).astype(np.float32)
    x[:, ::7] = x[:, 1:2]  # ties: stability decides the payload order
    text = sort_module(rows, n, k, d)
    name = f"srt_{rows}_{n}_{k}_{d}.f"
    fp32_session.load_stablehlo(text)
    got = fp32_session.call(name, [x])
    ref = run(text, name, [x], dtype=np.float32)
    for g, r in zip(got, ref):
        assert np.array_equal(g, r)


@pytest.mark.gpu
def test_device_generate_tokens(fp32_session):
    c = M.GPTConfig(2, 2, 64, 64, 65, 1, 64)
    low = G.gpt_generate_program(c, 200, 0.8)
    inp = M.gpt_inputs(c, batch=1, seed=5)
    params = [inp[n] for n in low.arg_names[:-2]]
    ids = inp["idx"].copy()
    key = RG.key_of_seed(2024)
    fp32_session.load_stablehlo(low.text)
    for _ in range(4):
        nid, nkey = fp32_session.call(low.qualified, params + [ids, key])
        rid, rkey = run(low.text, low.qualified, params + [ids, key], dtype=np.float32)
        assert float(nid) == float(rid) and np.array_equal(nkey.view(np.int32), rkey.view(np.int32))
        assert 0 <= float(nid) < c.vocab_size
        # slide-window (sample.shf: append-and-roll)
        ids = np.concatenate([ids[:, 1:], np.float32([[nid]])], axis=1)
        key = nkey


def test_decode_program_plans(lib):
    from sheaf_b200.session import inspect_module
    c = M.GPTConfig(2, 2, 64, 64, 65, 1, 64)
    assert "sort=1" in inspect_module(G.gpt_decode_program(c).text, "fp32")


@pytest.mark.gpu
def test_kv_cache_logits_equal_full_forward(fp32_session):
    """Decoding with the key/value cache: the logits at position p (prompt fed
    one token per call) equal the full forward's last-position logits on the
    prefix 0..p (the oracle), within the fp32 tolerance."""
    c = M.GPTConfig(2, 2, 64, 64, 65, 1, 64)
    dec = G.gpt_decode_forward_program(c)
    inp = M.gpt_inputs(c, batch=1, seed=5)
    params = [inp[n] for n, _ in M.gpt_param_leaves(c)]
    caches = [np.zeros(s, np.float32) for _, s in G.cache_leaves(c)]
    toks = inp["idx"][0, :5]
    fp32_session.load_stablehlo(dec.text)
    for p, tk in enumerate(toks):
        outs = fp32_session.call(dec.qualified, params + caches + [np.float32([[tk]]), np.float32([p])])
        logits, caches = outs[0], outs[1:]
        f = M.gpt_fwd(M.GPTConfig(2, 2, 64, 64, 65, 1, p + 1), batch=1)
        fi = {**inp, "idx": toks[None, :p + 1].astype(np.float32)}
        ref = run(f.text, f.qualified, [fi[n] for n in f.arg_names])[0][0, -1]
        assert np.max(np.abs(logits[0, 0] - ref)) <= 1e-5 * np.max(np.abs(ref))


@pytest.mark.gpu
def test_device_decode_tokens(fp32_session):
    """A 4-token prompt fed through the cache, then 4 sampled tokens: every
    call's next id, key and caches are those of the oracle run of the same
    program."""
    c = M.GPTConfig(2, 2, 64, 64, 65, 1, 64)
    low = G.gpt_decode_program(c, 200, 0.8)
    inp = M.gpt_inputs(c, batch=1, seed=6)
    params = [inp[n] for n, _ in M.gpt_param_leaves(c)]
    caches = [np.zeros(s, np.float32) for _, s in G.cache_leaves(c)]
    rcaches = list(caches)
    key = RG.key_of_seed(99)
    fp32_session.load_stablehlo(low.text)
    tok = float(inp["idx"][0, 0])
    for p in range(8):
        if p < 4:
            tok = float(inp["idx"][0, p])
        args = [np.float32([[tok]]), np.float32([p]), key]
        outs = fp32_session.call(low.qualified, params + caches + args)
        ref = run(low.text, low.qualified, params + rcaches + args, dtype=np.float32)
        assert float(outs[0]) == float(ref[0])
        assert np.array_equal(outs[1].view(np.int32), ref[1].view(np.int32))
        for a, b in zip(outs[2:], ref[2:]):
            np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-6)
        caches, rcaches, key = outs[2:], ref[2:], outs[1]
        tok = float(outs[0])
