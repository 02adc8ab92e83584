"""The full decode step on the GPU against the reference (golden vectors from
the reference engine, the reference built from its sources, or the C
restatement of its step). Mirrors tests/native.cpp:206-241 of the reference."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from conftest import dcb, oracle, synthetic
from gpu_util import Checker, has_avx512, host_threads, with_max_positions

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
REF = np.load(GOLDEN / "reference_outputs.npz")
TOKENS = json.loads((GOLDEN / "reference_outputs.json").read_text())["tokens"]
# Logit tolerance of the north-star parity bar (FP32 KV).
LOGIT_ATOL = 1e-3


@pytest.mark.parametrize("name,atol", [("tiny", 1e-5), ("small", 1e-4), ("odd", 1e-4)])
@pytest.mark.parametrize("rope", ["cached", "direct"])
def test_step_matches_reference_goldens(name, atol, rope, tiny_int8, small_int8, odd_int8):
    model = {"tiny": tiny_int8, "small": small_int8, "odd": odd_int8}[name]
    eng = dcb.Engine(model, 16, cached_rope=(rope == "cached"))
    got = []
    for t in TOKENS:
        logits, best = eng.step(t)
        assert best == int(np.argmax(logits))
        got.append(logits.copy())
    got = np.stack(got)
    np.testing.assert_allclose(got, REF[f"{name}_simd512x4_{rope}"], atol=atol, rtol=0)
    np.testing.assert_allclose(got, REF[f"{name}_scalar_{rope}"], atol=atol, rtol=0)


def test_rewind_reset_and_errors(tiny_int8):
    # tests/native.cpp:219-227, 240-241
    eng = dcb.Engine(tiny_int8, 8)
    for t in (1, 4, 2):
        eng.step(t)
    eng.rewind(2)
    replay = oracle.Oracle(tiny_int8, 8)
    for t in (1, 4):
        replay.step(t)
    expected = replay.step(5).copy()
    got, _ = eng.step(5)
    np.testing.assert_allclose(got, expected, atol=1e-5)
    with pytest.raises(ValueError, match="token ID outside vocabulary"):
        eng.step(11)
    with pytest.raises(RuntimeError, match="cannot rewind forward"):
        eng.rewind(4)
    eng.reset()
    fresh = oracle.Oracle(tiny_int8, 8)
    got, _ = eng.step(2)
    np.testing.assert_allclose(got, fresh.step(2), atol=1e-5)
    before = got.copy()
    logits, best = eng.step(1, head=False)
    assert logits is None and best is None and eng.position == 2
    np.testing.assert_array_equal(eng.logits, before)  # a head-less step leaves logits alone
    short = dcb.Engine(tiny_int8, 1)
    short.step(1, head=False)
    with pytest.raises(RuntimeError, match="context capacity exceeded"):
        short.step(1)


def test_f16_kv_matches_f16_oracle(small_int8):
    eng = dcb.Engine(small_int8, 32, kv_dtype="f16")
    orc = oracle.Oracle(small_int8, 32, kv_f16=True)
    for t in [3, 999, 0, 512, 77, 78, 79, 80, 81]:
        got, _ = eng.step(t)
        np.testing.assert_allclose(got, orc.step(t), atol=1e-4)
    k, v = eng.kv_read(1, 0, 9)
    ko, vo = orc.kv_view()
    np.testing.assert_allclose(k, ko[1, :9], atol=2e-3, rtol=1e-3)
    np.testing.assert_allclose(v, vo[1, :9], atol=2e-3, rtol=1e-3)


def test_odd_shapes_many_positions(odd_int8):
    # rows that are not multiples of 16 bytes, several KV splits (positions > 64)
    eng = dcb.Engine(odd_int8, 128)
    orc = oracle.Oracle(odd_int8, 128)
    rng = np.random.default_rng(1)
    for i, t in enumerate(rng.integers(0, 333, size=100)):
        head = i % 9 == 0 or i > 90
        got, _ = eng.step(int(t), head=head)
        exp = orc.step(int(t), head=head)
        if head:
            np.testing.assert_allclose(got, exp, atol=1e-4)


def _greedy(engine_step, prompt, steps):
    """src/main.cpp:115-127: prefill with the head on the last prompt token,
    then steps greedy tokens; returns (tokens, per-step logits)."""
    logits = None
    for i, t in enumerate(prompt):
        logits = engine_step(t, i + 1 == len(prompt))
    out, seen = [], []
    nxt = int(np.argmax(logits))
    for i in range(steps):
        out.append(nxt)
        seen.append(logits.copy())
        if i + 1 < steps:
            logits = engine_step(nxt, True)
            nxt = int(np.argmax(logits))
    return out, seen


def test_qwen05_greedy_64_steps_match_reference(qwen05_int8):
    """Config 0: 128-token random prompt, 64 greedy steps, FP32 KV."""
    prompt = synthetic.random_tokens(128, synthetic.QWEN05.vocab, seed=11)
    eng = dcb.Engine(qwen05_int8, 128 + 64)
    chk = Checker(qwen05_int8, 128 + 64)

    def gpu_step(t, head):
        logits, best = eng.step(t, head)
        if head:
            assert best == int(np.argmax(logits))  # device argmax is bit-exact first-index
        return logits

    got_tokens, got_logits = _greedy(gpu_step, prompt, 64)
    ref_tokens, ref_logits = _greedy(chk.step, prompt, 64)
    diffs = [float(np.abs(a - b).max()) for a, b in zip(got_logits, ref_logits)]
    assert max(diffs) < LOGIT_ATOL, (chk.kind, max(diffs))
    assert got_tokens == ref_tokens, chk.kind


def test_device_chained_greedy_matches_host_loop(small_int8):
    import torch
    prompt = [5, 9, 300, 2]
    eng = dcb.Engine(small_int8, 64)
    host_tokens, _ = _greedy(lambda t, h: eng.step(t, h)[0], prompt, 20)
    eng.reset()
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    for i, t in enumerate(prompt):
        eng.step_async(t, head=(i + 1 == len(prompt)), argmax_dev=tok.data_ptr())
    dev_tokens = []
    for i in range(20):
        eng.synchronize()
        dev_tokens.append(int(tok.item()))
        if i + 1 < 20:
            eng.step_async(token_dev=tok.data_ptr(), head=True, argmax_dev=tok.data_ptr())
    assert dev_tokens == host_tokens


@pytest.mark.parametrize("kv", ["f32", "f16"])
@pytest.mark.parametrize("ctx,steps", [(4096, 16), (32768, 3)])
def test_long_context_prefilled_kv(qwen05_int8, tmp_path, kv, ctx, steps):
    """Config 3 at 4096 and 32768 positions: KV pre-filled with seeded N(0,1)
    keys/values. The reference Engine cannot hold 32768 + steps positions
    (src/model.cpp:190-191), so the checker is the C restatement of its step
    over a caller-owned KV buffer."""
    model = with_max_positions(qwen05_int8, tmp_path / "long", 40960)
    d = synthetic.QWEN05
    eng = dcb.Engine(model, ctx + steps, kv_dtype=kv)
    orc = oracle.Oracle(model, ctx + steps, kv_f16=(kv == "f16"), threads=8)
    kc, vc = orc.kv_view()
    rng = np.random.default_rng(2024)
    for l in range(d.layers):
        k = rng.standard_normal((ctx, d.kv_dim), dtype=np.float32)
        v = rng.standard_normal((ctx, d.kv_dim), dtype=np.float32)
        if kv == "f16":
            k, v = oracle.f16_round(k), oracle.f16_round(v)
        kc[l, :ctx] = k
        vc[l, :ctx] = v
        eng.kv_write(l, 0, k, v)
    eng.set_position(ctx)
    orc.pos = ctx
    tok = 1234
    for _ in range(steps):
        got, best = eng.step(tok)
        exp = orc.step(tok)
        np.testing.assert_allclose(got, exp, atol=LOGIT_ATOL)
        assert best == oracle.argmax(exp)
        tok = best


@pytest.mark.parametrize("which,ctx", [("g64", 1000), ("g64", 1100), ("g64", 2300), ("g64b", 1500)])
def test_group_attention_units_match_oracle(which, ctx, g64_int8, g64b_int8):
    """head_dim 64 with 7 (g64) and 2 (g64b) query heads per KV head, KV
    pre-filled with seeded N(0,1) rows: below 1024 attended positions the
    step uses one block per (query head, split), from 1024 on one block per
    (KV group, split); partial last chunks and split counts that do not divide
    the context are included."""
    from conftest import G64, G64B
    model, d = (g64_int8, G64) if which == "g64" else (g64b_int8, G64B)
    steps = 3
    eng = dcb.Engine(model, ctx + steps)
    orc = oracle.Oracle(model, ctx + steps, threads=8)
    kc, vc = orc.kv_view()
    rng = np.random.default_rng(ctx)
    for l in range(d.layers):
        k = rng.standard_normal((ctx, d.kv_dim), dtype=np.float32)
        v = rng.standard_normal((ctx, d.kv_dim), dtype=np.float32)
        kc[l, :ctx] = k
        vc[l, :ctx] = v
        eng.kv_write(l, 0, k, v)
    eng.set_position(ctx)
    orc.pos = ctx
    tok = 5
    for _ in range(steps):
        got, best = eng.step(tok)
        exp = orc.step(tok)
        np.testing.assert_allclose(got, exp, atol=LOGIT_ATOL)
        assert best == oracle.argmax(exp)
        tok = best


# Channels whose residual grows large, and gate/up rows with large outputs.
OUTLIER_CHANNELS = (3, 250, 777)
OUTLIER_GU_ROWS = (10, 2000, 4000)


def outlier_values(seed: int):
    """The seeded random model with activation outliers: the W_down rows of
    OUTLIER_CHANNELS scaled by 300, so those residual channels grow to the
    order of 1e2-1e3 over the layers while the others stay near 1, and the
    W_gate/W_up rows of OUTLIER_GU_ROWS scaled by 30 (SiLU(gate)*up inputs in
    the tens to hundreds). Per-row quantisation keeps every scaled row exact."""
    base = synthetic.random_values(seed)

    def values(name, shape):
        w = base(name, shape)
        if name.endswith("mlp.down_proj.weight"):
            w = w.copy()
            w[list(OUTLIER_CHANNELS)] *= np.float32(300.0)
        elif name.endswith(("mlp.gate_proj.weight", "mlp.up_proj.weight")):
            w = w.copy()
            w[list(OUTLIER_GU_ROWS)] *= np.float32(30.0)
        return w
    return values


def test_outlier_activations_greedy_64_steps(tmp_path_factory):
    """GEMV inputs are staged as 24-bit fixed point scaled to their largest
    element, and the O/down outputs are summed in 2^-26 fixed point; a model
    with a few residual channels orders of magnitude above the rest checks
    both over 64 greedy steps.

    This model amplifies FP32 rounding: the reference's own scalar and
    simd512x4 kernels, which differ only in summation order, already differ by
    about 1e-3 in the logits. Each engine is therefore measured against the
    float64 evaluation of the same step (oracle.exact64), along the shared
    greedy path: the B200 logits may be no further from it than the larger of
    1e-3 and the reference kernels' own distance (the C restatement, which
    follows the scalar kernel, always; the reference's scalar and SIMD kernels
    when they are built), and every greedy stream is identical."""
    from oracle.exact64 import Exact64
    d = synthetic.QWEN05
    model = synthetic.write_int8_model(tmp_path_factory.mktemp("outlier") / "m", d, outlier_values(7))
    prompt = synthetic.random_tokens(32, d.vocab, seed=13)
    steps, cap = 64, 32 + 64
    threads = host_threads()
    eng = dcb.Engine(model, cap)
    got_tokens, got_logits = _greedy(lambda t, h: eng.step(t, h)[0], prompt, steps)
    fp32 = {"oracle": _greedy(oracle.Oracle(model, cap, threads=threads).step, prompt, steps)}
    if oracle.ref_available():
        for k in ("scalar", "simd512x4" if has_avx512() else "simd256"):
            fp32["ref_" + k] = _greedy(oracle.RefEngine(model, cap, k, threads, True).step, prompt, steps)
    exact = Exact64(model, cap)
    exact_logits = [None]
    for i, t in enumerate(prompt):
        exact_logits[0] = exact.step(t, i + 1 == len(prompt))
    exact_logits += [exact.step(t, True) for t in got_tokens[:-1]]

    def dist(a):
        return max(float(np.abs(x - y).max()) for x, y in zip(a, exact_logits))
    errors = {k: dist(lg) for k, (_, lg) in fp32.items()}
    for k, (toks, _) in fp32.items():
        assert toks == got_tokens, k
    assert [int(np.argmax(x)) for x in exact_logits] == got_tokens
    gpu = dist(got_logits)
    assert gpu <= max(LOGIT_ATOL, max(errors.values())), (gpu, errors)
