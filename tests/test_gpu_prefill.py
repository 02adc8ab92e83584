"""Batched prefill (dcb_prefill) against the reference's token-by-token prompt
loop (src/main.cpp:134-137: Engine::step per prompt token, the LM head on the
last only), restated by the oracle over its own KV cache: the K/V rows every
prompt position leaves in the cache, the last token's logits and argmax, the
engine's position, and the greedy continuation from there."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import dcb, oracle, synthetic
from gpu_util import host_threads

pytestmark = pytest.mark.gpu

LOGIT_ATOL = 1e-3
KV_ATOL = {"f32": 1e-4, "f16": 2e-3}


def _oracle_after(model, cap, prompt, kv: str, pre=()):
    orc = oracle.Oracle(model, cap, kv_f16=(kv == "f16"), threads=host_threads())
    for t in pre:
        orc.step(t, False)
    logits = None
    for i, t in enumerate(prompt):
        logits = orc.step(t, i + 1 == len(prompt))
    return orc, logits.copy()


def _check_prefill(model, n, kv="f32", pre=(), follow=8, seed=1):
    d, _ = synthetic.load_model(model)
    prompt = synthetic.random_tokens(n, d.vocab, seed=seed)
    cap = len(pre) + n + follow + 4
    eng = dcb.Engine(model, cap, kv_dtype=kv)
    for t in pre:
        eng.step(t, head=False)
    logits, best = eng.prefill(prompt)
    orc, exp = _oracle_after(model, cap, prompt, kv, pre)
    assert eng.position == len(pre) + n
    np.testing.assert_allclose(logits, exp, atol=LOGIT_ATOL)
    assert best == oracle.argmax(exp)
    kc, vc = orc.kv_view()
    p1 = len(pre) + n
    for layer in range(d.layers):
        k, v = eng.kv_read(layer, 0, p1)
        np.testing.assert_allclose(k, kc[layer, :p1], atol=KV_ATOL[kv], rtol=1e-4)
        np.testing.assert_allclose(v, vc[layer, :p1], atol=KV_ATOL[kv], rtol=1e-4)
    # The engine decodes on from the prefilled cache as the oracle does.
    tok = best
    for _ in range(follow):
        got, gbest = eng.step(tok)
        want = orc.step(tok)
        np.testing.assert_allclose(got, want, atol=LOGIT_ATOL)
        assert gbest == oracle.argmax(want)
        tok = gbest


@pytest.mark.parametrize("n", [1, 17, 64, 65, 130])
def test_prefill_small_model(small_int8, n):
    # one slot, a partial chunk, one full chunk, a chunk and one, three chunks
    _check_prefill(small_int8, n, seed=n)


@pytest.mark.parametrize("kv", ["f32", "f16"])
def test_prefill_after_steps_head_dim_64(g64_int8, kv):
    # head_dim 64 (the tensor-core attention path), a prompt entering an
    # engine that already holds 40 positions
    d, _ = synthetic.load_model(g64_int8)
    _check_prefill(g64_int8, 90, kv=kv, pre=synthetic.random_tokens(40, d.vocab, seed=4), seed=5)


def test_prefill_qwen_shape_128(qwen05_int8):
    # the bench's prompt length on the Qwen2.5-0.5B shape
    _check_prefill(qwen05_int8, 128, follow=4, seed=7)


def test_prefill_errors(small_int8):
    d, _ = synthetic.load_model(small_int8)
    eng = dcb.Engine(small_int8, 8)
    # the messages and exception types of dcb_step (src/model.cpp:259-260)
    with pytest.raises(RuntimeError, match="context capacity exceeded"):
        eng.prefill(synthetic.random_tokens(9, d.vocab, seed=1))
    with pytest.raises(ValueError, match="token ID outside vocabulary"):
        eng.prefill([1, d.vocab])
    assert eng.position == 0
    eng.prefill([1, 2, 3])
    assert eng.position == 3


@pytest.mark.parametrize("which,n", [("small", 70), ("g64", 33)])
def test_prefill_logits_every_position(which, n, small_int8, g64_int8):
    # the reference's `logits` command: one step with the head per prompt
    # token, every position's logits and argmax (src/main.cpp:93-114)
    model = {"small": small_int8, "g64": g64_int8}[which]
    d, _ = synthetic.load_model(model)
    prompt = synthetic.random_tokens(n, d.vocab, seed=21)
    eng = dcb.Engine(model, n + 2)
    logits, best = eng.prefill_logits(prompt)
    assert logits.shape == (n, d.vocab) and eng.position == n
    orc = oracle.Oracle(model, n + 2, threads=host_threads())
    for i, t in enumerate(prompt):
        exp = orc.step(t, True)
        np.testing.assert_allclose(logits[i], exp, atol=LOGIT_ATOL)
        assert best[i] == oracle.argmax(exp)
