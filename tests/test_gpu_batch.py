"""Batched decode: independent sequences stepping together, every projection
one tcgen05 int8 GEMM over all of them. Checked sequence by sequence against
the C restatement of the reference's step (src/model.cpp:258-329), each
sequence with its own KV cache pre-filled with seeded N(0,1) rows (the long-
context convention), its own position and its own tokens."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import SMALL, dcb, oracle, synthetic

pytestmark = pytest.mark.gpu

LOGIT_ATOL = 1e-3  # the FP32-KV parity bar


def _setup(model_dir, d, contexts, steps, kv="f32", seed=7, threads=1):
    eng = dcb.Engine(model_dir, 1)
    cap = max(contexts) + steps + 1
    bat = dcb.Batch(eng, len(contexts), cap, kv_dtype=kv)
    rng = np.random.default_rng(seed)
    orcs = []
    for s, ctx in enumerate(contexts):
        orc = oracle.Oracle(model_dir, cap, kv_f16=(kv == "f16"), threads=threads)
        kc, vc = orc.kv_view()
        for l in range(d.layers):
            k = rng.standard_normal((ctx, d.kv_dim), dtype=np.float32)
            v = rng.standard_normal((ctx, d.kv_dim), dtype=np.float32)
            if kv == "f16":
                k, v = oracle.f16_round(k), oracle.f16_round(v)
            kc[l, :ctx] = k
            vc[l, :ctx] = v
            if ctx:
                bat.kv_write(s, l, 0, k, v)
        orc.pos = ctx
        bat.set_position(s, ctx)
        orcs.append(orc)
    return eng, bat, orcs


def _run_and_compare(bat, orcs, toks, steps):
    worst = 0.0
    for _ in range(steps):
        got, best = bat.step(toks)
        for s, orc in enumerate(orcs):
            exp = orc.step(int(toks[s]))
            worst = max(worst, float(np.abs(got[s] - exp).max()))
            np.testing.assert_allclose(got[s], exp, atol=LOGIT_ATOL, err_msg=f"sequence {s}")
            assert best[s] == oracle.argmax(exp), s
        toks = best
    return worst


@pytest.mark.parametrize("kv", ["f32", "f16"])
def test_batch_matches_oracle_per_sequence(small_int8, kv):
    # Contexts across the 64-position chunk and 256-position split boundaries.
    contexts = [0, 1, 63, 64, 257, 300]
    eng, bat, orcs = _setup(small_int8, SMALL, contexts, 4, kv)
    toks = np.random.default_rng(11).integers(0, SMALL.vocab, len(contexts))
    _run_and_compare(bat, orcs, toks, 4)
    for s, ctx in enumerate(contexts):
        assert bat.position(s) == ctx + 4


@pytest.mark.parametrize("kv", ["f32", "f16"])
@pytest.mark.parametrize("which", ["g64", "g64b"])
def test_batch_head_dim_64(which, kv, g64_int8, g64b_int8):
    """head_dim 64: the TMA-fed attention kernel, contexts across its
    64-position chunks and 512-position splits."""
    from conftest import G64, G64B
    model, d = (g64_int8, G64) if which == "g64" else (g64b_int8, G64B)
    contexts = [0, 1, 63, 64, 511, 512, 513, 1100]
    eng, bat, orcs = _setup(model, d, contexts, 3, kv)
    toks = np.random.default_rng(21).integers(0, d.vocab, len(contexts))
    _run_and_compare(bat, orcs, toks, 3)


def test_batch_fused_path(g64_int8, monkeypatch):
    """The optional fusions: the split merge by the last attention block of a
    sequence, the staging of the next input inside the projections (after a
    grid barrier)."""
    from conftest import G64
    monkeypatch.setenv("DCB_BATCH_FUSE", "1")
    contexts = [0, 64, 600]
    eng, bat, orcs = _setup(g64_int8, G64, contexts, 2)
    assert bat.kernels_per_step(3) == 1 + 5 * G64.layers + 2
    toks = np.random.default_rng(22).integers(0, G64.vocab, len(contexts))
    _run_and_compare(bat, orcs, toks, 2)


def test_batch_tiled_head(g64_int8, monkeypatch):
    """The tiled LM head (one CTA per row tile), which runs when the persistent
    head's ring does not fit in shared memory."""
    from conftest import G64
    monkeypatch.setenv("DCB_BATCH_HEAD", "0")
    contexts = [0, 64, 600]
    eng, bat, orcs = _setup(g64_int8, G64, contexts, 2)
    toks = np.random.default_rng(24).integers(0, G64.vocab, len(contexts))
    _run_and_compare(bat, orcs, toks, 2)


def test_batch_all_64_slots(small_int8):
    contexts = list(np.random.default_rng(3).integers(0, 400, 64))
    eng, bat, orcs = _setup(small_int8, SMALL, contexts, 2)
    assert bat.slots == 64
    toks = np.random.default_rng(12).integers(0, SMALL.vocab, 64)
    _run_and_compare(bat, orcs, toks, 2)


def test_batch_odd_shapes(odd_int8):
    """Row lengths that are multiples of 4 but not of 16 or 128 (zero-padded
    rows, partial reduction tiles), head_dim 12."""
    from conftest import ODD
    contexts = [0, 5, 70]
    eng, bat, orcs = _setup(odd_int8, ODD, contexts, 3)
    toks = np.random.default_rng(13).integers(0, ODD.vocab, len(contexts))
    _run_and_compare(bat, orcs, toks, 3)


def test_batch_qwen05_shape(qwen05_int8):
    """The Qwen2.5-0.5B shape: 7/38 reduction stages, 1187 LM-head tiles."""
    d = synthetic.QWEN05
    contexts = [3, 200, 700]
    eng, bat, orcs = _setup(qwen05_int8, d, contexts, 2, threads=8)
    toks = np.random.default_rng(14).integers(0, d.vocab, len(contexts))
    _run_and_compare(bat, orcs, toks, 2)


def test_batch_device_chained_greedy_matches_host_loop(small_int8):
    contexts = [10, 100, 260]
    toks = np.array([5, 6, 7])
    _, host, _ = _setup(small_int8, SMALL, contexts, 6)
    _, dev, _ = _setup(small_int8, SMALL, contexts, 6)
    seq = []
    t = toks
    for _ in range(6):
        _, t = host.step(t, logits=False)
        seq.append(t.copy())
    dev.step(toks, logits=False)
    dev.step_greedy(3, 5)
    last, _ = dev.read(3)
    assert list(last) == list(seq[-1])
    for s, ctx in enumerate(contexts):
        assert dev.position(s) == ctx + 6


def test_batch_errors(small_int8):
    eng = dcb.Engine(small_int8, 1)
    bat = dcb.Batch(eng, 3, 8)
    with pytest.raises(ValueError, match="outside vocabulary"):
        bat.step([1, SMALL.vocab, 2])
    with pytest.raises(ValueError, match="sequence count"):
        bat.step(list(range(bat.slots + 1)))
    bat.set_position(1, 7)
    bat.step([1, 2, 3], logits=False)
    with pytest.raises(RuntimeError, match="capacity"):
        bat.step([1, 2, 3], logits=False)
    with pytest.raises(ValueError, match="max_seqs"):
        dcb.Batch(eng, 65, 8)
