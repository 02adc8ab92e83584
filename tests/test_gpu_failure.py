"""Failure detection on the device without a GPU fault: a step whose wait for
data that never comes runs out.

One engine is set up as rank 0 of a two-GPU KV split whose rank 1 never
writes its attention partials (both exchange pointers are this engine's own
buffer). The step kernel's bounded wait gives up after about a second, every
block leaves through its abort path, and the call returns DCB_ERR_DEVICE_WAIT
(TimeoutError) with the position unchanged. Set back to one GPU, the same
engine then steps with the logits of an engine that never failed.

The scenario runs in a child process with a time limit, so that a kernel
that failed to end would cost the process, not the test session."""
from __future__ import annotations

import json
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

CHILD = r"""
import json, sys, time
sys.path.insert(0, sys.argv[2])
sys.path.insert(0, sys.argv[2] + "/tests")
import numpy as np
from conftest import dcb

model = sys.argv[1]
out = {}
eng = dcb.Engine(model, 16)
own = eng.exchange_buffer()
eng.step(1)
eng.set_kv_shard(0, 2, 0, None, [own, own])
t = time.perf_counter()
try:
    eng.step(2)
    out["raised"] = None
except Exception as exc:
    out["raised"] = type(exc).__name__
    out["message"] = str(exc)
out["seconds"] = time.perf_counter() - t
out["position"] = eng.position
eng.set_kv_shard(0, 1, 0, None, [own])
logits, tok = eng.step(2)
ref = dcb.Engine(model, 16)
ref.step(1)
ref_logits, ref_tok = ref.step(2)
out["recovered_equal"] = bool(np.array_equal(logits, ref_logits)) and tok == ref_tok
print(json.dumps(out))
"""


def test_absent_peer_ends_the_step_with_a_wait_error(small_int8):
    r = subprocess.run([sys.executable, "-c", CHILD, str(small_int8), str(ROOT)], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["raised"] == "TimeoutError", out
    assert "ran out of time" in out["message"]
    assert out["seconds"] < 10.0, out  # one wait limit (1 s) plus the blocks' exits
    assert out["position"] == 1
    assert out["recovered_equal"], out
