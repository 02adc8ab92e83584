"""dcb_attention_noalloc (static device scratch, no per-call allocation)
against dcb_attention on the same inputs, through the C ABI. The file is
collected last so that it also runs after every other GPU test in the same
process; it passes alone as well (its first call then does the per-device
setup)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import dcb

pytestmark = pytest.mark.gpu

KV_CODE = {"f32": 0, "f16": 1}


def _inputs(length, heads, kvh, dim, kv, seed):
    import torch
    rng = np.random.default_rng(seed)
    q = torch.from_numpy(rng.standard_normal(heads * dim, dtype=np.float32)).cuda()
    tdt = torch.float16 if kv == "f16" else torch.float32
    k = torch.from_numpy(rng.standard_normal((length, kvh * dim), dtype=np.float32)).cuda().to(tdt)
    v = torch.from_numpy(rng.standard_normal((length, kvh * dim), dtype=np.float32)).cuda().to(tdt)
    return q, k, v


def _noalloc(q, k, v, kv, out, length, heads, kvh, dim, theta):
    return dcb.lib().dcb_attention_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), KV_CODE[kv], out.data_ptr(),
                                           length, heads, kvh, dim, float(theta), None)


@pytest.mark.parametrize("length,heads,kvh,dim,theta", [
    (1, 14, 2, 64, 1e6), (200, 14, 2, 64, 1e6), (4096, 14, 2, 64, 1e6), (32768, 14, 2, 64, 1e6),
    (77, 6, 2, 24, 0.0)])
@pytest.mark.parametrize("kv", ["f32", "f16"])
def test_noalloc_matches_allocating_entry_point(length, heads, kvh, dim, theta, kv):
    import torch
    q, k, v = _inputs(length, heads, kvh, dim, kv, seed=length + dim)
    want = torch.zeros(heads * dim, device="cuda")
    dcb.attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), kv, want.data_ptr(), length, heads, kvh, dim, theta)
    torch.cuda.synchronize()
    want = want.cpu().numpy()
    # Two calls in a row: the second finds the scratch as the first left it.
    for _ in range(2):
        got = torch.full((heads * dim,), float("nan"), device="cuda")
        assert _noalloc(q, k, v, kv, got, length, heads, kvh, dim, theta) == 0, dcb.lib().dcb_last_error()
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), want, atol=2e-5, rtol=1e-4)


def test_noalloc_rejects_scratch_beyond_its_size():
    import torch
    # 64 heads over one KV head at 4096 positions: 64 splits x 64 heads x 130
    # floats is about 2 MiB of partials, above the 1 MiB static scratch.
    length, heads, kvh, dim = 4096, 64, 1, 128
    q, k, v = _inputs(length, heads, kvh, dim, "f32", seed=1)
    out = torch.zeros(heads * dim, device="cuda")
    rc = _noalloc(q, k, v, "f32", out, length, heads, kvh, dim, 1e6)
    assert rc == 1  # DCB_ERR_ARGUMENT
    msg = dcb.lib().dcb_last_error().decode()
    assert "static scratch holds 1048576 bytes" in msg and "needs" in msg
    torch.cuda.synchronize()
    assert not out.any()
