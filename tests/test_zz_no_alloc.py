"""zt_pass_static, the pass for callers that cannot allocate device memory.

Some callers cannot give the library a workspace: their device memory belongs to an
allocator that reserved it up front, or they must not call cudaMalloc/cudaFree inside
a training step. zt_pass_static keeps the descriptor table in a fixed array inside the
library instead. These tests call it through the C ABI and check that two calls in a
row give exactly what the workspace-based zt_pass gives (0 ulp, the tolerance of the
other pass tests), and that a table over the size limit is refused.

The file is named to be collected last, so a run that stops at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SIZES = [(1, torch.bfloat16), (7, torch.float32), (1023, torch.bfloat16), (2049, torch.float16),
         (100003, torch.bfloat16), (5000, torch.float32)]


def make(seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    out = []
    for n, dt in SIZES:
        t = torch.empty(n, dtype=torch.float32, device="cuda")
        t.normal_(0.0, 0.02, generator=g)
        out.append(t.to(dt))
    return out


def test_static_pass_matches_workspace_pass_twice():
    from zotitan_b200 import _lib as L
    from zotitan_b200 import kernels as K
    f = lambda x: float(np.float32(x))  # noqa: E731
    a, b = make(3), make(3)
    m_a = [torch.zeros_like(t) for t in a]
    m_b = [torch.zeros_like(t) for t in b]
    calls = [
        (K.PassCfg(), [K.Stream(11, (f(1e-3),)), K.Stream(2**40 + 5, (f(1e-3),))]),
        (K.PassCfg(ge_mode=L.ZT_GE_ACCUM, momentum=L.ZT_MOM_STORED_EMA, beta1=f(0.9), one_minus_beta1=f(0.1),
                   m_scale=f(1 / f(0.1)), update=True, lr=f(1e-2)),
         [K.Stream(12, (), ge=f(0.5)), K.Stream(13, (f(1e-3),), ge=f(-0.7))]),
    ]
    table = K.ParamTable(a, n_params=20, m=m_a)
    for cfg, streams in calls:
        table.run(cfg, streams)
        K.pass_static(b, cfg, streams, n_params=20, m=m_b)
        torch.cuda.synchronize()
        for x, y in zip(a + m_a, b + m_b):
            assert torch.equal(x, y)


def test_static_pass_rejects_too_many_tensors():
    from zotitan_b200 import _lib as L
    lib = L.load()
    n = L.ZT_STATIC_MAX_TENSORS + 1
    arr = (L.ZtTensor * n)()
    cfg = L.ZtPassCfg()
    cfg.src, cfg.dst = L.ZT_BUF_DATA, L.ZT_BUF_DATA
    streams = (L.ZtStream * 1)()
    rc = lib.zt_pass_static(arr, n, n, ctypes.byref(cfg), streams, 0, None)
    assert rc == L.ZT_ERR_LIMIT
    assert b"ZT_STATIC_MAX_TENSORS" in lib.zt_last_error()
