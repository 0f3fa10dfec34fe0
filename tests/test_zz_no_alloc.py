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


def test_static_pass_allocates_nothing():
    """After a first call has resolved the array's address, further calls leave the
    device's free memory exactly where it was: the entry point allocates nothing."""
    from zotitan_b200 import _lib as L
    from zotitan_b200 import kernels as K
    f = lambda x: float(np.float32(x))  # noqa: E731
    b = make(5)
    m_b = [torch.zeros_like(t) for t in b]
    cfg = K.PassCfg(ge_mode=L.ZT_GE_ACCUM, momentum=L.ZT_MOM_STORED_EMA, beta1=f(0.9), one_minus_beta1=f(0.1),
                    m_scale=f(1 / f(0.1)), update=True, lr=f(1e-2))
    streams = [K.Stream(21, (), ge=f(0.25)), K.Stream(22, (f(1e-3),), ge=f(-0.5))]
    K.pass_static(b, cfg, streams, n_params=20, m=m_b)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for i in range(8):
        K.pass_static(b, cfg, [K.Stream(30 + i, (f(1e-3),), ge=f(0.1))], n_params=20, m=m_b)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def test_static_pass_refuses_capture_and_bad_arguments():
    """A capturing stream is refused (the table copy would replay from a reused host
    image), a rejected call reports its error, and the next call still runs."""
    from zotitan_b200 import _lib as L
    from zotitan_b200 import kernels as K
    lib = L.load()
    a, b = make(7), make(7)
    K.pass_static(b, K.PassCfg(), [K.Stream(1, (1e-3,))], n_params=20)  # resolves the address first
    desc = K.ParamTable.__new__(K.ParamTable)
    desc._describe(b, 20, None, None, None, None, None, None)
    good = K.PassCfg().to_c()
    streams = K._streams_array([K.Stream(2, (1e-3,))])
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        graph.capture_begin()
        try:
            rc = lib.zt_pass_static(desc._host, len(b), 20, ctypes.byref(good), streams, 1, ctypes.c_void_p(side.cuda_stream))
        finally:
            graph.capture_end()
    assert rc == L.ZT_ERR_INVALID
    assert b"capturing" in lib.zt_last_error()
    bad = K.PassCfg().to_c()
    bad.src = 7
    rc = lib.zt_pass_static(desc._host, len(b), 20, ctypes.byref(bad), streams, 1, None)
    assert rc == L.ZT_ERR_INVALID
    # the rejected calls changed nothing: b still equals a after the same passes
    table = K.ParamTable(a, n_params=20)
    table.run(K.PassCfg(), [K.Stream(1, (1e-3,))])
    for st in ([K.Stream(2, (1e-3,))], [K.Stream(3, (-2e-3,))]):
        table.run(K.PassCfg(), st)
        K.pass_static(b, K.PassCfg(), st, n_params=20)
    torch.cuda.synchronize()
    for x, y in zip(a, b):
        assert torch.equal(x, y)
