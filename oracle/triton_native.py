"""Native-Triton checker for the noise source (test infrastructure, never shipped).

The reference's only GPU kernel, ``_philox_randn_kernel`` (zotitan/train_zo.py:18-22,
launched by ``_philox_randn`` at :25-28 with BLOCK=1024 and int32 offsets), stores
``tl.random.randn(seed, offs)``. Its arithmetic lives in the third-party Triton
library (3.6.0 in this image, triton/language/random.py), so the exact device
lowering of its ``log``/``cos``/``sqrt`` can only be pinned by running Triton
itself on the GPU. The functions here do that, with the reference's launch shape,
and are used only by the tests and by ``tests/golden/make_native_triton.py`` to
produce committed golden vectors. Nothing in ``zotitan_b200`` imports this module.
"""
from __future__ import annotations

import torch
import triton
import triton.language as tl


@triton.jit
def _randn_ref_shape(out_ptr, seed, n, BLOCK: tl.constexpr):
    # Same launch shape and offset arithmetic as zotitan/train_zo.py:18-22.
    pid = tl.program_id(0)
    offs = pid * BLOCK + tl.arange(0, BLOCK)
    tl.store(out_ptr + offs, tl.random.randn(seed, offs), mask=offs < n)


@triton.jit
def _randn_at(out_ptr, seed, offs_ptr, n, BLOCK: tl.constexpr):
    i = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
    m = i < n
    offs = tl.load(offs_ptr + i, mask=m, other=0)
    tl.store(out_ptr + i, tl.random.randn(seed, offs), mask=m)


@triton.jit
def _words_at(out_ptr, seed, offs_ptr, n, BLOCK: tl.constexpr):
    i = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
    m = i < n
    offs = tl.load(offs_ptr + i, mask=m, other=0)
    a, b, c, d = tl.random.randint4x(seed, offs)
    tl.store(out_ptr + 4 * i + 0, a, mask=m)
    tl.store(out_ptr + 4 * i + 1, b, mask=m)
    tl.store(out_ptr + 4 * i + 2, c, mask=m)
    tl.store(out_ptr + 4 * i + 3, d, mask=m)


@triton.jit
def _elementary(x_ptr, out_ptr, n, BLOCK: tl.constexpr):
    i = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
    m = i < n
    x = tl.load(x_ptr + i, mask=m, other=1.0)
    tl.store(out_ptr + 0 * n + i, tl.math.log(x), mask=m)
    tl.store(out_ptr + 1 * n + i, tl.math.cos(x), mask=m)
    tl.store(out_ptr + 2 * n + i, tl.math.sqrt(x), mask=m)


def randn_ref_shape(seed: int, n: int, device="cuda") -> torch.Tensor:
    """``_philox_randn(seed, n)`` as the reference launches it."""
    out = torch.empty(n, dtype=torch.float32, device=device)
    _randn_ref_shape[(triton.cdiv(n, 1024),)](out, seed, n, BLOCK=1024)
    return out


def randn_at(seed: int, offsets: torch.Tensor) -> torch.Tensor:
    """``tl.random.randn(seed, offs)`` at arbitrary int32 offsets."""
    offs = offsets.to(torch.int32).contiguous()
    n = offs.numel()
    out = torch.empty(n, dtype=torch.float32, device=offs.device)
    _randn_at[(triton.cdiv(n, 1024),)](out, seed, offs, n, BLOCK=1024)
    return out


def words_at(seed: int, offsets: torch.Tensor) -> torch.Tensor:
    """The four Philox words ``tl.random.randint4x(seed, offs)`` as int32 [n, 4]."""
    offs = offsets.to(torch.int32).contiguous()
    n = offs.numel()
    out = torch.empty(4 * n, dtype=torch.int32, device=offs.device)
    _words_at[(triton.cdiv(n, 1024),)](out, seed, offs, n, BLOCK=1024)
    return out.view(n, 4)


def elementary(x: torch.Tensor) -> torch.Tensor:
    """Triton's fp32 ``log``, ``cos`` and ``sqrt`` of x, as rows of a [3, n] tensor."""
    x = x.to(torch.float32).contiguous()
    n = x.numel()
    out = torch.empty(3 * n, dtype=torch.float32, device=x.device)
    _elementary[(triton.cdiv(n, 1024),)](x, out, n, BLOCK=1024)
    return out.view(3, n)
