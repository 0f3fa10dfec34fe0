"""Thin torch-facing wrappers over the C ABI (include/zotitan_b200.h).

Every call is enqueued on torch's current CUDA stream; none synchronises.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib as L

_DT = {torch.float32: L.ZT_F32, torch.bfloat16: L.ZT_BF16, torch.float16: L.ZT_F16}


def _stream_ptr(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def param_key(seed: int, n_params: int, index: int) -> int:
    """(seed * n_params + index) & 0x7FFFFFFF with uint64 wrap-around (train_zo.py:302)."""
    return int(L.load().zt_param_key(seed & 0xFFFFFFFFFFFFFFFF, n_params, index))


def _check_cuda(t: torch.Tensor, name: str):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")


def philox_words(key: int, offsets: torch.Tensor) -> torch.Tensor:
    """[n, 4] int32 tensor holding the uint32 Philox words at `offsets` (int32/uint32 bits)."""
    _check_cuda(offsets, "offsets")
    offs = offsets.to(torch.int32).contiguous()
    out = torch.empty((offs.numel(), 4), dtype=torch.int32, device=offs.device)
    L.check(L.load().zt_philox_words(key, offs.data_ptr(), offs.numel(), out.data_ptr(), _stream_ptr(offs.device)),
            "zt_philox_words")
    return out


def randn(key: int, n: int, device, off0: int = 0) -> torch.Tensor:
    """The reference's ``_philox_randn(key, n)`` (zotitan/train_zo.py:25-28), offsets off0..off0+n-1."""
    device = torch.device(device)
    out = torch.empty(n, dtype=torch.float32, device=device)
    L.check(L.load().zt_randn(key, off0, n, out.data_ptr() if n else None, _stream_ptr(device)), "zt_randn")
    return out


def randn_keys(keys: list[int], n: int, device) -> torch.Tensor:
    """[len(keys), n] fp32: row j is the Gaussian field of key keys[j] at offsets 0..n-1."""
    device = torch.device(device)
    out = torch.empty((len(keys), n), dtype=torch.float32, device=device)
    arr = (ctypes.c_uint32 * max(1, len(keys)))(*keys)
    L.check(L.load().zt_randn_keys(arr, len(keys), n, out.data_ptr() if out.numel() else None, _stream_ptr(device)),
            "zt_randn_keys")
    return out


def randn_at(key: int, offsets: torch.Tensor) -> torch.Tensor:
    _check_cuda(offsets, "offsets")
    offs = offsets.to(torch.int32).contiguous()
    out = torch.empty(offs.numel(), dtype=torch.float32, device=offs.device)
    L.check(L.load().zt_randn_at(key, offs.data_ptr(), offs.numel(), out.data_ptr(), _stream_ptr(offs.device)),
            "zt_randn_at")
    return out


@dataclass
class Stream:
    """One noise stream of a pass (see zt_stream)."""
    seed: int
    chain: tuple = ()
    ge: float | None = None
    mom: float | None = None
    ge_dev: bool = False      # ge coefficient computed on the device from the pass's dev values
    z_store: bool = False     # also write the regenerated field to the pass's noise cache
    z_load: bool = False      # read the field from the noise cache instead of regenerating it
    z_field: int | None = None  # read the field from this slot of the pass's field store

    def to_c(self) -> L.ZtStream:
        if len(self.chain) > L.ZT_MAX_CHAIN:
            raise ValueError("at most 3 chained perturbations per stream")
        s = L.ZtStream()
        s.seed = self.seed & 0xFFFFFFFFFFFFFFFF
        for k, a in enumerate(self.chain):
            s.chain[k] = a
        s.n_chain = len(self.chain)
        s.flags = ((L.ZT_STREAM_GE if (self.ge is not None or self.ge_dev) else 0)
                   | (L.ZT_STREAM_MOM if self.mom is not None else 0)
                   | (L.ZT_STREAM_GE_DEV if self.ge_dev else 0)
                   | (L.ZT_STREAM_Z_STORE if self.z_store else 0)
                   | (L.ZT_STREAM_Z_LOAD if self.z_load else 0)
                   | (L.ZT_STREAM_Z_FIELD if self.z_field is not None else 0))
        s.zslot = self.z_field if self.z_field is not None else 0
        s.ge_coef = self.ge if self.ge is not None else 0.0
        s.mom_coef = self.mom if self.mom is not None else 0.0
        return s


@dataclass
class PassCfg:
    """Python view of zt_pass_cfg; scalars must already be fp32-representable."""
    src: int = L.ZT_BUF_DATA
    dst: int = L.ZT_BUF_DATA
    ge_mode: int = L.ZT_GE_NONE
    ge_scale: float | None = None
    momentum: int = L.ZT_MOM_NONE
    beta1: float = 0.0
    one_minus_beta1: float = 0.0
    m_scale: float = 1.0
    second_moment: bool = False
    beta2: float = 0.0
    one_minus_beta2: float = 0.0
    bc2: float = 1.0
    denom_eps: float = 0.0
    update: bool = False
    lr: float = 0.0
    wd: int = L.ZT_WD_NONE
    wd_lam: float = 0.0
    wd_factor: float = 1.0
    ge_load: bool = False
    ge_store: bool = False
    dev_pair: int | None = None     # pair whose device values feed a ge_dev stream
    dev_vals: int = 0               # device address of that pair's (v+, v-), set at launch
    dev_inv2eps: float = 0.0
    dev_invz: float = 0.0
    dev_tau: float = float("inf")
    unit_begin: int = 0             # work-unit range of the pass (unit_end 0: all units)
    unit_end: int = 0
    zcache: int = 0                 # device address of the plan's noise cache (n_units x 2048 fp32)
    zfield: int = 0                 # device address of the field store of the pass's unit range
    zfield_stride: int = 0          # fp32 elements between two slots of the field store
    zpush: tuple = ()               # per rank: device address (peer mapping) of its field store
    zpush_slot: int = 0             # slot the pushed field goes to
    zpush_chunk_units: int = 0      # units of one rank in one chunk of the flat layout
    zpush_stride: int = 0           # fp32 elements between two slots of a store

    def to_c(self) -> L.ZtPassCfg:
        c = L.ZtPassCfg()
        c.src, c.dst, c.ge_mode = self.src, self.dst, self.ge_mode
        c.ge_scale_on = int(self.ge_scale is not None)
        c.ge_scale = self.ge_scale if self.ge_scale is not None else 1.0
        c.momentum, c.beta1, c.one_minus_beta1, c.m_scale = self.momentum, self.beta1, self.one_minus_beta1, self.m_scale
        c.second_moment, c.beta2, c.one_minus_beta2 = int(self.second_moment), self.beta2, self.one_minus_beta2
        c.bc2, c.denom_eps, c.update, c.lr = self.bc2, self.denom_eps, int(self.update), self.lr
        c.wd, c.wd_lam, c.wd_factor = self.wd, self.wd_lam, self.wd_factor
        c.ge_load, c.ge_store = int(self.ge_load), int(self.ge_store)
        c.dev_vals = self.dev_vals or None
        c.dev_inv2eps, c.dev_invz, c.dev_tau = self.dev_inv2eps, self.dev_invz, self.dev_tau
        c.unit_begin, c.unit_end = self.unit_begin, self.unit_end
        c.zcache = self.zcache or None
        c.zfield = self.zfield or None
        c.zfield_stride = self.zfield_stride
        if self.zpush:
            if len(self.zpush) > L.ZT_MAX_PUSH_RANKS:
                raise ValueError(f"zpush: at most {L.ZT_MAX_PUSH_RANKS} ranks")
            for i, ptr in enumerate(self.zpush):
                c.zpush[i] = ptr
            c.zpush_ranks = len(self.zpush)
            c.zpush_slot, c.zpush_chunk_units, c.zpush_stride = self.zpush_slot, self.zpush_chunk_units, self.zpush_stride
        return c


def _streams_array(streams):
    if len(streams) > L.ZT_MAX_STREAMS:
        raise ValueError(f"{len(streams)} noise streams > {L.ZT_MAX_STREAMS}")
    arr = (L.ZtStream * max(1, len(streams)))()
    for i, s in enumerate(streams):
        arr[i] = s.to_c()
    return arr


def pass_static(params, cfg: PassCfg, streams: list, n_params=None, indices=None, live=None, m=None, v=None,
                anchor=None, ge=None) -> None:
    """One fused pass through zt_pass_static: no workspace, nothing allocated on the device.

    For callers that cannot allocate device memory (see include/zotitan_b200.h). Same
    arguments and result as ParamTable(...).run(cfg, streams); at most
    ZT_STATIC_MAX_TENSORS tensors. Calls that can overlap on the GPU race on the
    library's one descriptor array, so keep them on one stream."""
    desc = ParamTable.__new__(ParamTable)
    desc._describe(params, n_params, indices, live, m, v, anchor, ge)
    arr = _streams_array(streams)
    c = cfg.to_c()
    with torch.cuda.device(desc.device):
        L.check(L.load().zt_pass_static(desc._host, len(desc.params), desc.n_params, ctypes.byref(c), arr,
                                        len(streams), _stream_ptr(desc.device)), "zt_pass_static")


class ParamTable:
    """A zt_plan over trainable tensors, resident on their device.

    params[i] is the tensor at position indices[i] of an n_params-long trainable list
    (the reference's ``named_params``; the index feeds the per-tensor noise key).
    Optional parallel lists: live (second copy read by the model), m, v, anchor.
    The table keeps references to every tensor, so the pointers stay valid.
    """

    def __init__(self, params, n_params=None, indices=None, live=None, m=None, v=None, anchor=None, ge=None):
        self._describe(params, n_params, indices, live, m, v, anchor, ge)
        lib = L.load()
        n = len(self.params)
        nbytes = lib.zt_plan_workspace_bytes(n)
        self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        self.plan = L.ZtPlan()
        with torch.cuda.device(self.device):
            L.check(lib.zt_plan_init(self._host, n, self.n_params, self.workspace.data_ptr(), nbytes,
                                     ctypes.byref(self.plan), _stream_ptr(self.device)), "zt_plan_init")
        self.numel = int(self.plan.numel_total)

    def noise_cache(self) -> torch.Tensor:
        """A noise cache for this plan's passes (zt_pass_cfg.zcache): one fp32 per element
        slot of every work unit, i.e. about 4 bytes per parameter."""
        return torch.empty(int(self.plan.n_units) * L.ZT_UNIT_ELEMS, dtype=torch.float32, device=self.device)

    def _describe(self, params, n_params, indices, live, m, v, anchor, ge=None):
        """Validate the tensors and build the host zt_tensor array."""
        params = list(params)
        if not params:
            raise ValueError("empty parameter list")
        self.device = params[0].device
        if self.device.type != "cuda":
            raise ValueError("ParamTable needs CUDA tensors (no CPU fallback)")
        self.n_params = len(params) if n_params is None else n_params
        self.indices = list(range(len(params))) if indices is None else list(indices)
        self.params, self.live, self.m, self.v, self.anchor, self.ge = params, live, m, v, anchor, ge
        arr = (L.ZtTensor * len(params))()
        for i, p in enumerate(params):
            self._check(p, p, f"param {i}")
            arr[i].data = p.data_ptr()
            for name in ("live", "m", "v", "anchor", "ge"):
                lst = getattr(self, name)
                if lst is not None and lst[i] is not None:
                    self._check(lst[i], p, f"{name}[{i}]")
                    setattr(arr[i], name, lst[i].data_ptr())
            arr[i].numel = p.numel()
            arr[i].dtype = _DT[p.dtype]
            arr[i].index = self.indices[i]
        self._host = arr

    def _check(self, t: torch.Tensor, like: torch.Tensor, name: str):
        if t.device != self.device:
            raise ValueError(f"{name} is on {t.device}, expected {self.device}")
        if t.dtype not in _DT:
            raise ValueError(f"{name} has unsupported dtype {t.dtype}")
        if t.dtype != like.dtype or t.numel() != like.numel():
            raise ValueError(f"{name} must match its parameter's dtype and numel")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")

    def run(self, cfg: PassCfg, streams: list[Stream]) -> None:
        """One fused pass (zt_pass) on torch's current stream."""
        arr = _streams_array(streams)
        c = cfg.to_c()
        with torch.cuda.device(self.device):
            L.check(L.load().zt_pass(ctypes.byref(self.plan), ctypes.byref(c), arr, len(streams),
                                     _stream_ptr(self.device)), "zt_pass")


def eggroll_linear(x: torch.Tensor, w: torch.Tensor, a: torch.Tensor, b: torch.Tensor | None, sigma: torch.Tensor,
                   rows_per_member: int, out: torch.Tensor | None = None, xb: torch.Tensor | None = None,
                   xb_ready: bool = False, x_ext: torch.Tensor | None = None,
                   w_ext: torch.Tensor | None = None, test_stall_loads: bool = False) -> torch.Tensor:
    """EGGROLL population linear layer (zt_eggroll_linear):
    Y = X W^T + sigma_i (X B_i) A_i^T for the rows of member i.

    x [M, K] bf16, w [N, K] bf16, a [members, N, 4] fp32, b [members, K, 4] fp32,
    sigma [members] fp32; returns Y [M, N] bf16. M % 128, N % 256, K % 64 must be 0 and
    rows_per_member a multiple of 128 dividing M. With xb_ready, xb already holds X B_i
    (from eggroll_xb) and b may be None. With x_ext (eggroll_xb_ext) and w_ext (the
    factors' A_ext) the rank-4 term runs on the tensor cores as a K = 16 slab.
    test_stall_loads: test hook (zt_eggroll_args.test_stall_loads), the GEMM loads nothing
    and reports an expired wait through eggroll_take_error."""
    if (x_ext is None) != (w_ext is None):
        raise ValueError("x_ext and w_ext go together")
    if x_ext is not None:
        M, K = x.shape
        N = w.shape[0]
        for t, name in ((x, "x"), (w, "w"), (x_ext, "x_ext"), (w_ext, "w_ext")):
            _check_cuda(t, name)
            if not t.is_contiguous() or t.dtype != torch.bfloat16:
                raise ValueError(f"{name} must be contiguous bf16")
        if w.shape[1] != K or x_ext.shape != (M, 16) or w_ext.shape != (M // rows_per_member, N, 16):
            raise ValueError("inconsistent shapes")
        if out is None:
            out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
        args = L.ZtEggrollArgs(x.data_ptr(), w.data_ptr(), None, None, None, None, out.data_ptr(), M, N, K,
                               rows_per_member, 4, 0, int(test_stall_loads), x_ext.data_ptr(), w_ext.data_ptr())
        with torch.cuda.device(x.device):
            L.check(L.load().zt_eggroll_linear(ctypes.byref(args), _stream_ptr(x.device)), "zt_eggroll_linear")
        return out
    if xb_ready and xb is None:
        raise ValueError("xb_ready needs xb")
    named = [(x, "x"), (w, "w"), (a, "a"), (sigma, "sigma")] + ([] if xb_ready else [(b, "b")])
    for t, name in named:
        _check_cuda(t, name)
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise ValueError("x and w must be bf16")
    if a.dtype != torch.float32 or sigma.dtype != torch.float32 or (b is not None and b.dtype != torch.float32):
        raise ValueError("a, b and sigma must be fp32")
    M, K = x.shape
    N = w.shape[0]
    members = M // rows_per_member
    if w.shape[1] != K or a.shape != (members, N, 4) or sigma.shape != (members,):
        raise ValueError("inconsistent shapes")
    if b is not None and b.shape != (members, K, 4):
        raise ValueError("inconsistent shapes")
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    if xb is None:
        xb = torch.empty((M, 4), dtype=torch.float32, device=x.device)
    args = L.ZtEggrollArgs(x.data_ptr(), w.data_ptr(), a.data_ptr(), b.data_ptr() if b is not None else None,
                           sigma.data_ptr(), xb.data_ptr(), out.data_ptr(), M, N, K, rows_per_member, 4,
                           1 if xb_ready else 0, int(test_stall_loads))
    with torch.cuda.device(x.device):
        L.check(L.load().zt_eggroll_linear(ctypes.byref(args), _stream_ptr(x.device)), "zt_eggroll_linear")
    return out


def eggroll_xb_ext(x: torch.Tensor, bs: list, scales: list, slots: list, rows_per_member: int,
                   bt: torch.Tensor | None = None) -> list:
    """K-slab rows of sigma_i X B_s (zt_eggroll_xb with xe outputs): slot 0 gives a set its
    own [M, 16] bf16 buffer [hi, lo, 0 x 8]; slots 1 and 2 share one buffer (columns 0-7
    and 8-15, the gated gate/up form). Returns one buffer per set (shared ones repeated).
    With bt (all sets' B^T, [members, 16, K] bf16 from eggroll_factors' b_ext) the product
    runs on the tensor cores and the fp32 bs are not read."""
    if bt is not None:
        _check_cuda(bt, "bt")
        if bt.dtype != torch.bfloat16 or not bt.is_contiguous() or \
                bt.shape != (x.shape[0] // rows_per_member, 16, x.shape[1]):
            raise ValueError("bt must be a contiguous bf16 [members, 16, K] tensor")
    if not 1 <= len(bs) <= 3 or len(scales) != len(bs) or len(slots) != len(bs):
        raise ValueError("one to three factor sets, with a scale and a slot each")
    _check_cuda(x, "x")
    if x.dtype != torch.bfloat16 or not x.is_contiguous() or x.dim() != 2:
        raise ValueError("x must be a contiguous bf16 matrix")
    M, K = x.shape
    shared = None
    xes = []
    for b, sc, slot in zip(bs, scales, slots):
        _check_cuda(b, "b")
        if b.dtype != torch.float32 or not b.is_contiguous() or b.shape != (M // rows_per_member, K, 4):
            raise ValueError("each b must be a contiguous fp32 [members, K, 4] tensor")
        if sc.dtype != torch.float32 or sc.shape != (M // rows_per_member,):
            raise ValueError("each scale must be fp32 [members]")
        if slot == 0:
            xes.append(torch.empty((M, 16), dtype=torch.bfloat16, device=x.device))
        elif slot in (1, 2):
            if shared is None:
                shared = torch.empty((M, 16), dtype=torch.bfloat16, device=x.device)
            xes.append(shared)
        else:
            raise ValueError("slot must be 0, 1 or 2")
    n = len(bs)
    pad = [0] * (3 - n)
    args = L.ZtEggrollXbArgs(x.data_ptr(), (ctypes.c_void_p * 3)(*([b.data_ptr() for b in bs] + pad)),
                             (ctypes.c_void_p * 3)(*([0] * 3)), M, K, n, rows_per_member,
                             (ctypes.c_void_p * 3)(*([sc.data_ptr() for sc in scales] + pad)),
                             (ctypes.c_void_p * 3)(*([t.data_ptr() for t in xes] + pad)),
                             (ctypes.c_int32 * 3)(*(list(slots) + pad)), 0, bt.data_ptr() if bt is not None else None)
    with torch.cuda.device(x.device):
        L.check(L.load().zt_eggroll_xb(ctypes.byref(args), _stream_ptr(x.device)), "zt_eggroll_xb")
    return xes


def eggroll_xb(x: torch.Tensor, bs: list, rows_per_member: int) -> list:
    """X B_s for 1-3 factor sets sharing x [M, K] bf16 (zt_eggroll_xb): returns one
    [M, 4] fp32 tensor per b in bs ([members, K, 4] fp32 each)."""
    if not 1 <= len(bs) <= 3:
        raise ValueError("one to three factor sets")
    _check_cuda(x, "x")
    if x.dtype != torch.bfloat16 or not x.is_contiguous() or x.dim() != 2:
        raise ValueError("x must be a contiguous bf16 matrix")
    M, K = x.shape
    for b in bs:
        _check_cuda(b, "b")
        if b.dtype != torch.float32 or not b.is_contiguous() or b.shape != (M // rows_per_member, K, 4):
            raise ValueError("each b must be a contiguous fp32 [members, K, 4] tensor")
    xbs = [torch.empty((M, 4), dtype=torch.float32, device=x.device) for _ in bs]
    bp = [b.data_ptr() for b in bs] + [0] * (3 - len(bs))
    xp = [t.data_ptr() for t in xbs] + [0] * (3 - len(bs))
    args = L.ZtEggrollXbArgs(x.data_ptr(), (ctypes.c_void_p * 3)(*bp), (ctypes.c_void_p * 3)(*xp), M, K, len(bs),
                             rows_per_member, (ctypes.c_void_p * 3)(0, 0, 0), (ctypes.c_void_p * 3)(0, 0, 0),
                             (ctypes.c_int32 * 3)(0, 0, 0), 0, None)
    with torch.cuda.device(x.device):
        L.check(L.load().zt_eggroll_xb(ctypes.byref(args), _stream_ptr(x.device)), "zt_eggroll_xb")
    return xbs


def eggroll_gated(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor, fac_gate, fac_up, xb_gate, xb_up,
                  rows_per_member: int, x_ext: torch.Tensor | None = None) -> torch.Tensor:
    """bf16(bf16(silu(G)) * U) for the population rows x [M, K] (zt_eggroll_gated):
    G, U the EGGROLL linear outputs of the gate and up projections. fac_* = (A, B, scale)
    from eggroll_factors; xb_* = X B from eggroll_xb. M % 256 == 0. With x_ext (the shared
    slot-1/2 buffer of eggroll_xb_ext) the factors carry A_ext (slots 0 and 1) and both
    rank-4 terms run on the tensor cores; xb_* may then be None."""
    named = [(x, "x"), (w_gate, "w_gate"), (w_up, "w_up")]
    named += [(x_ext, "x_ext"), (fac_gate[3], "gate A_ext"), (fac_up[3], "up A_ext")] if x_ext is not None else \
        [(xb_gate, "xb_gate"), (xb_up, "xb_up")]
    for t, name in named:
        _check_cuda(t, name)
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    M, K = x.shape
    N = w_gate.shape[0]
    if w_up.shape != (N, K) or w_gate.shape[1] != K:
        raise ValueError("inconsistent shapes")
    members = M // rows_per_member
    for fac in (fac_gate, fac_up):
        if fac[0].shape != (members, N, 4) or fac[2].shape != (members,):
            raise ValueError("inconsistent factor shapes")
        if x_ext is not None and (len(fac) < 4 or fac[3].shape != (members, N, 16)):
            raise ValueError("the K-slab form needs the factors' A_ext")
    y = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    ext = x_ext is not None
    args = L.ZtEggrollGatedArgs(x.data_ptr(), w_gate.data_ptr(), w_up.data_ptr(), fac_gate[0].data_ptr(),
                                fac_up[0].data_ptr(), fac_gate[2].data_ptr(), fac_up[2].data_ptr(),
                                None if ext else xb_gate.data_ptr(), None if ext else xb_up.data_ptr(), y.data_ptr(),
                                M, N, K, rows_per_member, 4, x_ext.data_ptr() if ext else None,
                                fac_gate[3].data_ptr() if ext else None, fac_up[3].data_ptr() if ext else None)
    with torch.cuda.device(x.device):
        L.check(L.load().zt_eggroll_gated(ctypes.byref(args), _stream_ptr(x.device)), "zt_eggroll_gated")
    return y


def eggroll_take_error() -> int:
    """Read and clear the EGGROLL kernels' device error code (synchronous)."""
    code = ctypes.c_int32(0)
    L.check(L.load().zt_eggroll_take_error(ctypes.byref(code)), "zt_eggroll_take_error")
    return int(code.value)


_DT = {torch.float32: L.ZT_F32, torch.bfloat16: L.ZT_BF16, torch.float16: L.ZT_F16}


def _keys_array(keys):
    arr = (ctypes.c_uint32 * max(1, len(keys)))(*[int(k) & 0xFFFFFFFF for k in keys])
    return arr


def _dev_seeds(dev_seeds, device):
    """(seeds, n_params, *indices) with seeds an int64 CUDA tensor of uint64 pair seeds."""
    seeds = dev_seeds[0]
    _check_cuda(seeds, "seeds")
    device = torch.device(device)
    if device.index is None:
        device = torch.device(device.type, torch.cuda.current_device())
    if seeds.dtype != torch.int64 or not seeds.is_contiguous() or seeds.device != device:
        raise ValueError("seeds must be a contiguous int64 tensor on the call's device")
    return seeds, int(dev_seeds[1]), [int(i) & 0xFFFFFFFF for i in dev_seeds[2:]]


def eggroll_factors(keys_a: list[int] | None, keys_b: list[int] | None, n: int, k: int, sigma: float, device,
                    dtype: torch.dtype = torch.bfloat16, normalize: bool = True, ext_slot: int | None = None,
                    b_ext: torch.Tensor | None = None, b_ext_row: int = 0, dev_seeds=None):
    """Rank-4 factors of an [n, k] tensor for antithetic pairs (zt_eggroll_factors):
    returns A [2p, n, 4], B [2p, k, 4] (fp32 holding dtype-rounded values) and the signed
    scale [2p] (+sigma c_j, -sigma c_j), ready for eggroll_linear. With ext_slot (0 or 1)
    also A_ext [2p, n, 16] bf16, the GEMM's K-slab operand, as a fourth element. With
    b_ext ([2p, 16, k] bf16, zeroed by the caller) B^T is also written to its rows
    b_ext_row .. b_ext_row + 3 (the tensor-core X B operand of eggroll_xb_ext).
    dev_seeds = (seeds, n_params, index_a, index_b) derives the keys on the device from
    the pair seeds in `seeds` (int64 CUDA tensor, one per pair): zt_param_key(seed,
    n_params, index_a / index_b); keys_a and keys_b are then not used. A captured CUDA
    graph of the call stays valid for new pairs once their seeds are copied into `seeds`."""
    seeds = None
    if dev_seeds is not None:
        seeds, n_params, (ia, ib) = _dev_seeds(dev_seeds, device)
        keys_a = keys_b = [0] * seeds.numel()
    if b_ext is not None:
        _check_cuda(b_ext, "b_ext")
        if b_ext.dtype != torch.bfloat16 or not b_ext.is_contiguous() or b_ext.shape != (2 * len(keys_a), 16, k):
            raise ValueError("b_ext must be a contiguous bf16 [2p, 16, k] tensor")
    pairs = len(keys_a)
    if pairs != len(keys_b) or pairs == 0:
        raise ValueError("keys_a and keys_b must be non-empty and of equal length")
    if pairs > L.ZT_EGGROLL_MAX_PAIRS:
        raise ValueError(f"at most {L.ZT_EGGROLL_MAX_PAIRS} pairs per call")
    device = torch.device(device)
    a = torch.empty((2 * pairs, n, 4), dtype=torch.float32, device=device)
    b = torch.empty((2 * pairs, k, 4), dtype=torch.float32, device=device)
    scale = torch.empty(2 * pairs, dtype=torch.float32, device=device)
    work = torch.empty(pairs * L.ZT_EGGROLL_FACTOR_WORK_FLOATS, dtype=torch.float32, device=device)
    a_ext = None if ext_slot is None else torch.empty((2 * pairs, n, 16), dtype=torch.bfloat16, device=device)
    ka, kb = _keys_array(keys_a), _keys_array(keys_b)
    args = L.ZtEggrollFactorArgs(ctypes.addressof(ka), ctypes.addressof(kb), pairs, 4, n, k, _DT[dtype],
                                 1 if normalize else 0, float(sigma), 0, a.data_ptr(), b.data_ptr(), scale.data_ptr(),
                                 work.data_ptr(), a_ext.data_ptr() if a_ext is not None else None,
                                 int(ext_slot or 0), 0, b_ext.data_ptr() if b_ext is not None else None,
                                 int(b_ext_row), 0)
    if seeds is not None:
        args.seeds, args.n_params, args.key_index_a, args.key_index_b = seeds.data_ptr(), n_params, ia, ib
    with torch.cuda.device(device):
        L.check(L.load().zt_eggroll_factors(ctypes.byref(args), _stream_ptr(device)), "zt_eggroll_factors")
    return (a, b, scale) if a_ext is None else (a, b, scale, a_ext)


def eggroll_rmsnorm(x: torch.Tensor, w: torch.Tensor, keys: list[int] | None, sigma: float, eps: float,
                    rows_per_member: int, dev_seeds=None) -> torch.Tensor:
    """Llama RMSNorm of population rows x [M, d] with member-perturbed weights
    (zt_eggroll_rmsnorm): members 2j / 2j+1 use bf16(w +- sigma randn(keys[j])).
    dev_seeds = (seeds, n_params, index): keys derived on the device, as eggroll_factors."""
    seeds = None
    if dev_seeds is not None:
        seeds, n_params, (ki,) = _dev_seeds(dev_seeds, x.device)
        keys = [0] * seeds.numel()
    _check_cuda(x, "x")
    _check_cuda(w, "w")
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise ValueError("x and w must be bf16")
    if not x.is_contiguous() or not w.is_contiguous():
        raise ValueError("x and w must be contiguous")
    d = w.shape[0]
    x2 = x.reshape(-1, d)
    pairs = len(keys)
    wm = torch.empty((2 * pairs, d), dtype=torch.bfloat16, device=x.device)
    y = torch.empty_like(x2)
    ka = _keys_array(keys)
    args = L.ZtEggrollNormArgs(x2.data_ptr(), w.data_ptr(), ctypes.addressof(ka), wm.data_ptr(), y.data_ptr(),
                               x2.shape[0], d, pairs, rows_per_member, float(sigma), float(eps))
    if seeds is not None:
        args.seeds, args.n_params, args.key_index = seeds.data_ptr(), n_params, ki
    with torch.cuda.device(x.device):
        L.check(L.load().zt_eggroll_rmsnorm(ctypes.byref(args), _stream_ptr(x.device)), "zt_eggroll_rmsnorm")
    return y.view(x.shape)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """Llama RMSNorm of bf16 rows x [..., d] with weight w [d] (zt_rmsnorm):
    w * bf16(x * rsqrt(mean(x^2) + eps)), statistics in fp32."""
    _check_cuda(x, "x")
    _check_cuda(w, "w")
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise ValueError("x and w must be bf16")
    if not x.is_contiguous() or not w.is_contiguous():
        raise ValueError("x and w must be contiguous")
    d = w.shape[0]
    if x.shape[-1] != d:
        raise ValueError("x's last dimension must equal w's length")
    y = torch.empty_like(x)
    with torch.cuda.device(x.device):
        L.check(L.load().zt_rmsnorm(x.data_ptr(), w.data_ptr(), y.data_ptr(), x.numel() // d, d, float(eps),
                                    _stream_ptr(x.device)), "zt_rmsnorm")
    return y


def eggroll_rope_(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, seq: int, head_dim: int):
    """In-place rotary embedding of q [rows, Hq*hd] and k [rows, Hk*hd] (bf16, row r at
    position r % seq) with cos, sin [seq, hd] bf16 (zt_eggroll_rope)."""
    for t, name in ((q, "q"), (k, "k"), (cos, "cos"), (sin, "sin")):
        _check_cuda(t, name)
        if t.dtype != torch.bfloat16 or not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous bf16")
    rows = q.numel() // q.shape[-1]
    if cos.shape != (seq, head_dim) or sin.shape != (seq, head_dim):
        raise ValueError("cos and sin must be [seq, head_dim]")
    hq, hk = q.shape[-1] // head_dim, k.shape[-1] // head_dim
    with torch.cuda.device(q.device):
        L.check(L.load().zt_eggroll_rope(q.data_ptr(), k.data_ptr(), cos.data_ptr(), sin.data_ptr(), rows, seq, hq, hk,
                                         head_dim, _stream_ptr(q.device)), "zt_eggroll_rope")
    return q, k


def eggroll_swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """bf16(bf16(silu(gate)) * up) (zt_eggroll_swiglu)."""
    for t, name in ((gate, "gate"), (up, "up")):
        _check_cuda(t, name)
        if t.dtype != torch.bfloat16 or not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous bf16")
    if gate.shape != up.shape:
        raise ValueError("gate and up must have the same shape")
    out = torch.empty_like(gate)
    with torch.cuda.device(gate.device):
        L.check(L.load().zt_eggroll_swiglu(gate.data_ptr(), up.data_ptr(), out.data_ptr(), gate.numel(),
                                           _stream_ptr(gate.device)), "zt_eggroll_swiglu")
    return out


def gemm_swiglu(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    """bf16(bf16(silu(bf16(x w_gate^T))) * bf16(x w_up^T)) as one tcgen05 GEMM
    (zt_gemm_swiglu): x [m, k], w_gate / w_up [n, k] bf16, m % 256 == 0, n % 128 == 0,
    k % 64 == 0."""
    for t, name in ((x, "x"), (w_gate, "w_gate"), (w_up, "w_up")):
        _check_cuda(t, name)
        if t.dtype != torch.bfloat16 or not t.is_contiguous() or t.dim() != 2:
            raise ValueError(f"{name} must be a contiguous bf16 matrix")
    m, k = x.shape
    n = w_gate.shape[0]
    if w_gate.shape != (n, k) or w_up.shape != (n, k):
        raise ValueError("w_gate and w_up must be [n, k] with x's k")
    y = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    with torch.cuda.device(x.device):
        L.check(L.load().zt_gemm_swiglu(x.data_ptr(), w_gate.data_ptr(), w_up.data_ptr(), y.data_ptr(), m, n, k,
                                        _stream_ptr(x.device)), "zt_gemm_swiglu")
    return y


def xent_rows(logits: torch.Tensor, targets: torch.Tensor, want_lse: bool = True, want_correct: bool = True):
    """Per-row cross-entropy statistics of bf16 logits [rows, vocab] against int64
    targets [rows] (negative = ignored), zt_xent_rows: returns (loss, lse | None,
    correct | None) as fp32, fp32, int32 [rows]."""
    _check_cuda(logits, "logits")
    _check_cuda(targets, "targets")
    if logits.dtype != torch.bfloat16 or logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be a bf16 [rows, vocab] matrix with unit column stride")
    if targets.dtype != torch.int64 or targets.shape != (logits.shape[0],) or not targets.is_contiguous():
        raise ValueError("targets must be a contiguous int64 [rows] vector")
    rows, vocab = logits.shape
    dev = logits.device
    loss = torch.empty(rows, dtype=torch.float32, device=dev)
    lse = torch.empty(rows, dtype=torch.float32, device=dev) if want_lse else None
    correct = torch.empty(rows, dtype=torch.int32, device=dev) if want_correct else None
    with torch.cuda.device(dev):
        L.check(L.load().zt_xent_rows(logits.data_ptr(), logits.stride(0), rows, vocab, targets.data_ptr(),
                                      loss.data_ptr(), lse.data_ptr() if lse is not None else None,
                                      correct.data_ptr() if correct is not None else None, _stream_ptr(dev)),
                "zt_xent_rows")
    return loss, lse, correct


def gemm_addto(w: torch.Tensor, a: torch.Tensor, b: torch.Tensor, alpha: float) -> torch.Tensor:
    """In place: w <- bf16(w + alpha * a @ b.T) (zt_gemm_addto), w [m, n], a [m, k], b [n, k]
    bf16 contiguous; one rounding of w, the product accumulated in fp32 on the tensor cores."""
    for t, name in ((w, "w"), (a, "a"), (b, "b")):
        _check_cuda(t, name)
        if t.dtype != torch.bfloat16 or t.dim() != 2 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous bf16 matrix")
    m, n = w.shape
    k = a.shape[1]
    if a.shape != (m, k) or b.shape != (n, k):
        raise ValueError("inconsistent shapes")
    with torch.cuda.device(w.device):
        L.check(L.load().zt_gemm_addto(w.data_ptr(), n, a.data_ptr(), b.data_ptr(), float(np.float32(alpha)), m, n, k,
                                       _stream_ptr(w.device)), "zt_gemm_addto")
    return w


def gemm_addto_supported(w: torch.Tensor, k: int) -> bool:
    return (w.is_cuda and w.dtype == torch.bfloat16 and w.dim() == 2 and w.is_contiguous() and w.shape[1] % 32 == 0
            and k % 64 == 0 and w.data_ptr() % 16 == 0)


def gemm_take_error() -> int:
    code = ctypes.c_int32(0)
    L.check(L.load().zt_gemm_take_error(ctypes.byref(code)), "zt_gemm_take_error")
    return int(code.value)


def linear_xent_supported(x: torch.Tensor, w: torch.Tensor) -> bool:
    """Whether zt_linear_xent takes these operands: bf16, contiguous, 16-byte aligned, the
    inner dimension a multiple of 64."""
    return (x.is_cuda and w.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.dim() == 2
            and w.dim() == 2 and x.shape[1] == w.shape[1] and x.shape[1] % 64 == 0 and x.is_contiguous()
            and w.is_contiguous() and x.data_ptr() % 16 == 0 and w.data_ptr() % 16 == 0 and x.shape[0] > 0)


_LCE_WS: dict = {}


def linear_xent(x: torch.Tensor, w: torch.Tensor, targets: torch.Tensor, want_lse: bool = True,
                want_correct: bool = True, test_stall_loads: bool = False, test_wait_cycles: int = 0):
    """Fused lm_head + cross-entropy statistics (zt_linear_xent): x [rows, k] bf16 hidden
    states, w [vocab, k] bf16 head weight, int64 targets [rows] (negative = ignored).
    Returns (loss, lse | None, correct | None) as zt_xent_rows on bf16(x @ w.T) would,
    without writing the logits. test_stall_loads / test_wait_cycles: the test hooks of
    zt_lce_args (the GEMM loads nothing and reports an expired wait)."""
    if not linear_xent_supported(x, w):
        raise ValueError("x and w must be contiguous 16-byte aligned bf16 CUDA matrices with k % 64 == 0")
    if targets.dtype != torch.int64 or targets.shape != (x.shape[0],) or not targets.is_contiguous():
        raise ValueError("targets must be a contiguous int64 [rows] vector")
    rows, k = x.shape
    vocab = w.shape[0]
    dev = x.device
    lib = L.load()
    with torch.cuda.device(dev):
        need = lib.zt_linear_xent_workspace_bytes(rows, vocab, k)
        if need == 0:
            L.check(L.ZT_ERR_INVALID, "zt_linear_xent_workspace_bytes")
        ws = _LCE_WS.get(dev)
        if ws is None or ws.numel() < need:
            ws = torch.empty(need, dtype=torch.uint8, device=dev)
            _LCE_WS[dev] = ws
        loss = torch.empty(rows, dtype=torch.float32, device=dev)
        lse = torch.empty(rows, dtype=torch.float32, device=dev) if want_lse else None
        correct = torch.empty(rows, dtype=torch.int32, device=dev) if want_correct else None
        args = L.ZtLceArgs(x.data_ptr(), w.data_ptr(), targets.data_ptr(), loss.data_ptr(),
                           lse.data_ptr() if lse is not None else None,
                           correct.data_ptr() if correct is not None else None, ws.data_ptr(), ws.numel(), rows,
                           vocab, k, int(test_stall_loads), 0, int(test_wait_cycles))
        L.check(lib.zt_linear_xent(ctypes.byref(args), _stream_ptr(dev)), "zt_linear_xent")
    return loss, lse, correct


def linear_xent_take_error() -> int:
    code = ctypes.c_int32(0)
    L.check(L.load().zt_linear_xent_take_error(ctypes.byref(code)), "zt_linear_xent_take_error")
    return int(code.value)


def eggroll_update_operands(a: torch.Tensor, b: torch.Tensor, scale: torch.Tensor, coef: torch.Tensor,
                            sigma: float, dtype: torch.dtype = torch.bfloat16):
    """(a_cat [n, 8p], b_cat [k, 8p]) bf16 operands of the ES update GEMM of one 2-D tensor
    (zt_eggroll_update_operands), from eggroll_factors' outputs for p pairs and the pairs'
    coefficients: a_cat @ b_cat.T = sum_j coef_j c_j P_j Psi_j."""
    if dtype != torch.bfloat16:
        raise NotImplementedError("bf16 update operands only")
    pairs = coef.numel()
    n, k = a.shape[1], b.shape[1]
    for t, name in ((a, "a"), (b, "b"), (scale, "scale"), (coef, "coef")):
        _check_cuda(t, name)
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous fp32")
    if a.shape != (2 * pairs, n, 4) or b.shape != (2 * pairs, k, 4) or scale.shape != (2 * pairs,):
        raise ValueError("inconsistent shapes")
    a_cat = torch.empty((n, 8 * pairs), dtype=torch.bfloat16, device=a.device)
    b_cat = torch.empty((k, 8 * pairs), dtype=torch.bfloat16, device=a.device)
    with torch.cuda.device(a.device):
        L.check(L.load().zt_eggroll_update_operands(a.data_ptr(), b.data_ptr(), scale.data_ptr(), coef.data_ptr(),
                                                    pairs, n, k, float(sigma), a_cat.data_ptr(), b_cat.data_ptr(),
                                                    _stream_ptr(a.device)), "zt_eggroll_update_operands")
    return a_cat, b_cat


def lora_add_(out: torch.Tensor, xa: torch.Tensor, b: torch.Tensor, scale: float) -> torch.Tensor:
    """out += bf16(scale * xa @ b.T) in place with bf16 rounding of the delta and of the sum
    (zt_lora_add): out [rows, n] bf16, xa [rows, r] fp32, b [n, r] fp32."""
    for t, name in ((out, "out"), (xa, "xa"), (b, "b")):
        _check_cuda(t, name)
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if out.dtype != torch.bfloat16 or xa.dtype != torch.float32 or b.dtype != torch.float32:
        raise ValueError("out must be bf16, xa and b fp32")
    rows, n = out.shape
    r = xa.shape[1]
    if xa.shape[0] != rows or b.shape != (n, r):
        raise ValueError("inconsistent shapes")
    with torch.cuda.device(out.device):
        L.check(L.load().zt_lora_add(out.data_ptr(), xa.data_ptr(), b.data_ptr(), float(scale), rows, n, r,
                                     _stream_ptr(out.device)), "zt_lora_add")
    return out


def lora_add3_(out: torch.Tensor, xa3: torch.Tensor, b: torch.Tensor, scale: float) -> torch.Tensor:
    """lora_add_ with xa given as three partial products xa3 [rows, 3r] fp32, summed as
    ((p0 + p1) + p2) in fp32 inside the kernel (zt_lora_add3)."""
    for t, name in ((out, "out"), (xa3, "xa3"), (b, "b")):
        _check_cuda(t, name)
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if out.dtype != torch.bfloat16 or xa3.dtype != torch.float32 or b.dtype != torch.float32:
        raise ValueError("out must be bf16, xa3 and b fp32")
    rows, n = out.shape
    r = b.shape[1]
    if xa3.shape != (rows, 3 * r) or b.shape != (n, r):
        raise ValueError("inconsistent shapes")
    with torch.cuda.device(out.device):
        L.check(L.load().zt_lora_add3(out.data_ptr(), xa3.data_ptr(), b.data_ptr(), float(scale), rows, n, r,
                                      _stream_ptr(out.device)), "zt_lora_add3")
    return out


def lora_split(a: torch.Tensor) -> torch.Tensor:
    """[3, *a.shape] bf16 parts of the fp32 tensor a that sum to it exactly (zt_lora_split):
    bf16(a), bf16(a - p0), bf16(a - p0 - p1)."""
    _check_cuda(a, "a")
    if a.dtype != torch.float32 or not a.is_contiguous():
        raise ValueError("a must be a contiguous fp32 tensor")
    out = torch.empty((3, *a.shape), dtype=torch.bfloat16, device=a.device)
    with torch.cuda.device(a.device):
        L.check(L.load().zt_lora_split(a.data_ptr(), out.data_ptr(), a.numel(), _stream_ptr(a.device)), "zt_lora_split")
    return out


# ---- low-rank directions (distribution "low_rank") -----------------------------------

_LR_DTYPES = {torch.bfloat16: L.ZT_BF16, torch.float16: L.ZT_F16, torch.float32: L.ZT_F32}


def lowrank_supported(p: torch.Tensor) -> bool:
    """Whether zt_lowrank_* take this parameter: a contiguous 2-D bf16, f16 or fp32 CUDA
    tensor at an address aligned to its element size."""
    return (p.is_cuda and p.dim() == 2 and p.dtype in _LR_DTYPES and p.is_contiguous()
            and p.data_ptr() % p.element_size() == 0 and p.numel() > 0)


def _split3(x: torch.Tensor) -> list:
    """The exact three-way bf16 split of an fp32 tensor: x = hi + mid + lo."""
    hi = x.bfloat16()
    r1 = x - hi.float()
    mid = r1.bfloat16()
    lo = (r1 - mid.float()).bfloat16()
    return [hi, mid, lo]


class LowRankFactors:
    """The low-rank directions of one 2-D parameter for up to ZT_LOWRANK_MAX_STREAMS pair
    seeds, prepared on the device (zt_lowrank_prepare): P and Psi^T of every seed in
    K-major buffers padded to a multiple of 64, and each seed's rounded scale. The
    direction z itself is never stored; `apply` recomputes it tile by tile.

    keys_p / keys_psi are the noise keys of P and Psi (positions i + 2N and i + N of the
    reference's _sample_z, zotitan/train_zo.py:311-315)."""

    def __init__(self, shape, r: int, dtype: torch.dtype, keys_p, keys_psi, device, _given=None):
        m, n = int(shape[0]), int(shape[1])
        S = len(keys_p)
        if not 1 <= S <= L.ZT_LOWRANK_MAX_STREAMS or len(keys_psi) != S:
            raise ValueError(f"1..{L.ZT_LOWRANK_MAX_STREAMS} streams with one P and one Psi key each")
        if dtype not in _LR_DTYPES:
            raise ValueError("low-rank directions take bf16, f16 or fp32 parameters")
        # fp32: nine blocks of r along K (the cross products of the three-way bf16 splits)
        width = 9 * r if dtype == torch.float32 else r
        kp = 64 * ((width + 63) // 64)
        op = torch.float16 if dtype == torch.float16 else torch.bfloat16
        self.shape, self.r, self.kp, self.dtype, self.n_streams = (m, n), r, kp, dtype, S
        if _given is None:
            self.p = torch.empty((S * m, kp), dtype=op, device=device)
            self.psi_t = torch.empty((S * n, kp), dtype=op, device=device)
        else:
            self.p, self.psi_t = _given
        self.scale = torch.empty(S, dtype=torch.float32, device=device)
        lib = L.load()
        ws = ctypes.c_size_t()
        L.check(lib.zt_lowrank_workspace_bytes(m, n, S, ctypes.byref(ws)), "zt_lowrank_workspace_bytes")
        self._ws = torch.empty(max(16, ws.value), dtype=torch.uint8, device=device)
        d = L.ZtLowrankDesc()
        d.m, d.n, d.r, d.kp, d.dtype, d.n_streams = m, n, r, kp, _LR_DTYPES[dtype], S
        for s in range(S):
            d.keys_p[s], d.keys_psi[s] = int(keys_p[s]), int(keys_psi[s])
        d.p, d.psi_t, d.scale = self.p.data_ptr(), self.psi_t.data_ptr(), self.scale.data_ptr()
        d.workspace, d.workspace_bytes = self._ws.data_ptr(), self._ws.numel()
        d.factors_given = 1 if _given is not None else 0
        self.desc = d
        self.device = torch.device(device)
        with torch.cuda.device(self.device):
            L.check(lib.zt_lowrank_prepare(ctypes.byref(d), _stream_ptr(self.device)), "zt_lowrank_prepare")

    @classmethod
    def from_factors(cls, shape, Ps: list, Psis: list, dtype: torch.dtype) -> "LowRankFactors":
        """Directions from factors computed by the caller (the polar distribution: P after
        QR, Psi after the Newton-Schulz iteration, zotitan/train_zo.py:307-317), one
        (P [m, r], Psi [r, n]) per stream, in the parameter dtype. Only the product, its
        norm and its uses run here."""
        m, n = int(shape[0]), int(shape[1])
        S, r = len(Ps), int(Ps[0].shape[1])
        dev = Ps[0].device
        width = 9 * r if dtype == torch.float32 else r
        kp = 64 * ((width + 63) // 64)
        op = torch.float16 if dtype == torch.float16 else torch.bfloat16
        A = torch.zeros((S * m, kp), dtype=op, device=dev)
        B = torch.zeros((S * n, kp), dtype=op, device=dev)
        for s, (P, Psi) in enumerate(zip(Ps, Psis)):
            P, Psi = P.to(dtype), Psi.to(dtype)
            if dtype == torch.float32:
                ps, qs = _split3(P), _split3(Psi.t())
                for blk in range(9):
                    A[s * m:(s + 1) * m, blk * r:(blk + 1) * r] = ps[blk // 3]
                    B[s * n:(s + 1) * n, blk * r:(blk + 1) * r] = qs[blk % 3]
            else:
                A[s * m:(s + 1) * m, :r] = P
                B[s * n:(s + 1) * n, :r] = Psi.t()
        return cls(shape, r, dtype, [0] * S, [0] * S, dev, _given=(A, B))

    def apply(self, src: torch.Tensor | None = None, dst: torch.Tensor | None = None, alphas=(), ge=None, coefs=None,
              ge_init: bool = False, test_stall_loads: bool = False, test_wait_cycles: int = 0) -> None:
        """For each stream in order: dst <- round(dst + a z) for each a in `alphas` (stream
        0 reads src), ge <- round(ge + coef z) (ge = round(coef z) for stream 0 with
        ge_init)."""
        for t, name in ((src, "src"), (dst, "dst"), (ge, "ge")):
            if t is not None:
                _check_cuda(t, name)
                if tuple(t.shape) != self.shape or t.dtype != self.dtype or not t.is_contiguous():
                    raise ValueError(f"{name} must be a contiguous {self.dtype} tensor of shape {self.shape}")
        if len(alphas) > 3:
            raise ValueError("at most 3 chained coefficients")
        a = L.ZtLowrankApplyArgs()
        a.src = src.data_ptr() if src is not None else None
        a.dst = dst.data_ptr() if dst is not None else None
        a.ge = ge.data_ptr() if ge is not None else None
        a.n_alpha = len(alphas)
        for t, v in enumerate(alphas):
            a.alpha[t] = float(np.float32(v))
        a.ge_init = 1 if ge_init else 0
        if coefs is not None:
            if len(coefs) != self.n_streams:
                raise ValueError("one grad-estimate coefficient per stream")
            for s, v in enumerate(coefs):
                a.coef[s] = float(np.float32(v))
        a.test_stall_loads = 1 if test_stall_loads else 0
        a.test_wait_cycles = int(test_wait_cycles)
        with torch.cuda.device(self.device):
            L.check(L.load().zt_lowrank_apply(ctypes.byref(self.desc), ctypes.byref(a), _stream_ptr(self.device)),
                    "zt_lowrank_apply")

    def directions(self) -> torch.Tensor:
        """The scaled directions [S, m, n] (test use: writes them into a zero tensor)."""
        S, (m, n) = self.n_streams, self.shape
        out = torch.empty((S, m, n), dtype=self.dtype, device=self.device)
        zero = torch.zeros((m, n), dtype=self.dtype, device=self.device)
        for s in range(S):
            one = LowRankFactors.__new__(LowRankFactors)
            one.__dict__.update(self.__dict__)
            d = L.ZtLowrankDesc()
            ctypes.pointer(d)[0] = self.desc
            esz = self.p.element_size()
            d.n_streams = 1
            d.factors_given = 1
            d.keys_p[0], d.keys_psi[0] = self.desc.keys_p[s], self.desc.keys_psi[s]
            d.p = self.p.data_ptr() + s * m * self.kp * esz
            d.psi_t = self.psi_t.data_ptr() + s * n * self.kp * esz
            d.scale = self.scale.data_ptr() + 4 * s
            one.desc, one.n_streams = d, 1
            one.apply(src=zero, dst=out[s], alphas=(1.0,))
        return out


def lowrank_take_error() -> int:
    code = ctypes.c_int32(0)
    L.check(L.load().zt_lowrank_take_error(ctypes.byref(code)), "zt_lowrank_take_error")
    return int(code.value)
