"""Generate ``native_triton_randn.npz``: the reference's noise kernel run natively.

Runs Triton's ``tl.random.randint4x`` / ``tl.random.randn`` (the calls behind
zotitan/train_zo.py:18-28) on a CUDA GPU, in the reference's launch shape, for a
fixed set of keys and offsets, and writes words + Gaussians. Needs a GPU and
Triton; the output is committed so the GPU tests do not depend on Triton.

    python tests/golden/make_native_triton.py OUT.npz
"""
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", ".."))
from oracle import triton_native as tn  # noqa: E402

KEYS = [0, 1, 7, 1234, 2**31 - 1, 987654321]


def offsets_for(key: int) -> np.ndarray:
    rng = np.random.default_rng(key % (2**32))
    head = np.arange(0, 2048, dtype=np.int64)
    rand = rng.integers(0, 2**31 - 1, 2048, dtype=np.int64)
    edge = np.arange(2**31 - 64, 2**31, dtype=np.int64)
    return np.concatenate([head, rand, edge]).astype(np.int32)


def main(path: str) -> None:
    rec = {"keys": np.array(KEYS, dtype=np.int64)}
    for key in KEYS:
        offs = offsets_for(key)
        t = torch.from_numpy(offs).cuda()
        rec[f"offs_{key}"] = offs
        rec[f"words_{key}"] = tn.words_at(key, t).cpu().numpy().view(np.uint32)
        rec[f"randn_{key}"] = tn.randn_at(key, t).cpu().numpy()
    # the reference's own launch shape: _philox_randn(seed, n) over offsets 0..n-1
    rec["refshape_key"] = np.array(1234)
    rec["refshape_randn"] = tn.randn_ref_shape(1234, 5000).cpu().numpy()
    rec["triton_version"] = np.array(__import__("triton").__version__)
    rec["device"] = np.array(torch.cuda.get_device_name(0))
    np.savez_compressed(path, **rec)
    print("wrote", path)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "native_triton_randn.npz")
