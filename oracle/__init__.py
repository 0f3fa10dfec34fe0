"""Oracle: CPU restatement of the reference's zeroth-order hot path.

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may import anything under ``oracle/``, and only
as the checker (or as the timed CPU baseline), never as the thing measured or
shipped. The product package ``zotitan_b200`` never imports it and has no CPU
fallback: when its CUDA library is missing it raises.

Contents
  philox_oracle.c / philox.py  Philox4x32-10 words, uniforms, Box-Muller Gaussians and
                               the per-element perturb / restore / update chains in
                               plain C (fmaf, bf16 round-to-nearest-even), called via ctypes.
  zo_step.py                   the optimizer step (seeds, clipping, fitness shaping,
                               momentum, weight decay) driven by the C chains.
  triton_native.py             the reference's Triton noise kernel shape, run natively on
                               a GPU to pin the device lowering of log/cos/sqrt.

Pinning: the C restatement is checked bit-exact against golden vectors produced by
running the reference's own code in the build container (tests/golden/make_golden.py,
Triton interpreter), and its Gaussians against native-Triton vectors generated on a
B200 (tests/golden/make_native_triton.py).
"""
