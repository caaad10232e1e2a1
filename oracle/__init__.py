"""CPU oracle of the hot path: a restatement of the reference's algorithms in numpy and C.

TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / reference legs may import, call or link anything in this package, and
only as the checker or the timed CPU baseline -- never as the thing measured or shipped.
The product (hsd_b200, libhsd.so) has no CPU path and never imports this package.

Pinning (what each part was checked against):
  layout   outputs of the reference's own hsd/layout.py:34-74 and of its test's
           known-answer transpose (tests/test_layout_decode.py:38-52), run unmodified on a
           numpy stand-in of mlx.core (tests/golden/make_reference_golden.py ->
           tests/golden/reference_layout.npz); also the known-answer test restated in
           tests/test_oracle.py (exactness, self-inverse, the reference test's shapes).
  decode   the reference test's fp32 dequantised reference (tests/test_layout_decode.py
           :128-142) and, independently, the Metal kernel's per-group affine algebra
           (hsd/decode.py:105-144); the two restatements must agree. That test reference
           itself, run unmodified on the numpy stand-in of mlx.core, produced
           tests/golden/reference_down.npz; the oracle reproduces it to 1e-5 once the
           dequantised weights are rounded to bf16 as mx.dequantize returns them. The
           Metal kernels' own outputs do not exist offline (MLX needs Apple silicon).
  prefill  tile order: outputs of the reference's own hsd/prefill.py:247-278 on seeded
           routings, run the same way (tests/golden/reference_tiles.npz); union, gain
           epilogue and partial sum restated from hsd/prefill.py:48-222,281-321 (Metal).
  mamba    fixtures made with transformers' NemotronHMamba2Mixer (an independent
           implementation of the same layer), tests/golden/make_mamba_golden.py.
"""
