"""CPU oracle of the hot path: a restatement of the reference's algorithms in numpy and C.

TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / reference legs may import, call or link anything in this package, and
only as the checker or the timed CPU baseline -- never as the thing measured or shipped.
The product (hsd_b200, libhsd.so) has no CPU path and never imports this package.

Pinning (what each part was checked against):
  layout   the reference's own known-answer test (tests/test_layout_decode.py:38-67 of
           the reference: a slow per-nibble numpy unpack / move / pack, exactness and
           self-inverse) restated in tests/test_oracle.py and the fixture in tests/golden/.
  decode   the reference test's fp32 dequantised reference (tests/test_layout_decode.py
           :128-142) and, independently, the Metal kernel's per-group affine algebra
           (hsd/decode.py:105-144); the two restatements must agree. No output of the
           reference itself exists offline (MLX needs Apple silicon), so the decode
           oracle is pinned by algebra only.
  prefill  hsd/prefill.py:247-321 (tile order, union, gain epilogue, partial sum).
  mamba    fixtures made with transformers' NemotronHMamba2Mixer (an independent
           implementation of the same layer), tests/golden/make_mamba_golden.py.
"""
