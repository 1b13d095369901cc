"""CPU oracle for the NVFP4-weight / BF16-activation MoE layer — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the arithmetic of xCalibur's ``kernels/moe_w4a16_h200`` operator and of the
north_star layer built on it.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline
and reference arms) may import it, and only as the checker or the timed CPU baseline; the product package
``xcalibur_b200`` never calls into it.

Parity status
-------------
* The layer as a whole is **unpinned** at its boundary: the reference repository ships no torch reference of
  the layer and no golden layer vectors (its operator was checked by an external harness that is not
  available).  The layer restatement here follows kernels/moe_w4a16_h200/moe_w4a16.py:8-33 (algorithm),
  :616-657 (epilogues: SwiGLU rounded to bf16, fp32 down projection), :2654-2796 (final weighted sum,
  eps 1e-8, mean over H) and kernels/moe_w4a16_h200/README.md:10-19.
* Pinned pieces: the GF(2) machinery against the reference's own test vectors (tests/test_core.py:6-20), and
  the FP4/FP8 dequantisation bit semantics against outputs of the reference's own packers and decoder,
  generated in a container that has the reference (``tests/golden/make_golden.py``), committed as fixtures.
"""
