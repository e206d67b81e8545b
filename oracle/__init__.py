"""CPU oracle for the GEMM hot path - TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference's own correctness path for
C = A @ B^T (jamesbowley/gfx950-gluon-tutorials):
  - a16w16: torch.matmul in the input dtype
    (kernels/gemm/intra_wave/a16w16/bench.py:167-187)
  - a8w8:   torch.matmul(a.to(fp16), b.to(fp16)) on e5m2 inputs
    (kernels/gemm/intra_wave/a8w8/bench.py:129-142)
  - a4w4:   dequantise with mxfp4_to_f32 / e8m0_to_f32, fp32 mm, cast to bf16
    (kernels/gemm/intra_wave/a4w4/bench.py:80-164)
plus the quantisers the B200 build adds (MXFP4 per the OCP MX rule, scaled
e5m2) and torch's float -> float8_e5m2 rounding.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import
it, and only as a checker or as the timed CPU baseline. The product path
(gfx950_gluon_tutorials_b200) never calls into it.

Pinning: mx.py is checked against golden vectors produced by running the
reference's own functions (AST-extracted from its bench.py, see
tests/golden/make_golden.py) and torch's e5m2 cast in this container; the
vectors are committed under tests/golden/.
"""
