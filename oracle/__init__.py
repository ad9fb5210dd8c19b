"""CPU oracle for the MLX-affine quantized-matmul path (test infrastructure).

Two independent restatements of MLX's affine semantics live here:
  - nq_oracle.c   (C; bit-exact quantize/dequantize, fp64-accumulated qmm),
    driven through oracle.py (ctypes);
  - np_oracle.py  (numpy; vectorised, used to cross-check the C restatement).
Neither is importable from the product package.
"""
