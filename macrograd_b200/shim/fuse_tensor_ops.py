"""Writes the fused drop-in build's copy of the reference's tensor_ops.cpp:

    python fuse_tensor_ops.py <reference tensor_ops.cpp> <output .cpp>

The copy is build output (under _build/, never committed). Three edits,
each the change INTEGRATION.md describes for the reference itself, each
asserted to apply exactly as many times as the reference has such lines:
  1. Functional::matmul's output (both forms) is allocated without MemPool's
     zero fill -- the GEMM overwrites all of it:
         Tensor out(out_shape, A.device(), requires_grad);
     is bracketed by mg_seam_skip_zero_fill(true) / (false);
  2. MatMulOp / MatMulBiasOp::_backward's
         X.internal_gradient() += matmul(...);
     becomes mg_seam_accumulate_matmul(X.internal_gradient(), ...);
  3. MatMulBiasOp::_backward's bias.internal_gradient() += out.gradient();
     becomes mg_seam_accumulate_sum(bias.internal_gradient(), out.gradient());
The declarations come from seam_fused.h, forced in by the Makefile."""
import re
import sys


def main():
    src, dst = sys.argv[1], sys.argv[2]
    text = open(src, encoding="latin-1").read()   # the file is not all UTF-8; bytes pass through unchanged
    alloc = "Tensor out(out_shape, A.device(), requires_grad);"
    n = text.count(alloc)
    if n != 2:
        sys.exit(f"expected 2 matmul output allocations, found {n}")
    text = text.replace(alloc, "mg_seam_skip_zero_fill(true); " + alloc + " mg_seam_skip_zero_fill(false);")
    pat = re.compile(r"\b(mat[01])\.internal_gradient\(\) \+= matmul\(")
    text, n = pat.subn(r"mg_seam_accumulate_matmul(\1.internal_gradient(), ", text)
    if n != 8:
        sys.exit(f"expected 8 gradient GEMM accumulations, found {n}")
    bias = "bias.internal_gradient() += out.gradient();"
    n = text.count(bias)
    if n != 1:
        sys.exit(f"expected 1 bias gradient accumulation, found {n}")
    text = text.replace(bias, "mg_seam_accumulate_sum(bias.internal_gradient(), out.gradient());")
    open(dst, "w", encoding="latin-1").write(text)


if __name__ == "__main__":
    main()
