"""macrograd_b200 -- B200-native (sm_100a) replacement for the matmul hot path
of Macrograd: Functional::matmul, its bias form, and the two gradient GEMMs of
its backward, on tcgen05 tensor cores in fp32-accurate 3xTF32 (default) or
TF32 mode. The C ABI is include/mg_gemm.h; this package is its Python host
mirror (functional.py: matmul, its backward, the fused attention-score
softmax and its backward, strided-view GEMMs), the row-sharded multi-GPU layer
(sharded.py), the data-parallel training step over the drop-in build
(training.py) and the build script (build.py).
"""
from ._lib import MacrogradError, load, lib_path  # noqa: F401
from .functional import (attention_scores, attention_softmax_backward, matmul, matmul_backward,  # noqa: F401
                         matmul_view)

__all__ = ["MacrogradError", "load", "lib_path", "matmul", "matmul_backward", "matmul_view",
           "attention_scores", "attention_softmax_backward"]
