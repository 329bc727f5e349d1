"""nvfp4_b200: NVFP4 (e2m1 + e4m3 block-16 scales) inference kernels for B200.

Importable as ``nvfp4_b200`` through ``__graft_entry__.load_package()`` (the
directory name is not a Python identifier).

* ``gemv.custom_kernel(a, b, scale_a, scale_b, c)`` - batched block-scaled GEMV,
  the operator of the reference (blackwell_nvfp4_gemv.cu:500-524);
  ``nvfp4_gemv_forward(a, b, sa, sb, c, M, K, L)`` is the reference's own
  binding name and signature over the same kernel.
* ``dual_gemm(a, b1, b2, scale_a, scale_b1, scale_b2, c)`` - silu(a.b1^T)*(a.b2^T).
* ``grouped_gemm(a_list, b_list, scale_a_list, scale_b_list, c_list)``.
* ``skinny_gemm(x, w, scale_x, scale_w, out)`` - decode-batch GEMM (1..64 rows).
* ``quantize(x)`` - fp16 activations to e2m1 codes + blocked e4m3 scales.
"""
from . import _lib, gemm, gemv, inputs, layout, quant, sharded  # noqa: F401
from .quant import quantize  # noqa: F401
from .gemm import dual_gemm, grouped_gemm, skinny_gemm  # noqa: F401
from .gemv import custom_kernel, nvfp4_gemv_forward  # noqa: F401

__all__ = ["custom_kernel", "nvfp4_gemv_forward", "dual_gemm", "grouped_gemm", "skinny_gemm", "quantize", "gemm", "gemv", "inputs", "layout", "quant", "sharded"]
