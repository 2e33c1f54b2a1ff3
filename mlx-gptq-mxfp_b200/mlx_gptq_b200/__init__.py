"""B200-native GPTQ calibration engine (Stage A of mlx_gptq, sm_100a).

Host side of the C ABI in include/gptq_b200.h: the reference's Python surface
(``solve_gptq``, ``gptq_quantize``, grid functions, packing, ``Stash.hessian``,
the artifact store) backed by hand-written CUDA kernels in libgptq_b200.so.
"""

from . import _lib  # noqa: F401
from .capture import Stash, hessian_accumulate, hessian_from_rows, hessian_grouped  # noqa: F401
from .gptq import gptq_quantize, solve_gptq  # noqa: F401

__all__ = ["solve_gptq", "gptq_quantize", "Stash", "hessian_accumulate", "hessian_from_rows"]
