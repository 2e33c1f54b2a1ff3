"""CPU oracle for the GPTQ calibration hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy float32, the reference's algorithm for the path
(mlx_gptq/capture.py Stash.hessian, mlx_gptq/gptq.py, mlx_gptq/grid.py,
mlx_gptq/packing.py, mlx_gptq/artifacts.py nibble packing). Every function cites
the reference file:line it follows.

It is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference`` arm) may import
it. The CUDA library under ``mlx-gptq-mxfp_b200/`` never routes through it.

Parity pin: the oracle is checked against golden vectors produced by the real
reference (imported read-only in the development container) and committed under
``tests/golden/`` together with the script that made them.
"""

from . import grid, gptq, hessian, packing  # noqa: F401
