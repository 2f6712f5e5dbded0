"""CPU oracle for the QuIP W8A8 quantized-linear path.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this
module; only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline``
leg / ``--impl reference`` arm of ``bench.py`` may use it, and only as the
checker or as the timed CPU baseline -- never as the thing measured on the GPU.

The oracle is a numpy restatement of the reference's torch CPU algorithm
(ThunderFun/convert_to_quant_QuIP_INT8 v0.8.2).  Each function cites the
reference file:line it restates.  Parity of the restatement is pinned by the
golden vectors under ``tests/golden/``, which ``tests/golden/make_golden.py``
produced by importing and running the reference itself (its torch CPU path,
and its Triton kernels under the Triton CPU interpreter).
"""

from .qi8_oracle import *  # noqa: F401,F403
