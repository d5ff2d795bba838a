"""B200 (sm_100a) implementation of the INT8 hybrid MoE forward path of
PatchouliTIS/INT8BlockwiseGEMM.

Importing the package loads libi8moe.so (``INT8_HYBRID_MOE_LIB`` overrides
the in-tree path) and registers the reference's operator namespace
``torch.ops.int8_hybrid_moe``.  The Python modules mirror the reference's
``int8_hybrid_moe`` package: ``ops``, ``permute``, ``quant``, ``activation``
and ``cutlass_runner``.
"""

from . import _lib  # noqa: F401  (loads the shared library, raises if missing)
from . import _ops

_ops.register()

from . import activation, cutlass_runner, ops, permute, quant  # noqa: E402,F401

__all__ = ["activation", "cutlass_runner", "ops", "permute", "quant"]
