"""B200 (sm_100a) backend for tinygrad-dx12's packed low-bit matmul path.

Importing the package registers the backend without opening hardware, as
``import tinygrad_dx12`` does (tinygrad-dx12 ``src/tinygrad_dx12/__init__.py:8-10``).
"""

from .compat import register as register
from .packed import FORMATS, FP8_CANDIDATES, PackedTensor, matrix_intermediate
from .linalg import Estimates, choose_matrix, estimates, matmul, matvec, set_profile_hook
from .graph import GraphStep

register()

__all__ = ["register", "FORMATS", "FP8_CANDIDATES", "PackedTensor", "matrix_intermediate", "matmul", "matvec",
           "choose_matrix", "Estimates", "estimates", "set_profile_hook", "GraphStep"]
