"""flash-mHC for B200: the mHC-lite hot path as hand-written sm_100a CUDA kernels.

Drop-in for alint77/flash-mHC: the same ``torch.ops.flash_mhc`` ops (schemas,
fakes, autograd) and the same ``MHCLiteBlock`` / ``build_permutation_matrices``
API.  The kernels live in ``libflashmhc_sm100.so`` (C ABI: include/flashmhc.h).
"""

from .block import MHCLiteBlock, build_permutation_matrices
from . import ops as _ops  # registers the torch.library custom ops

__all__ = ["MHCLiteBlock", "build_permutation_matrices"]
__version__ = "0.1.0"
