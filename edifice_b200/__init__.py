"""edifice_b200 -- B200 (sm_100a) kernels for Edifice's fused sequence-mixing path.

The product is libedifice_b200.so (C ABI: include/edifice_b200.h) plus the two
reference-named shim libraries (include/edifice_cuda_kernels.h).  This Python
package is the host-side mirror of ``Edifice.CUDA.FusedScan`` over torch CUDA
tensors; it has no CPU path.
"""
from ._lib import EdbError, LIB_PATH, load, device_errors  # noqa: F401
from . import fused_scan  # noqa: F401
from .fused_scan import (  # noqa: F401
    linear_scan, linear_scan_backward, mingru, mingru_scan, mingru_backward,
    LinearScanFn, MinGRUFn, selective_scan, selective_scan_backward, SelectiveScanFn,
    flash_attention, flash_attention_backward, FlashAttentionFn,
    delta_net_scan, delta_rule_backward, DeltaNetFn,
)

__version__ = "0.1.0"
