"""cpu_mamba_b200 -- the cpu-mamba Mamba S6 block on NVIDIA B200 (sm_100a).

Same public API as the reference package (src/cpu_mamba/__init__.py:22-34):
CPUMamba, assert_state_dict_compatible, QuantConfig, QuantizedLinear,
quantize_block, memory_footprint -- plus the scan ops of the reference's
backends (selective_scan for the C++ op, selective_scan_assoc[_chunked] for
the associative scans).  Every op runs in the CUDA library libmamba_b200.so
(C ABI: include/mamba_b200.h); there is no CPU fallback.
"""
from .module import CPUMamba, StepGraph, assert_state_dict_compatible
from .quant import QuantConfig, QuantizedLinear, memory_footprint, quantize_block
from .ops import selective_scan
from .scan_assoc import selective_scan_assoc, selective_scan_assoc_chunked
from .stack import MambaLayer, MambaStack
from . import export, surgery, torch_ops

B200Mamba = CPUMamba

__version__ = "0.4.0+b200"
__all__ = [
    "CPUMamba", "B200Mamba", "StepGraph", "assert_state_dict_compatible", "QuantConfig",
    "QuantizedLinear", "quantize_block", "memory_footprint", "selective_scan",
    "selective_scan_assoc", "selective_scan_assoc_chunked", "MambaLayer", "MambaStack",
    "__version__",
]
