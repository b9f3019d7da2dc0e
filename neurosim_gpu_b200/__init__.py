"""B200-native dendritic tick for NeuroSim-GPU (sm_100a CUDA behind a C ABI).

Drop-in for the reference's native dendritic runtimes: the same classes,
constructor arguments, ``step`` signature, state tensors and checkpoint
layout, with every inference tick running in ``libneurosim_b200.so``.
"""

from .dynamics import DendriticDynamics, Dynamics
from .native import load_native_extension
from .precision import PRECISIONS, encode_sparse_weights, quantize_dequantize
from .runtime import (NativeDendriticMatrixRuntime, NativeDendriticPELSRuntime, RuntimeStats,
                      validate_emission_threshold)
from .topology import SparseTopology, random_topology

__all__ = [
    "DendriticDynamics", "Dynamics", "NativeDendriticMatrixRuntime",
    "NativeDendriticPELSRuntime", "PRECISIONS", "RuntimeStats", "SparseTopology",
    "encode_sparse_weights", "load_native_extension", "quantize_dequantize",
    "random_topology", "validate_emission_threshold",
]
