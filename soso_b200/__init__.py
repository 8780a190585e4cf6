"""soso_b200 -- B200-native (sm_100a) quantized decode hot path of soso-llm-core.

The kernels live in libsosob200.so (csrc/, C ABI in include/sosob200.h).  This
package is the host-side mirror of the reference's operator boundary
(`trait GpuDispatch`, crates/soso-llm-core/src/gpu.rs:338-737) plus the device
pointer kernel API used by the decode engine and the benchmarks.
"""
from .formats import DTYPE_F32, DTYPE_Q4_K, DTYPE_Q6_K, DTYPE_Q8_0, row_bytes  # noqa: F401

__all__ = ["DTYPE_F32", "DTYPE_Q8_0", "DTYPE_Q4_K", "DTYPE_Q6_K", "row_bytes"]
