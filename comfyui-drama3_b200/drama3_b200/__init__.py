"""drama3_b200: ComfyUI-Drama3's routed-expert MoE path (routing, expert GEMV / grouped GEMM, weighted combine,
expert slot cache) on hand-written sm_100a kernels behind a C ABI (libdrama3_b200.so).

Modules mirror the reference's: `kernels` (drama3/kernels.py), `offload` (drama3/offload.py) and `model` (the MoE
block of drama3/model.py); besides them `ep` (expert parallelism over several GPUs) and `pack` (the converter's
expert packing, tools/convert.py, on the host cores). The library is loaded on first use; there is no fallback
implementation.
"""
__version__ = "0.1.0"
