"""TEST INFRASTRUCTURE ONLY: the CPU oracle for the routed-expert MoE path.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import anything here, and only as the
checker or the timed CPU baseline, never as the thing measured or shipped. The product (comfyui-drama3_b200/) never
imports this package.

  oracle.moe      numpy restatement of the reference's arithmetic (PedroMarinhoDev/ComfyUI-Drama3, drama3/kernels.py,
                  drama3/offload.py, drama3/model.py), citing the lines each function follows. Pinned against golden
                  vectors produced by the reference's own Python CPU functions (tests/golden/make_golden.py).
  oracle.build_ref / oracle.ref_gpu
                  the reference's own CUDA kernels, compiled here from the reference source into oracle/_ref/ (never
                  committed) and launched on a GPU through the driver API: the bit-exact pin for the GPU-only pieces
                  (decode routing, slot resolve) and the reference GPU timing.
"""
