"""d3_moe_decode_static: the fused decode for callers that cannot allocate device memory themselves (a host whose
memory manager owns every device allocation, or a C host without a device allocator). It takes no workspace and
uses a scratch array held inside the library. Checked through the C ABI against d3_moe_decode with a workspace, on
two calls in a row (the shared array keeps the first call's contents). Collected last on purpose: the library-held
array stays allocated on the device for the rest of the process."""
import pytest
import torch

import gpu_data as gd

pytestmark = pytest.mark.gpu

E, H, I, K = 128, 2048, 768, 8
TOL = 1e-3


def _call_static(lib, kind, x, ids, w, banks, cbs, out):
    from drama3_b200 import _lib
    gate_up, down = banks
    wkey = gd.WKEY[kind]
    ptr = lambda t: None if t is None else t.data_ptr()
    s13 = gate_up["scale"].view(torch.uint8) if kind in ("w4", "w6") else gate_up["scale"]
    s2 = down["scale"].view(torch.uint8) if kind in ("w4", "w6") else down["scale"]
    return lib.d3_moe_decode_static(_lib.FORMATS[kind], ptr(x), int(x.dtype == torch.bfloat16), x.shape[0],
                                    ids.shape[1], E, H, I, ptr(ids), ptr(w), ptr(gate_up[wkey]), ptr(s13),
                                    ptr(gate_up.get("s_channel")), ptr(down[wkey]), ptr(s2),
                                    ptr(down.get("s_channel")), ptr(cbs[0]), ptr(cbs[1]), ptr(out),
                                    torch.cuda.current_stream().cuda_stream)


# fp8 and w4 run the mma.sync decode; fp8c and w4a8 the tensor-core decodes, whose per-segment counters live in the
# same array and are cleared by the kernel at its end (the second call checks they were)
@pytest.mark.parametrize("kind,M", [("fp8", 16), ("w4", 4), ("fp8c", 16), ("w4a8", 16)])
def test_static_scratch_decode_matches_workspace_decode(cuda, kind, M):
    from drama3_b200 import _lib, kernels
    lib = _lib.lib()
    banks = (gd.rand_bank(kind, E, 2 * I, H, 61, cuda), gd.rand_bank(kind, E, H, I, 62, cuda))
    cbs = gd.codebooks(kind, cuda)
    for call in range(2):
        x = gd.rand_rows(M, H, 70 + call, cuda)
        ids, w = gd.rand_routing(M, E, K, 80 + call, cuda)
        expect = kernels.moe_decode(kind, x, ids, w, banks, cbs)
        out = torch.empty_like(expect)
        assert _call_static(lib, kind, x, ids, w, banks, cbs, out) == _lib.D3_OK
        torch.cuda.synchronize()
        assert _lib.take_fault() == 0
        assert gd.rel_l2(out.float(), expect.float()) <= TOL, (kind, M, call)


def test_static_scratch_rejects_shapes_beyond_its_size(cuda):
    from drama3_b200 import _lib
    lib = _lib.lib()
    args = [0, 16, 1, 17, 8, E, H, I] + [16] * 11 + [None]  # 17 x 8 = 136 routed pairs > 128
    assert lib.d3_moe_decode_static(*args) == _lib.D3_ERR_TOO_LARGE
    args = [0, 16, 1, 1, 8, E, H, 1024] + [16] * 11 + [None]  # intermediate 1024 > 768
    assert lib.d3_moe_decode_static(*args) == _lib.D3_ERR_TOO_LARGE
    args = [0, 16, 1, 1, 8, E, 1024, I] + [16] * 11 + [None]  # hidden 1024: a bad argument, not a size limit
    assert lib.d3_moe_decode_static(*args) == _lib.D3_ERR_ARG
