"""lastro_moe_block_forward_noalloc against lastro_layer_forward, through the C ABI.

The allocation-free entry point has no counterpart in the reference; its output must match the existing block
forward (itself checked against the oracle in test_gpu_block.py) within that file's gate, on two calls in a row that
share the file-scope scratch.  Named so that pytest collects it last: it passes alone in a fresh process and after
every other test.
"""
import numpy as np
import pytest

import lastro_b200 as LB
from helpers import rel_l2, synthetic_layer, values

pytestmark = pytest.mark.gpu

REL = 1e-5  # the block gate of test_gpu_block.py (f32 arithmetic)


def _dev(a, torch):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a).to("cuda:0")


@pytest.mark.parametrize("E,H,I,k", [(4, 256, 128, 2), (32, 1024, 512, 8), (40, 1536, 512, 8)])
def test_noalloc_matches_layer_forward(gpu_ctx, E, H, I, k):
    import torch
    router, gu, dn = synthetic_layer(E, H, I)
    layer = LB.GpuLayer(gpu_ctx, router, gu, dn, k)
    torch.cuda.set_device(0)
    d_router, d_gu, d_dn = _dev(router, torch), _dev(gu, torch), _dev(dn, torch)
    y = torch.empty(H, dtype=torch.float32, device="cuda:0")
    ids = torch.empty(k, dtype=torch.int32, device="cuda:0")
    w = torch.empty(k, dtype=torch.float32, device="cuda:0")
    stream = torch.cuda.current_stream()
    for t in range(2):  # two calls in a row: the second reuses the scratch the first left behind
        x = values(H, 300 + t)
        d_x = _dev(x, torch)
        rc = LB.moe_block_forward_noalloc(d_x.data_ptr(), d_router.data_ptr(), d_gu.data_ptr(), d_dn.data_ptr(),
                                          E, H, I, k, y.data_ptr(), ids.data_ptr(), w.data_ptr(), stream.cuda_stream)
        assert rc == LB.OK, rc
        stream.synchronize()
        want_y, want_ids, want_w, _ = layer.forward(x)
        assert ids.cpu().numpy().tolist() == want_ids.tolist(), f"call {t}"
        np.testing.assert_allclose(w.cpu().numpy(), want_w, rtol=2e-6, atol=1e-7)
        assert rel_l2(y.cpu().numpy(), want_y) < REL, f"call {t}"
        # every bounded copy wait of the call completed: the error word the status call copies out is 0
        status = torch.full((1,), -1, dtype=torch.int32, device="cuda:0")
        assert LB.moe_block_noalloc_status(status.data_ptr(), stream.cuda_stream) == LB.OK
        stream.synchronize()
        assert int(status.item()) == 0, f"call {t}"
    layer.close()


def test_noalloc_refuses_shapes_beyond_its_scratch():
    import torch
    torch.cuda.set_device(0)
    buf = torch.zeros(8, dtype=torch.float32, device="cuda:0")
    p = buf.data_ptr()
    # 65 experts exceed the logits slots; k * I above 8 * 2048 = 16384 floats exceeds the activation scratch
    assert LB.moe_block_forward_noalloc(p, p, p, p, 65, 256, 128, 8, p, p, p, None) == LB.E_UNSUPPORTED
    assert LB.moe_block_forward_noalloc(p, p, p, p, 8, 256, 2056, 8, p, p, p, None) == LB.E_UNSUPPORTED
    assert LB.moe_block_forward_noalloc(p, p, p, p, 16, 256, 2048, 9, p, p, p, None) == LB.E_UNSUPPORTED
    assert LB.moe_block_forward_noalloc(0, p, p, p, 8, 256, 128, 2, p, p, p, None) == LB.E_ARG
    assert LB.moe_block_noalloc_status(0, None) == LB.E_ARG
