"""MoE block (GpuLayer) on the GPU through the C ABI, checked against the CPU oracle and naive f64.

Restates rust/moe-rt/tests/block.rs:268-366 (block vs f64, fused expert kernels at the real (H, I)) and
rust/moe-rt/src/route.rs:130-269 (router top-k on eight logit families, E = 32 and 40, padding mask).
"""
import numpy as np
import pytest

import lastro_b200 as LB
import oracle as O
import synth_np as S
from helpers import exact_logit_router, naive_block, rel_l2, synthetic_layer, values
from test_oracle import FAMILIES, family_logits, reference_topk

pytestmark = pytest.mark.gpu

# gate of tests/block.rs:280, 296, 351 (f32 arithmetic, different summation order)
REL = 1e-5


@pytest.mark.parametrize("E,H,I,k", [(4, 256, 128, 2), (4, 768, 128, 2), (32, 1024, 512, 8), (40, 1536, 512, 8),
                                     (4, 256, 768, 2), (6, 24, 16, 2)])
def test_block_on_gpu_matches_oracle_and_f64(gpu_ctx, pool, E, H, I, k):
    router, gu, dn = synthetic_layer(E, H, I)
    layer = LB.GpuLayer(gpu_ctx, router, gu, dn, k)
    for t in range(4):
        x = values(H, 200 + t)
        y, ids, w, lg = layer.forward(x)
        yo, io, wo, lo = O.block_forward(pool, router, gu, dn, E, H, I, k, x)
        want, wids = naive_block(router, gu, dn, x, k)
        assert ids.tolist() == wids.tolist() == io.tolist(), f"token {t}"
        # the kernel's softmax over its own top-k logits (block.rs:85-88) ...
        ex = np.exp((lg[ids] - lg[ids[0]]).astype(np.float32))
        np.testing.assert_allclose(w, ex / ex.sum(), rtol=2e-6, atol=1e-7)
        # ... and against the oracle: logits differ by summation order (~1e-6 relative), which the softmax scales
        # by the logit magnitude
        np.testing.assert_allclose(lg, lo, rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(w, wo, rtol=1e-3, atol=1e-6)
        assert rel_l2(y, want) < REL, f"token {t}: {rel_l2(y, want):.2e}"
        assert rel_l2(y, yo) < REL
    layer.close()


def test_block_c1_golden(gpu_ctx):
    """BASELINE config 0 against transformers (tests/golden/block_c1.npz)."""
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "block_c1.npz"))
    from test_golden import c1_weights
    router, gu, dn = c1_weights()
    layer = LB.GpuLayer(gpu_ctx, router, gu, dn, 8)
    for t in range(g["x"].shape[0]):
        y, ids, w, lg = layer.forward(g["x"][t])
        assert ids.tolist() == g["idx"][t].tolist()
        np.testing.assert_allclose(w, g["w"][t], rtol=1e-5, atol=1e-7)
        assert rel_l2(y, g["y"][t]) < REL
    layer.close()


@pytest.mark.parametrize("E", [32, 40])
def test_router_top_k_on_all_logit_families(gpu_ctx, E):
    """route.rs:212-227: ids identical to the host's sort for every family; the padded tail (E = 40 of a 64-wide
    selection) never wins, even when every logit is negative (route.rs:261-269)."""
    H, I, k = 256, 16, 8
    state = [7]
    bad = {}
    for kind in FAMILIES:
        for _ in range(10):
            v = family_logits(kind, E, state)
            rw, x = exact_logit_router(v, H)
            gu = np.zeros((E, 2 * I, H), np.uint16)
            dn = np.zeros((E, H, I), np.uint16)
            layer = LB.GpuLayer(gpu_ctx, rw, gu, dn, k)
            _, ids, w, lg = layer.forward(x)
            layer.close()
            assert np.array_equal(lg, v), kind
            if ids.tolist() != reference_topk(v, k):
                bad[kind] = bad.get(kind, 0) + 1
            top = v[ids[0]]
            ex = np.exp((v[ids] - top).astype(np.float32))
            np.testing.assert_allclose(w, ex / ex.sum(), rtol=2e-6, atol=1e-7)
    assert not bad, bad


def test_add_into_accumulates_into_device_residual(gpu_ctx, pool):
    """GpuLayer::add_into (gpu.rs:480-505): h <- h + resid * moe(xn) on device buffers."""
    torch = pytest.importorskip("torch")
    E, H, I, k = 8, 512, 128, 4
    router, gu, dn = synthetic_layer(E, H, I)
    layer = LB.GpuLayer(gpu_ctx, router, gu, dn, k)
    x = values(H, 31)
    h0 = values(H, 32)
    xd = torch.from_numpy(x).cuda()
    hd = torch.from_numpy(h0).cuda()
    ids = torch.zeros(k, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    layer.add_into(xd.data_ptr(), hd.data_ptr(), 0.22, ids.data_ptr(), None)
    gpu_ctx.synchronize()
    y, io, _, _ = O.block_forward(pool, router, gu, dn, E, H, I, k, x)
    want = h0 + np.float32(0.22) * y
    assert rel_l2(hd.cpu().numpy(), want) < REL
    assert ids.cpu().numpy().tolist() == io.tolist()
    layer.close()


def test_shape_refusals_leave_the_context_usable(gpu_ctx):
    """Shape errors are refused before any launch (gpu.rs:406-410 asserts; here status codes)."""
    r = np.zeros((4, 20), np.uint16)
    with pytest.raises(LB.LastroError) as e:
        LB.GpuLayer(gpu_ctx, r, np.zeros((4, 16, 20), np.uint16), np.zeros((4, 20, 8), np.uint16), 2)
    assert e.value.code == LB.E_UNSUPPORTED
    with pytest.raises(LB.LastroError) as e:
        LB.GpuLayer(gpu_ctx, np.zeros((4, 64), np.uint16), np.zeros((4, 32, 64), np.uint16),
                    np.zeros((4, 64, 16), np.uint16), 5)
    assert e.value.code == LB.E_ARG
    router, gu, dn = synthetic_layer(4, 64, 16)
    layer = LB.GpuLayer(gpu_ctx, router, gu, dn, 2)
    y, ids, _, _ = layer.forward(values(64, 5))
    assert np.isfinite(y).all() and len(set(ids.tolist())) == 2
    layer.close()
