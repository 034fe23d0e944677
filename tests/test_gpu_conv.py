"""Conv2D forward and backward against the reference's Conv2D
(include/layers/conv2d.h:192-414) run through oracle.ref(), elementwise at
the north-star tolerance with float64 adjudication of the elements that miss
(oracle/fp64.conv2d_*).  Shapes: the reference test's odd sizes, 1x1 and
5x5 kernels, stride 2 with padding 1 (the U-Net's down path), channel counts
whose k*k*IC rows do not fill a tensor-core tile, few output channels or
column rows (the direct CUDA-core paths, stride 1 and 2), and the diffusion
U-Net's first levels and head at 64x64 (batch 32 per GPU).
"""
import numpy as np
import pytest
import torch

import oracle
from neuralsuite_b200 import kernels as nk
from oracle import fp64
from tests._util import close_report

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref():
    if not oracle.ref_available():
        pytest.skip("oracle/_ref/libnsref.so not built (needs the reference sources)")
    o = oracle.ref()
    o.set_threads(16)
    return o


def dev(a):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=torch.float32, device="cuda")


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


CASES = [
    # B, IC, H, W, OC, k, stride, pad
    (2, 3, 9, 7, 4, 3, 1, 1),
    (2, 5, 8, 8, 6, 3, 2, 1),
    (1, 2, 5, 5, 3, 1, 1, 0),
    (3, 4, 11, 13, 8, 5, 1, 2),
    (2, 16, 16, 16, 32, 3, 1, 1),
    (4, 64, 32, 32, 64, 3, 2, 1),
    (2, 3, 64, 64, 64, 3, 1, 1),
    (3, 6, 10, 12, 3, 3, 2, 1),
    (3, 6, 16, 16, 3, 3, 2, 1),
    (2, 5, 12, 8, 2, 1, 1, 0),
    (2, 64, 64, 64, 3, 3, 1, 1),
]


@pytest.mark.parametrize("B,IC,H,W,OC,k,s,p", CASES)
def test_conv2d_matches_reference(cuda, ref, B, IC, H, W, OC, k, s, p):
    r = np.random.default_rng(B * 1000 + IC * 100 + H + OC + k + s)
    x = r.standard_normal((B, IC, H, W)).astype(np.float32)
    w = (r.standard_normal((OC, IC, k, k)) / np.sqrt(IC * k * k)).astype(np.float32)
    b = (r.standard_normal(OC) * 0.1).astype(np.float32)
    OH, OW = (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1
    dy = r.standard_normal((B, OC, OH, OW)).astype(np.float32)
    y_r, dx_r, dw_r, db_r = ref.conv2d(x, w, b, s, p, dy)
    xd, wd = dev(x), dev(w)
    y = host(nk.conv2d_fwd(xd, wd, dev(b), stride=s, pad=p))
    dx, dw, db = (host(t) for t in nk.conv2d_bwd(xd, dev(dy), wd, stride=s, pad=p))
    nk.kernel_health()
    want64 = [fp64.conv2d_fwd(x, w, b, s, p), *fp64.conv2d_bwd(x, w, dy, s, p)]
    for name, got, want, w64 in (("y", y, y_r, want64[0]), ("dx", dx, dx_r, want64[1]),
                                 ("dw", dw, dw_r, want64[2]), ("db", db, db_r, want64[3])):
        ok, info = close_report(got, want, w64)
        assert ok, (name, info)


@pytest.mark.slow
def test_conv2d_unet_first_layer_full_batch(cuda, ref):
    """The diffusion U-Net's widest convolution: 32 images of 64x64 with 64
    channels in and out, 3x3, stride 1, padding 1."""
    B, IC, H, W, OC = 32, 64, 64, 64, 64
    r = np.random.default_rng(55)
    x = r.standard_normal((B, IC, H, W)).astype(np.float32)
    w = (r.standard_normal((OC, IC, 3, 3)) / 24.0).astype(np.float32)
    b = (r.standard_normal(OC) * 0.1).astype(np.float32)
    dy = r.standard_normal((B, OC, H, W)).astype(np.float32)
    y_r, dx_r, dw_r, db_r = ref.conv2d(x, w, b, 1, 1, dy)
    xd, wd = dev(x), dev(w)
    y = host(nk.conv2d_fwd(xd, wd, dev(b), stride=1, pad=1))
    dx, dw, db = (host(t) for t in nk.conv2d_bwd(xd, dev(dy), wd, stride=1, pad=1))
    for name, got, want, fn in (
            ("y", y, y_r, lambda: fp64.conv2d_fwd(x, w, b, 1, 1)),
            ("dx", dx, dx_r, lambda: fp64.conv2d_bwd(x, w, dy, 1, 1)[0]),
            ("dw", dw, dw_r, lambda: fp64.conv2d_bwd(x, w, dy, 1, 1)[1]),
            ("db", db, db_r, lambda: fp64.conv2d_bwd(x, w, dy, 1, 1)[2])):
        ok, info = close_report(got, want)
        if not ok:
            ok, info = close_report(got, want, fn())
        assert ok, (name, info)


def test_conv2d_backward_is_deterministic_and_skips_dx(cuda):
    r = np.random.default_rng(2)
    x = dev(r.standard_normal((8, 16, 32, 32)))
    w = dev(r.standard_normal((32, 16, 3, 3)) * 0.1)
    dy = dev(r.standard_normal((8, 32, 16, 16)))
    a = nk.conv2d_bwd(x, dy, w, stride=2, pad=1)
    b = nk.conv2d_bwd(x, dy, w, stride=2, pad=1)
    for u, v in zip(a, b):
        assert np.array_equal(host(u).view(np.uint32), host(v).view(np.uint32))
    dx, dw, db = nk.conv2d_bwd(x, dy, w, stride=2, pad=1, want_dx=False)
    assert dx is None
    assert np.array_equal(host(dw).view(np.uint32), host(a[1]).view(np.uint32))
