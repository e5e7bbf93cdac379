"""Tensor-core projection (sx_linear_gemm, tcgen05) against the f32 truth.

Truth as for sx_linear: y = x . W in f64 with W the reference's dense twin `decodeDense`
(src/exl3/linear.zig:406-431).  Bar: max |y - truth| / max |truth| <= 1e-2 and relative RMS
<= 5e-3.  The kernel multiplies the reference's f16 inner weights (the sums of the codebook
halves rounded to f16, as reconstructInner does) with f32 accumulation, so it also agrees with
the decode-GEMV path (sx_linear) to within the same bar.  Shapes cover one and several row
tiles (128 rows each), split-K clusters of 1..16 ranks, every codebook family and window.
"""

import numpy as np
import pytest

from oracle import oracle as orc
from oracle import synth
from tests.helpers import MAX_REL_TOL, REL_RMS_TOL, dec_args, dev, max_rel, rel_rms, random_pack, to_f32

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def sx():
    import sushi_b200

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return sushi_b200


def _check(sx, in_f, out_f, n, rows, cb=orc.CB_MCG, w=16, dtype=torch.bfloat16, seed=0):
    tr, su, sv = random_pack(seed + n + rows, in_f, out_f, n)
    oargs, dec = dec_args(cb, w)
    proj = sx.Proj(dev(tr, torch), dev(su, torch), dev(sv, torch))
    x = torch.from_numpy(synth.activations(seed + rows, rows, in_f)).cuda().to(dtype)
    y = to_f32(sx.linear_gemm(x, proj, dec))
    torch.cuda.synchronize()
    assert sx.device_error() == 0
    W = orc.decode_dense(tr, su, sv, in_f, out_f, n, *oargs)
    truth = orc.matvec_f64(W, x.float().cpu().numpy())
    assert np.isfinite(y).all()
    assert max_rel(y, truth) <= MAX_REL_TOL, max_rel(y, truth)
    assert rel_rms(y, truth) <= REL_RMS_TOL, rel_rms(y, truth)
    return y, x, proj, dec


@pytest.mark.parametrize("in_f,out_f,rows", [(256, 128, 1), (512, 256, 17), (1024, 384, 64), (2048, 256, 128),
                                             (1024, 128, 130), (4096, 256, 300), (512, 1024, 33)])
def test_gemm_shapes(sx, in_f, out_f, rows):
    _check(sx, in_f, out_f, 32, rows)


@pytest.mark.parametrize("in_f,out_f,rows", [(256, 128 * 74, 1024), (2048, 256, 400), (4096, 128, 777)])
def test_gemm_four_row_tiles_per_cta(sx, in_f, out_f, rows):
    """From 384 rows, four 128-row accumulators per CTA share each decoded chunk; with few output
    blocks the input range is also split over a cluster (400 rows: the last tile holds 16)."""
    _check(sx, in_f, out_f, 32, rows)


@pytest.mark.parametrize("n", [16, 24, 32, 40, 48, 64, 96, 128])
def test_gemm_rates(sx, n):
    _check(sx, 512, 256, n, 40)


@pytest.mark.parametrize("cb,w,n", [(orc.CB_MUL1, 16, 32), (orc.CB_SPEC1, 15, 16), (orc.CB_STD1, 16, 48),
                                    (orc.CB_PAIR1, 16, 24), (orc.CB_MCG, 12, 32)])
def test_gemm_codebooks(sx, cb, w, n):
    _check(sx, 512, 256, n, 24, cb=cb, w=w)


@pytest.mark.parametrize("rows", [1, 7, 16])
def test_gemm_sixteen_row_tiles(sx, rows):
    """At most 16 rows the projection runs 16-row tiles (MMA N = 16, a 16-row prepared-row copy):
    the same result bar, over codebooks and a k split."""
    _check(sx, 2048, 512, 32, rows)
    _check(sx, 512, 256, 24, rows, cb=orc.CB_PAIR1)
    _check(sx, 512, 256, 32, rows, cb=orc.CB_MUL1)
    _check(sx, 7168, 256, 48, rows, cb=orc.CB_STD1)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_gemm_dtypes(sx, dtype):
    _check(sx, 512, 256, 32, 20, dtype=dtype)


def test_gemm_agrees_with_gemv(sx):
    y, x, proj, dec = _check(sx, 2048, 512, 32, 48)
    y2 = to_f32(sx.linear(x, proj, dec))
    assert max_rel(y, y2) <= MAX_REL_TOL


def test_gemm_refuses_small_workspace(sx):
    tr, su, sv = random_pack(1, 256, 128, 32)
    _, dec = dec_args(orc.CB_MCG, 16)
    proj = sx.Proj(dev(tr, torch), dev(su, torch), dev(sv, torch))
    x = torch.zeros((4, 256), device="cuda", dtype=torch.bfloat16)
    with pytest.raises(sx.Exl3Error) as e:
        sx.linear_gemm(x, proj, dec, workspace=torch.empty(16, dtype=torch.uint8, device="cuda"))
    assert e.value.name == "SX_ERR_WORKSPACE_TOO_SMALL"
