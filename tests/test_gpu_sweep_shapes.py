"""The dense projection at the full sizes of the GEMV sweep (out x in
2048x7168, 7168x2048 and 4096x14336; K2, K3 and K4; 1, 2, 4, 8, 16 and 64 rows), where each
launch picks its split-K cluster size and occupancy for the shape, rate and row count.

Up to eight rows go through the decode GEMV with static weights, as the bench calls it
(sx_linear_ex with SX_LINEAR_WEIGHTS_STATIC); 16 and 64 rows through the tensor-core projection
(sx_linear_gemm).  Random trellis words (the bench's weights), and one encoded weight as the
config names it: N(0, 0.02) with 1% of the input channels x8, quantized at window 12 by the
restated reference quantizer (quantizeNamed, src/encoder/quantize.zig:593), driven by activations
with outlier channels (src/exl3/f32_truth.zig:42-54).  Truth: y = x . W in f64 over the
reference's dense twin `decodeDense` (src/exl3/linear.zig:406-431); bars as the other parity
tests: max |y - truth| / max |truth| <= 1e-2 and relative RMS <= 5e-3.  The encoded pack's
dequantised inner matrix is also checked bit for bit against the reference's host decode.
"""

import os


import numpy as np
import pytest

from oracle import oracle as orc
from oracle import synth
from tests.helpers import MAX_REL_TOL, REL_RMS_TOL, dev, host_u16, max_rel, rel_rms, random_pack, to_f32

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SHAPES = [(7168, 2048), (2048, 7168), (14336, 4096)]  # (in, out)
RATES = [32, 48, 64]  # K2, K3, K4
CACHE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "_gen")


@pytest.fixture(scope="module")
def sx():
    import sushi_b200

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return sushi_b200


_CACHE = {}


def _pack(in_f, out_f, n):
    """The shape's pack on the device and its dense f32 twin (built once per shape and rate)."""
    if (in_f, out_f, n) not in _CACHE:
        seed = in_f // 7 + out_f if n == 32 else in_f // 7 + out_f + 1000 * n
        tr, su, sv = random_pack(seed, in_f, out_f, n)
        W = orc.decode_dense(tr, su, sv, in_f, out_f, n, orc.CB_MCG, 16)
        _CACHE.clear()  # one twin at a time (up to 235 MB)
        _CACHE[(in_f, out_f, n)] = (tr, su, sv, W)
    return _CACHE[(in_f, out_f, n)]


@pytest.mark.parametrize("rows", [1, 2, 4, 8, 16, 64])
@pytest.mark.parametrize("in_f,out_f", SHAPES)
@pytest.mark.parametrize("n", RATES)  # nearest the function: varies slowest, one twin per shape and rate
def test_sweep_shape(sx, n, in_f, out_f, rows):
    tr, su, sv, W = _pack(in_f, out_f, n)
    proj = sx.Proj(dev(tr, torch), dev(su, torch), dev(sv, torch))
    dec = sx.Decode(sx.Codebook.MCG, 16)
    x = torch.from_numpy(synth.activations(rows + in_f, rows, in_f)).cuda().to(torch.bfloat16)
    if rows < 16:
        y = to_f32(sx.linear(x, proj, dec, flags=sx.LINEAR_WEIGHTS_STATIC))
    else:
        y = to_f32(sx.linear_gemm(x, proj, dec))
    truth = orc.matvec_f64(W, x.float().cpu().numpy())
    assert np.isfinite(y).all()
    assert max_rel(y, truth) <= MAX_REL_TOL, max_rel(y, truth)
    assert rel_rms(y, truth) <= REL_RMS_TOL, rel_rms(y, truth)
    assert sx.device_error() == 0


@pytest.fixture(scope="module")
def encoded():
    pack = synth.config2_pack(CACHE)
    tr, su, sv = pack["trellis"], pack["suh"], pack["svh"]
    assert tr.shape == (128, 448, 32)
    W = orc.decode_dense(tr, su, sv, 2048, 7168, 32, orc.CB_MCG, 12)
    return tr, su, sv, W


def test_encoded_outlier_pack_dequant_bit_exact(sx, encoded):
    tr, su, sv, _ = encoded
    proj = sx.Proj(dev(tr, torch), dev(su, torch), dev(sv, torch))
    got = host_u16(sx.dequant_inner(proj, 0, sx.Decode(sx.Codebook.MCG, 12)))
    np.testing.assert_array_equal(got, orc.reconstruct_inner(tr, 2048, 7168, 32, orc.CB_MCG, 12))


@pytest.mark.parametrize("rows", [1, 2, 4, 8, 16, 64])
def test_encoded_outlier_pack_projection(sx, encoded, rows):
    tr, su, sv, W = encoded
    proj = sx.Proj(dev(tr, torch), dev(su, torch), dev(sv, torch))
    dec = sx.Decode(sx.Codebook.MCG, 12)
    x = torch.from_numpy(synth.outlier_activations(0xC0F2 + rows, rows, 2048)).cuda().to(torch.bfloat16)
    if rows < 16:
        y = to_f32(sx.linear(x, proj, dec, flags=sx.LINEAR_WEIGHTS_STATIC))
    else:
        y = to_f32(sx.linear_gemm(x, proj, dec))
    truth = orc.matvec_f64(W, x.float().cpu().numpy())
    assert np.isfinite(y).all()
    assert max_rel(y, truth) <= MAX_REL_TOL, max_rel(y, truth)
    assert rel_rms(y, truth) <= REL_RMS_TOL, rel_rms(y, truth)
    assert sx.device_error() == 0
