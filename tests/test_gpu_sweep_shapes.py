"""The dense projection at the full sizes of the GEMV sweep (out x in
2048x7168, 7168x2048 and 4096x14336, K2), where each launch picks its split-K cluster size and
occupancy for the shape and row count (two CTAs per SM at split 8 for 4096x14336 at one row).

One and eight rows go through the decode GEMV with static weights, as the bench calls it
(sx_linear_ex with SX_LINEAR_WEIGHTS_STATIC); 16 and 64 rows through the tensor-core projection
(sx_linear_gemm).  Truth: y = x . W in f64 over the reference's dense twin `decodeDense`
(src/exl3/linear.zig:406-431); bars as the other parity tests: max |y - truth| / max |truth| <=
1e-2 and relative RMS <= 5e-3.
"""

import numpy as np
import pytest

from oracle import oracle as orc
from oracle import synth
from tests.helpers import MAX_REL_TOL, REL_RMS_TOL, dev, max_rel, rel_rms, random_pack, to_f32

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SHAPES = [(7168, 2048), (2048, 7168), (14336, 4096)]  # (in, out)
N = 32  # K2


@pytest.fixture(scope="module")
def sx():
    import sushi_b200

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return sushi_b200


_CACHE = {}


def _pack(in_f, out_f):
    """The shape's pack on the device and its dense f32 twin (built once per shape)."""
    if (in_f, out_f) not in _CACHE:
        tr, su, sv = random_pack(in_f // 7 + out_f, in_f, out_f, N)
        W = orc.decode_dense(tr, su, sv, in_f, out_f, N, orc.CB_MCG, 16)
        _CACHE.clear()  # one shape's twin at a time (up to 235 MB)
        _CACHE[(in_f, out_f)] = (tr, su, sv, W)
    return _CACHE[(in_f, out_f)]


@pytest.mark.parametrize("rows", [1, 8, 16, 64])
@pytest.mark.parametrize("in_f,out_f", SHAPES)  # nearest the function: varies slowest, one twin per shape
def test_sweep_shape(sx, in_f, out_f, rows):
    tr, su, sv, W = _pack(in_f, out_f)
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
