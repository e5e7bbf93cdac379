"""a 4096x4096 dense linear, W ~ N(0, 0.02) bf16 from a seed, encoded to EXL3 K=2
(MCG, n32, window 16) by the restated reference encoder with an identity Hessian; one bf16 N(0,1)
activation row.  Checks: the device's dequantised inner matrix bit-exact against the reference's
host decode (reconstructInner), and y = x . W within the stated bar of the f32 truth over the
reference-decoded weights (decodeDense).

The pack takes about five minutes of CPU to encode; it is cached under tests/golden/_gen/ and
regenerated when missing.
"""

import os

import numpy as np
import pytest

from oracle import oracle as orc
from oracle import synth
from tests.helpers import MAX_REL_TOL, REL_RMS_TOL, dev, host_u16, max_rel, rel_rms

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
CACHE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "_gen")


@pytest.fixture(scope="module")
def pack():
    return synth.config1_pack(CACHE)


def test_config1_dequant_bit_exact_and_gemv_within_bar(pack):
    import sushi_b200 as sx

    tr, su, sv = pack["trellis"], pack["suh"], pack["svh"]
    assert tr.shape == (256, 256, 32)
    proj = sx.Proj(dev(tr, torch), dev(su, torch), dev(sv, torch))
    dec = sx.Decode(sx.Codebook.MCG, 16)
    got = host_u16(sx.dequant_inner(proj, 0, dec))
    want = orc.reconstruct_inner(tr, 4096, 4096, 32, orc.CB_MCG, 16)
    np.testing.assert_array_equal(got, want)

    x = synth.activations(0xC0F1 + 1, 1, 4096)
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    y = sx.linear(xt, proj, dec).float().cpu().numpy()
    W = orc.decode_dense(tr, su, sv, 4096, 4096, 32, orc.CB_MCG, 16)
    truth = orc.matvec_f64(W, xt.float().cpu().numpy())
    assert max_rel(y, truth) <= MAX_REL_TOL, max_rel(y, truth)
    assert rel_rms(y, truth) <= REL_RMS_TOL, rel_rms(y, truth)
    # The reference's own CPU projection of the same pack, to the same bar.
    ref = orc.project(xt.float().cpu().numpy(), tr, su, sv, 4096, 4096, 32, orc.CB_MCG, 16)
    assert max_rel(ref, truth) <= MAX_REL_TOL
    # Quantisation itself (not a parity bar): the K2 pack approximates the bf16 source weight.
    w_src = synth.dense_weight(synth.CONFIG1_SEED, 4096, 4096, 0.02)
    q_err = rel_rms(W, w_src)
    assert q_err < 0.5, q_err
