"""Bit-exact device decode against the oracle (the reference's host decoder).

The north star's first parity bar: dequantised weights bit-exact against the reference's decode.
sx_dequant_inner writes the inner f16 matrix as reconstructInner does
(src/exl3/expert_exl3.zig:416-438); sx_decode_codewords runs every codeword through the device
codebook, as the reference holds every Metal reader to the host decode over all 65536 codewords
(firstPair1PairMismatch, :361-369).
"""

import ctypes
import time

import numpy as np
import pytest

from oracle import oracle as orc
from tests.helpers import dec_args, dev, host_u16, random_pack

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def sx():
    import sushi_b200

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return sushi_b200


LINEAR_FIXTURES = [
    ("exl3_k4_linear", 64, orc.CB_MUL1, 16),
    ("exl3_k3_linear", 48, orc.CB_MUL1, 16),
    ("exl3_k2_linear", 32, orc.CB_MUL1, 16),
    ("exl3_k2p5_mcg_linear", 40, orc.CB_MCG, 16),
    ("exl3_k3_mcg_linear", 48, orc.CB_MCG, 16),
    ("exl3_k2p5_mcg_w12_linear", 40, orc.CB_MCG, 12),
]


@pytest.mark.parametrize("stem,n,cb,w", LINEAR_FIXTURES)
def test_device_dequant_matches_reference_fixture(sx, golden, stem, n, cb, w):
    g = golden(stem)
    proj = sx.Proj(dev(g["trellis"], torch), dev(g["suh"], torch), dev(g["svh"], torch))
    _, dec = dec_args(cb, w)
    got = host_u16(sx.dequant_inner(proj, 0, dec))
    np.testing.assert_array_equal(got, g["inner"])


def _cases():
    out = []
    for n in range(16, 129, 2):
        out.append((n, orc.CB_MCG, 16))
        if n % 8 == 0:
            out.append((n, orc.CB_MCG, 12))
            out.append((n, orc.CB_MUL1, 16))
            out.append((n, orc.CB_SPEC1, 15))
        if 24 <= n <= 64:
            out.append((n, orc.CB_PAIR1, 16))
            if n % 8 == 0:
                out.append((n, orc.CB_STD1, 9))
    return out


@pytest.mark.parametrize("n,cb,w", _cases())
def test_device_dequant_every_rate_matches_oracle(sx, n, cb, w):
    tr, su, sv = random_pack(1000 + n * 7 + cb, 128, 256, n)
    oargs, dec = dec_args(cb, w)
    want = orc.reconstruct_inner(tr, 128, 256, n, *oargs)
    proj = sx.Proj(dev(tr, torch), dev(su, torch), dev(sv, torch))
    got = host_u16(sx.dequant_inner(proj, 0, dec))
    np.testing.assert_array_equal(got, want)


def test_device_dequant_spec1_per_rate_table(sx):
    # The reference's test-only table whose row differs at every rate holds each reader to its own row.
    for n in (16, 24, 40, 64, 96, 128):
        tr, su, sv = random_pack(77 + n, 128, 128, n)
        want = orc.reconstruct_inner(tr, 128, 128, n, orc.CB_SPEC1, 12, orc.TABLE_SPEC1_TEST)
        proj = sx.Proj(dev(tr, torch), dev(su, torch), dev(sv, torch))
        got = host_u16(sx.dequant_inner(proj, 0, sx.Decode(sx.Codebook.SPEC1, 12, orc.TABLE_SPEC1_TEST)))
        np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize(
    "cb,n,w,table",
    [(orc.CB_MCG, 32, 16, -1), (orc.CB_MUL1, 32, 16, -1), (orc.CB_MCG, 40, 12, -1), (orc.CB_STD1, 32, 16, orc.TABLE_STD1)]
    + [(orc.CB_SPEC1, n, 15, orc.TABLE_SPEC1_W15) for n in (16, 24, 32, 48, 64, 96, 128)]
    + [(orc.CB_PAIR1, n, 16, -1) for n in range(24, 65, 2)],
)
def test_every_codeword_decodes_as_the_host(sx, cb, n, w, table):
    dec = sx.Decode(sx.Codebook(cb), w, None if table < 0 else table)
    got = sx.decode_codewords(n, dec).cpu().numpy().view(np.uint32)
    want = orc.decode_all(cb, n, w, table)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, f"first mismatching codeword {bad[0]:#x}: got {got[bad[0]]:#x} want {want[bad[0]]:#x}"


def test_refusals_are_named(sx):
    tr, su, sv = random_pack(5, 128, 128, 32)
    proj = sx.Proj(dev(tr, torch), dev(su, torch), dev(sv, torch))
    with pytest.raises(sx.Exl3Error) as e:
        sx.dequant_inner(proj, 0, sx.Decode(sx.Codebook.SPEC1, 15, None))
    assert e.value.name == "SX_ERR_CODEBOOK_TABLE_UNKNOWN"
    with pytest.raises(sx.Exl3Error) as e:
        sx.dequant_inner(proj, 0, sx.Decode(sx.Codebook.PAIR1, 15, None))
    assert e.value.name == "SX_ERR_CODEBOOK_TABLE_WINDOW_MISMATCH"
    with pytest.raises(sx.Exl3Error) as e:
        sx.dequant_inner(proj, 0, sx.Decode(sx.Codebook.MCG, 17, None))
    assert e.value.name == "SX_ERR_WINDOW_UNSUPPORTED"
    tr16, su16, sv16 = random_pack(6, 128, 128, 16)
    p16 = sx.Proj(dev(tr16, torch), dev(su16, torch), dev(sv16, torch))
    with pytest.raises(sx.Exl3Error) as e:
        sx.dequant_inner(p16, 0, sx.Decode(sx.Codebook.PAIR1, 16, None))
    assert e.value.name == "SX_ERR_CODEBOOK_TABLE_RATE_MISSING"
    assert sx.device_error() == 0


@pytest.mark.parametrize("n,E,in_f,out_f", [(32, 2, 256, 384), (18, 1, 128, 256), (64, 3, 384, 128)])
def test_tile_order_round_trip(n, E, in_f, out_f):
    """sx_tile_order_convert: pack order -> pair-major is layout.tileMajor (src/exl3/layout.zig:141),
    restated here in numpy, and pair-major -> pack undoes it bit for bit."""
    import sushi_b200 as sx

    rng = np.random.default_rng(n + E)
    src = rng.integers(0, 1 << 16, size=(E, in_f // 16, out_f // 16, n), dtype=np.uint16)
    IT, OT = in_f // 16, out_f // 16
    want = np.empty((E, OT // 2, IT, 2, n), np.uint16)
    for pair in range(OT // 2):
        for tk in range(IT):
            for o in range(2):
                want[:, pair, tk, o] = src[:, tk, pair * 2 + o]
    t = torch.from_numpy(src.view(np.int16)).cuda()
    pm = sx.tile_order_convert(t, sx.TileOrder.PAIR_MAJOR)
    np.testing.assert_array_equal(pm.cpu().numpy().view(np.uint16), want)
    back = sx.tile_order_convert(pm, sx.TileOrder.PACK, sx.TileOrder.PAIR_MAJOR)
    np.testing.assert_array_equal(back.cpu().numpy().view(np.uint16), src)


def test_bounded_wait_gives_up_and_the_context_stays_usable():
    """The failure-detection path: a kernel waits on a barrier nothing arrives at; the bounded wait
    gives up after its limit, latches code 3 (sx_device_error), and later work runs normally."""
    import sushi_b200 as sx
    from sushi_b200 import _lib

    L = _lib.load()
    assert sx.device_error() == 0
    t0 = time.perf_counter()
    assert L.sx_selftest_wait_timeout(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), 20) == 0
    assert sx.device_error() == 3  # synchronises, reads and clears the latch
    assert time.perf_counter() - t0 < 5.0
    assert sx.device_error() == 0
    tr, su, sv = random_pack(5, 256, 128, 32)
    _, dec = dec_args(orc.CB_MCG, 16)
    proj = sx.Proj(dev(tr, torch), dev(su, torch), dev(sv, torch))
    y = sx.linear(torch.ones((1, 256), device="cuda", dtype=torch.bfloat16), proj, dec)
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all() and sx.device_error() == 0
