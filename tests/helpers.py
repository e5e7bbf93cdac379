"""Shared helpers for the parity tests: device upload of packs, truth products, error metrics."""

import numpy as np

from oracle import oracle as orc

# The tolerance BASELINE.json's north star states for GEMV/GEMM outputs: max relative error
# <= 1e-2 against an fp32 accumulation of the reference-decoded weights.  "Relative" is taken
# against the largest truth magnitude of the output (the inf-norm), since a single element's
# relative error is unbounded near zero.
MAX_REL_TOL = 1e-2
# The reference's f32-truth bar on whole outputs (src/exl3/f32_truth.zig relRms, parity bars in
# docs/engine-exl3-experts.md "Parity bars"): relative RMS against the f64 truth.
REL_RMS_TOL = 5e-3


def max_rel(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))


def rel_rms(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.sqrt(((got - want) ** 2).sum() / max((want**2).sum(), 1e-30)))


def dev(a, torch):
    """numpy -> CUDA tensor (u16 bit patterns travel as int16)."""
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).cuda()


def host_u16(t):
    return t.cpu().numpy().view(np.uint16)


def to_f32(t):
    return t.float().cpu().numpy()


def dec_args(codebook, window_bits=16, table=None):
    """(oracle args, sushi_b200.Decode kwargs) for one decode."""
    import sushi_b200 as sx

    if table is None:
        table = {orc.CB_SPEC1: orc.TABLE_SPEC1_W15, orc.CB_STD1: orc.TABLE_STD1}.get(codebook, -1)
    return (codebook, window_bits, table), sx.Decode(sx.Codebook(codebook), window_bits, None if table < 0 else table)


def random_pack(seed, in_f, out_f, n, experts=1, suh_mag=0.05, svh_mag=1.0):
    from oracle import synth

    tr, su, sv = synth.random_bank(seed, experts, in_f, out_f, n, suh_mag, svh_mag)
    if experts == 1:
        return tr[0], su[0], sv[0]
    return tr, su, sv
