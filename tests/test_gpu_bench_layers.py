"""The MoE layers of BASELINE configs[3] and configs[4] at the sizes the bench runs them, against the
oracle's f64 truth.

the configs[2] layer (512 experts of hidden 2048 / intermediate 512, K2 MCG, top-10
softmax over bf16 logits, sigmoid-gated shared expert folded in) in prefill: 8192 tokens with a
Zipf(1.1) bias over a seeded rank permutation added to the logits, so the hottest expert takes
nearly every token.  That layer runs the tensor-core path: experts with at least 384 rows through
the CTA-pair (cta_group::2) kernel over 512-row chunks, the rest through the one-row-tile kernel
(the reference's moePrefill, src/exl3/expert_exl3_kernels.zig:2861).  The truth is taken on a
seeded sample of 40 of the 8192 rows, over the dense twins of every expert those rows touch.

one DeepSeek-style layer: hidden 7168, 256 routed experts of intermediate 2048 in two
rate groups of SPEC1 window 15 (K1 n16 experts 0..63, K2 n32 the rest), a K4 (n64) shared expert,
top-8 sigmoid routing with a bias, renormalised and x2.5 (rate_groups.moeDecode / moePrefill,
src/exl3/rate_groups.zig:1659, :2042).  Four tokens take the decode chain; 1024 tokens take the
tensor-core path (checked on a sample of 4 rows).

Truth: the f64 routed sum of the reference's f32-truth SwiGLU slot (src/exl3/f32_truth.zig:85-98)
over the reference-decoded dense twins, with the routing the kernel used, plus the shared expert
(gated where the layer gates it).  Bars as the other MoE parity tests: max relative 1e-2 (against
the largest truth magnitude), relative RMS 5e-3.
"""

import numpy as np
import pytest

from oracle import oracle as orc
from oracle import synth
from tests.helpers import MAX_REL_TOL, REL_RMS_TOL, dev, max_rel, rel_rms, to_f32

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _sx_bank(sx, parts):
    return sx.Bank(*[sx.Proj(dev(p[0], torch), dev(p[1], torch), dev(p[2], torch)) for p in parts])


def _expert_truth(parts, e, dims, n, oargs, xs):
    """The f64 SwiGLU expert e of a host bank on rows xs [r, D]."""
    dense = tuple(orc.decode_dense(p[0][e], p[1][e], p[2][e], i_f, o_f, n, *oargs) for p, (i_f, o_f) in zip(parts, dims))
    return np.stack([orc.expert_truth(dense, x) for x in xs])


def test_config3_prefill_layer_full_size():
    import sushi_b200 as sx

    assert torch.cuda.is_available()
    E, D, I, K, n, T = 512, 2048, 512, 10, 32, 8192
    dims = ((D, I), (D, I), (I, D))
    parts = [synth.random_bank(6000 + i, E, i_f, o_f, n, 0.05) for i, (i_f, o_f) in enumerate(dims)]
    sh_parts = [synth.random_bank(6100 + i, 1, i_f, o_f, n, 0.05) for i, (i_f, o_f) in enumerate(dims)]
    bank, shared = _sx_bank(sx, parts), _sx_bank(sx, sh_parts)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(6200)
    wr = (torch.randn((D, E), device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    wg = (torch.randn((D, 1), device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    ranks = torch.randperm(E, generator=torch.Generator().manual_seed(5)).double() + 1.0
    zb = ranks ** -1.1
    bias = torch.log(zb / zb.sum()).float().cuda()
    x = torch.from_numpy(synth.activations(6300, T, D)).cuda().to(torch.bfloat16)
    dec = sx.Decode(sx.Codebook.MCG, 16)
    inds, scores, _ = sx.router_topk_gate((x @ wr).float() + bias, K)
    gate = x @ wg
    y = to_f32(sx.moe_folded(x, bank, shared, inds, scores, dec, shared_gate=gate))
    torch.cuda.synchronize()
    assert sx.device_error() == 0
    assert np.isfinite(y).all()

    ii = inds.cpu().numpy()
    counts = np.bincount(ii.reshape(-1), minlength=E)
    assert counts.max() >= 4 * 384  # the hottest expert: 512-row chunks on the CTA-pair kernel
    assert ((counts > 0) & (counts < 384)).sum() > 100  # and many experts on the one-row-tile kernel

    rows = np.sort(np.random.default_rng(6400).choice(T, 40, replace=False))
    xv = x.float().cpu().numpy().astype(np.float64)[rows]
    ww = scores.cpu().numpy().astype(np.float64)[rows]
    sel = ii[rows]
    gv = gate.float().cpu().numpy().reshape(-1).astype(np.float64)[rows]
    oargs = (orc.CB_MCG, 16)
    truth = np.zeros((len(rows), D))
    for e in np.unique(sel):
        hit = np.nonzero(sel == e)
        out = _expert_truth(parts, int(e), dims, n, oargs, xv[hit[0]])
        truth[hit[0]] += ww[hit][:, None] * out
    truth += _expert_truth(sh_parts, 0, dims, n, oargs, xv) / (1.0 + np.exp(-gv))[:, None]
    got = y[rows]
    assert max_rel(got, truth) <= MAX_REL_TOL, max_rel(got, truth)
    assert rel_rms(got, truth) <= REL_RMS_TOL, rel_rms(got, truth)


@pytest.fixture(scope="module")
def deepseek_layer():
    import sushi_b200 as sx

    assert torch.cuda.is_available()
    H, I, E, K1 = 7168, 2048, 256, 64
    dims = ((H, I), (H, I), (I, H))
    g0 = [synth.random_bank(7000 + i, K1, i_f, o_f, 16, 0.02) for i, (i_f, o_f) in enumerate(dims)]
    g1 = [synth.random_bank(7100 + i, E - K1, i_f, o_f, 32, 0.02) for i, (i_f, o_f) in enumerate(dims)]
    sh = [synth.random_bank(7200 + i, 1, i_f, o_f, 64, 0.02) for i, (i_f, o_f) in enumerate(dims)]
    rb = sx.Ragged.from_banks([_sx_bank(sx, g0), _sx_bank(sx, g1)])
    shared = _sx_bank(sx, sh)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(7300)
    wr = (torch.randn((H, E), device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    bias = torch.randn((E,), device="cuda", generator=gen) * 0.1
    return sx, g0, g1, sh, rb, shared, wr, bias


@pytest.mark.parametrize("T,sample", [(4, 4), (1024, 4)])
def test_config4_deepseek_layer_full_size(deepseek_layer, T, sample):
    sx, g0, g1, sh, rb, shared, wr, bias = deepseek_layer
    H, I, E, K1, k = 7168, 2048, 256, 64, 8
    dims = ((H, I), (H, I), (I, H))
    dec = sx.Decode(sx.Codebook.SPEC1, 15, orc.TABLE_SPEC1_W15)
    x = torch.from_numpy(synth.activations(7400 + T, T, H)).cuda().to(torch.bfloat16)
    inds, scores, _ = sx.router_topk_gate(x @ wr, k, mode=sx.RouterMode.SIGMOID_BIAS, bias=bias, route_norm=True,
                                          route_scale=2.5)
    y = to_f32(sx.moe_folded(x, rb, shared, inds, scores, dec))
    torch.cuda.synchronize()
    assert sx.device_error() == 0
    assert np.isfinite(y).all()

    ii = inds.cpu().numpy()
    assert (ii < K1).any() and (ii >= K1).any()  # both rate groups in play
    rows = np.arange(T) if sample >= T else np.sort(np.random.default_rng(7500).choice(T, sample, replace=False))
    xv = x.float().cpu().numpy().astype(np.float64)[rows]
    ww = scores.cpu().numpy().astype(np.float64)[rows]
    sel = ii[rows]
    oargs = (orc.CB_SPEC1, 15, orc.TABLE_SPEC1_W15)
    truth = np.zeros((len(rows), H))
    for e in np.unique(sel):
        hit = np.nonzero(sel == e)
        parts, loc, n = (g0, int(e), 16) if e < K1 else (g1, int(e) - K1, 32)
        truth[hit[0]] += ww[hit][:, None] * _expert_truth(parts, loc, dims, n, oargs, xv[hit[0]])
    truth += _expert_truth(sh, 0, dims, 64, oargs, xv)
    got = y[rows]
    assert max_rel(got, truth) <= MAX_REL_TOL, max_rel(got, truth)
    assert rel_rms(got, truth) <= REL_RMS_TOL, rel_rms(got, truth)
