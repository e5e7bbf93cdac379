"""Router top-k and the routed-expert chain against the oracle's truth.

Router: inds exactly the oracle's (ties to the lowest id, src/moe_router.zig:130-150), weights
within 1e-5.  MoE: y against the f64 routed sum of the reference's f32-truth slot
(src/exl3/f32_truth.zig:85-98, routedErr :109-156) over dense twins of every expert, within the
stated GEMV bar (max relative 1e-2, relative RMS 5e-3).
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


@pytest.mark.parametrize("T,E,k", [(1, 512, 10), (8, 512, 10), (64, 512, 10), (5, 256, 8), (3, 64, 1), (2, 2048, 32)])
def test_router_softmax(sx, T, E, k):
    rng = np.random.default_rng(T * 1000 + E + k)
    logits = rng.standard_normal((T, E)).astype(np.float32)
    inds, scores = sx.router_topk(torch.from_numpy(logits).cuda(), k)
    wi, ww = orc.router_truth(logits, k)
    np.testing.assert_array_equal(inds.cpu().numpy(), wi)
    np.testing.assert_allclose(scores.cpu().numpy(), ww, rtol=1e-5, atol=1e-7)


def test_router_ties_go_to_lowest_id(sx):
    logits = np.zeros((2, 64), np.float32)
    logits[0, [5, 9, 40]] = 1.0
    inds, _ = sx.router_topk(torch.from_numpy(logits).cuda(), 4)
    assert inds.cpu().numpy()[0].tolist() == [5, 9, 40, 0]
    assert inds.cpu().numpy()[1].tolist() == [0, 1, 2, 3]


@pytest.mark.parametrize("grouped", [False, True])
def test_router_sigmoid_bias(sx, grouped):
    rng = np.random.default_rng(9 + grouped)
    T, E, k = 6, 256, 8
    logits = rng.standard_normal((T, E)).astype(np.float32)
    bias = (rng.standard_normal(E) * 0.1).astype(np.float32)
    mode = sx.RouterMode.SIGMOID_BIAS_GROUPED if grouped else sx.RouterMode.SIGMOID_BIAS
    kw = dict(n_group=8, topk_group=4) if grouped else {}
    inds, scores = sx.router_topk(torch.from_numpy(logits).cuda(), k, mode, torch.from_numpy(bias).cuda(),
                                  route_norm=True, route_scale=2.5, **kw)
    wi, ww = orc.router_truth(logits, k, "sigmoid_bias_grouped" if grouped else "sigmoid_bias", bias, True, 2.5, **kw)
    np.testing.assert_array_equal(inds.cpu().numpy(), wi)
    np.testing.assert_allclose(scores.cpu().numpy(), ww, rtol=1e-5, atol=1e-7)


def test_router_declines_like_the_reference(sx):
    lg = torch.zeros((1, 64), device="cuda")
    assert sx.router_topk(lg, 33) is None
    assert sx.router_topk(torch.zeros((1, 4096), device="cuda"), 8) is None
    assert sx.router_topk(lg, 4, sx.RouterMode.SIGMOID_BIAS_GROUPED, torch.zeros(64, device="cuda"), n_group=3,
                          topk_group=1) is None


def _gate_case(rng, gk, cancel):
    x = ((rng.random(gk) - 0.5) * 4.0).astype(np.float32)
    w = ((rng.random(gk) - 0.5) * 0.4).astype(np.float32)
    if cancel:  # the reference's test plants large cancelling products (src/moe_router.zig:786-793)
        for _ in range(3):
            i, j = rng.integers(0, gk, 2)
            if i != j:
                x[i], w[i], x[j], w[j] = 65536.0, 1.0, -65536.0, 1.0
    return x, w


@pytest.mark.parametrize("gk,tdt", [(2048, "bf16"), (7168, "bf16"), (2048, "f16"), (8, "bf16"), (1032, "bf16"),
                                    (16384, "bf16")])
def test_router_softmax_gate(sx, gk, tdt):
    """softmax_gate (moeRouterTopKGate, src/moe_router.zig:457): the gate logit is the oracle's
    restatement of MLX's dot order to the bit, and inds/scores equal the plain softmax mode's."""
    dt = torch.bfloat16 if tdt == "bf16" else torch.float16
    rng = np.random.default_rng(gk + (tdt == "f16"))
    for trial in range(3):
        x, w = _gate_case(rng, gk, cancel=trial > 0 and tdt == "bf16")
        gx, gw = torch.from_numpy(x).cuda().to(dt), torch.from_numpy(w).cuda().to(dt)
        logits = torch.from_numpy(((rng.random((1, 512)) - 0.5) * 8.0).astype(np.float32)).cuda().to(torch.bfloat16)
        got = sx.router_topk_gate(logits, 10, gate=(gx, gw))
        assert got is not None
        inds, scores, glog = got
        plain = sx.router_topk(logits.float(), 10)
        np.testing.assert_array_equal(inds.cpu().numpy(), plain[0].cpu().numpy())
        np.testing.assert_array_equal(scores.cpu().numpy(), plain[1].cpu().numpy())
        want = orc.router_gate_logit(gx.float().cpu().numpy(), gw.float().cpu().numpy())
        want_t = torch.tensor([want], dtype=torch.float32).to(dt)
        assert glog.dtype == dt
        assert glog.view(torch.int16).item() == want_t.view(torch.int16).item(), (glog.item(), want)


def test_router_logits_in_activation_dtypes(sx):
    """Logits of F16/BF16 (src/moe_router.zig:478) route exactly as their f32 values do."""
    rng = np.random.default_rng(5)
    for dt in (torch.bfloat16, torch.float16):
        lg = torch.from_numpy(rng.standard_normal((7, 256)).astype(np.float32)).cuda().to(dt)
        for mode, bias in ((sx.RouterMode.SOFTMAX, None),
                           (sx.RouterMode.SIGMOID_BIAS, torch.from_numpy(rng.standard_normal(256).astype(np.float32) * 0.1).cuda())):
            a = sx.router_topk_gate(lg, 8, mode=mode, bias=bias, route_scale=2.5)
            b = sx.router_topk(lg.float(), 8, mode, bias, route_scale=2.5)
            assert a[2] is None
            np.testing.assert_array_equal(a[0].cpu().numpy(), b[0].cpu().numpy())
            np.testing.assert_array_equal(a[1].cpu().numpy(), b[1].cpu().numpy())


def test_router_gate_declines_like_the_reference(sx):
    lg = torch.zeros((2, 64), device="cuda")
    g = torch.ones(2048, device="cuda", dtype=torch.bfloat16)
    assert sx.router_topk_gate(lg, 4, gate=(g, g)) is None  # two rows with a gate
    assert sx.router_topk_gate(lg[:1], 4, gate=(g[:12], g[:12])) is None  # not whole 8-element chunks
    big = torch.ones(16392, device="cuda", dtype=torch.bfloat16)
    assert sx.router_topk_gate(lg[:1], 4, gate=(big, big)) is None
    assert sx.router_topk_gate(lg[:1], 4, gate=(g.float(), g.float())) is None  # gate dtype
    # sigmoid modes ignore the gate (src/moe_router.zig:471)
    r = sx.router_topk_gate(lg, 4, gate=(g, g), mode=sx.RouterMode.SIGMOID_BIAS, bias=torch.zeros(64, device="cuda"))
    assert r is not None and r[2] is None


def _bank(seed, E, D, I, n_gu, n_d):
    g = random_pack(seed, D, I, n_gu, experts=E)
    u = random_pack(seed + 1, D, I, n_gu, experts=E)
    d = random_pack(seed + 2, I, D, n_d, experts=E, suh_mag=0.05)
    return g, u, d


def _truth(bank_np, D, I, n_gu, n_d, oargs, x, inds, wts, limit=0.0):
    dense = {}
    y = np.zeros((x.shape[0], D), np.float64)
    for r in range(x.shape[0]):
        for k in range(inds.shape[1]):
            e = int(inds[r, k])
            if e not in dense:
                g, u, d = bank_np
                dense[e] = (orc.decode_dense(g[0][e], g[1][e], g[2][e], D, I, n_gu, *oargs),
                            orc.decode_dense(u[0][e], u[1][e], u[2][e], D, I, n_gu, *oargs),
                            orc.decode_dense(d[0][e], d[1][e], d[2][e], I, D, n_d, *oargs))
            y[r] += wts[r, k] * orc.expert_truth(dense[e], x[r], limit)
    return y


def _sx_bank(sx, bank_np):
    return sx.Bank(*[sx.Proj(dev(p[0], torch), dev(p[1], torch), dev(p[2], torch)) for p in bank_np])


def _route(seed, T, E, k):
    rng = np.random.default_rng(seed)
    inds = np.stack([rng.choice(E, size=k, replace=False) for _ in range(T)]).astype(np.int32)
    wts = (0.05 + rng.random((T, k)) * 0.25).astype(np.float32)
    return inds, wts


@pytest.mark.parametrize("T", [1, 3, 8, 16, 37])
def test_moe_chain_matches_f32_truth(sx, T):
    E, D, I, k = 24, 512, 256, 4
    bank_np = _bank(T, E, D, I, 32, 32)
    oargs, dec = dec_args(orc.CB_MCG, 16)
    x = synth.activations(T, T, D)
    inds, wts = _route(T + 5, T, E, k)
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    y = to_f32(sx.moe(xt, _sx_bank(sx, bank_np), torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda(), dec))
    truth = _truth(bank_np, D, I, 32, 32, oargs, xt.float().cpu().numpy(), inds, wts)
    assert np.isfinite(y).all()
    assert max_rel(y, truth) <= MAX_REL_TOL, max_rel(y, truth)
    assert rel_rms(y, truth) <= REL_RMS_TOL, rel_rms(y, truth)
    assert sx.device_error() == 0


@pytest.mark.parametrize("cb,w,n_gu,n_d", [(orc.CB_PAIR1, 16, 24, 40), (orc.CB_SPEC1, 15, 16, 32), (orc.CB_MUL1, 16, 48, 32)])
def test_moe_codebooks_and_mixed_down_rate(sx, cb, w, n_gu, n_d):
    E, D, I, k, T = 12, 256, 128, 3, 5
    bank_np = _bank(cb * 10 + n_gu, E, D, I, n_gu, n_d)
    oargs, dec = dec_args(cb, w)
    x = synth.activations(77, T, D)
    inds, wts = _route(cb, T, E, k)
    xt = torch.from_numpy(x).cuda().to(torch.float16)
    y = to_f32(sx.moe(xt, _sx_bank(sx, bank_np), torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda(), dec))
    truth = _truth(bank_np, D, I, n_gu, n_d, oargs, xt.float().cpu().numpy(), inds, wts)
    assert max_rel(y, truth) <= MAX_REL_TOL, max_rel(y, truth)


def test_moe_clamped_and_shared(sx):
    E, D, I, k, T = 8, 256, 128, 2, 4
    bank_np = _bank(5, E, D, I, 32, 32)
    oargs, dec = dec_args(orc.CB_MCG, 16)
    x = synth.activations(5, T, D) * 4.0
    inds, wts = _route(6, T, E, k)
    xt = torch.from_numpy(x).cuda().to(torch.float32)
    b = _sx_bank(sx, bank_np)
    ii, ww = torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda()
    y = to_f32(sx.moe_clamped(xt, b, ii, ww, dec, 2))
    truth = _truth(bank_np, D, I, 32, 32, oargs, x, inds, wts, limit=2.0)
    assert max_rel(y, truth) <= MAX_REL_TOL, max_rel(y, truth)
    shared = torch.randn((T, D), device="cuda")
    gate = torch.randn((T,), device="cuda")
    y2 = to_f32(sx.moe_with_gated_shared(xt, b, ii, ww, dec, shared, gate))
    base = _truth(bank_np, D, I, 32, 32, oargs, x, inds, wts)
    want = base + (1 / (1 + np.exp(-gate.cpu().numpy().astype(np.float64))))[:, None] * shared.cpu().numpy()
    assert max_rel(y2, want) <= MAX_REL_TOL
    with pytest.raises(sx.Exl3Error) as e:
        sx.moe(xt, b, torch.zeros((T, 33), dtype=torch.int32, device="cuda"), torch.zeros((T, 33), device="cuda"), dec)
    assert e.value.name == "SX_ERR_TOPK_EXCEEDS_REDUCE_BANK"
    with pytest.raises(sx.Exl3Error) as e:
        sx.moe_clamped(xt, b, ii, ww, dec, 129)
    assert e.value.name == "SX_ERR_INVALID_CLAMP"


def _zipf_route(seed, T, E, k, s=1.1):
    """Top-k routes with a Zipf(s) preference over experts, so some experts take several
    128-row chunks and others none (the prefill config's skew)."""
    rng = np.random.default_rng(seed)
    p = 1.0 / np.arange(1, E + 1) ** s
    p = p[rng.permutation(E)]
    p /= p.sum()
    inds = np.stack([rng.choice(E, size=k, replace=False, p=p) for _ in range(T)]).astype(np.int32)
    wts = (0.05 + rng.random((T, k)) * 0.25).astype(np.float32)
    return inds, wts


@pytest.mark.parametrize("T,E,k,big", [(300, 64, 6, False), (200, 16, 4, False), (700, 16, 4, True)])
def test_moe_prefill_tensor_core_path(sx, T, E, k, big):
    """More than 16 rows take the tcgen05 path (prep, gate/up GEMMs, mid, down GEMM, reduce);
    experts with 384 or more rows take the four-row-tile kernel (`big`)."""
    D, I = 512, 256
    bank_np = _bank(T + E, E, D, I, 32, 32)
    oargs, dec = dec_args(orc.CB_MCG, 16)
    x = synth.activations(T + 1, T, D)
    inds, wts = _zipf_route(T, T, E, k)
    most = np.bincount(inds.ravel(), minlength=E).max()
    assert most > 128 and (most >= 384) == big  # an expert spans several row tiles
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    y = to_f32(sx.moe(xt, _sx_bank(sx, bank_np), torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda(), dec))
    truth = _truth(bank_np, D, I, 32, 32, oargs, xt.float().cpu().numpy(), inds, wts)
    assert np.isfinite(y).all()
    assert max_rel(y, truth) <= MAX_REL_TOL, max_rel(y, truth)
    assert rel_rms(y, truth) <= REL_RMS_TOL, rel_rms(y, truth)
    assert sx.device_error() == 0


def test_moe_prefill_clamped_gated_shared_and_codebook(sx):
    E, D, I, k, T = 8, 256, 128, 2, 80
    bank_np = _bank(15, E, D, I, 24, 40)
    oargs, dec = dec_args(orc.CB_PAIR1, 16)
    x = synth.activations(6, T, D) * 4.0
    inds, wts = _route(16, T, E, k)
    xt = torch.from_numpy(x).cuda().to(torch.float16)
    b = _sx_bank(sx, bank_np)
    ii, ww = torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda()
    y = to_f32(sx.moe_clamped(xt, b, ii, ww, dec, 2))
    truth = _truth(bank_np, D, I, 24, 40, oargs, xt.float().cpu().numpy(), inds, wts, limit=2.0)
    assert max_rel(y, truth) <= MAX_REL_TOL, max_rel(y, truth)
    shared = torch.randn((T, D), device="cuda").to(torch.float16)
    gate = torch.randn((T,), device="cuda").to(torch.float16)
    y2 = to_f32(sx.moe_with_gated_shared(xt, b, ii, ww, dec, shared, gate))
    base = _truth(bank_np, D, I, 24, 40, oargs, xt.float().cpu().numpy(), inds, wts)
    sg = 1 / (1 + np.exp(-gate.float().cpu().numpy().astype(np.float64)))
    want = base + sg[:, None] * shared.float().cpu().numpy()
    assert max_rel(y2, want) <= MAX_REL_TOL


@pytest.mark.parametrize("T,cb,w", [(5, orc.CB_MCG, 16), (200, orc.CB_MCG, 16), (7, orc.CB_SPEC1, 15)])
def test_moe_ragged_rate_groups(sx, T, cb, w):
    """rate_groups.Ragged: two rate groups (K1 n=16 and K2 n=32, as the DeepSeek config's routed
    experts) in one layer; every slot decodes at its expert's group rate.  T=5/7: decode chain per
    group; T=200: the tensor-core path per group."""
    D, I, k = 256, 128, 4
    E0, E1 = 6, 10
    g0 = _bank(400 + T, E0, D, I, 16, 16)
    g1 = _bank(500 + T, E1, D, I, 32, 32)
    oargs, dec = dec_args(cb, w)
    rb = sx.Ragged.from_banks([_sx_bank(sx, g0), _sx_bank(sx, g1)])
    x = synth.activations(T + 9, T, D)
    inds, wts = _route(T + 3, T, E0 + E1, k)
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    y = to_f32(sx.moe_ragged(xt, rb, torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda(), dec))
    torch.cuda.synchronize()
    assert sx.device_error() == 0
    xf = xt.float().cpu().numpy()
    truth = np.zeros((T, D))
    dense = {}
    for r in range(T):
        for j in range(k):
            e = int(inds[r, j])
            bank_np, loc, n = (g0, e, 16) if e < E0 else (g1, e - E0, 32)
            if e not in dense:
                dense[e] = tuple(orc.decode_dense(p[0][loc], p[1][loc], p[2][loc], a, b, n, *oargs)
                                 for p, a, b in zip(bank_np, (D, D, I), (I, I, D)))
            truth[r] += wts[r, j] * orc.expert_truth(dense[e], xf[r])
    assert np.isfinite(y).all()
    assert max_rel(y, truth) <= MAX_REL_TOL, max_rel(y, truth)
    assert rel_rms(y, truth) <= REL_RMS_TOL, rel_rms(y, truth)


def test_moe_wide_hidden_decode_chain(sx):
    """A wide hidden size (7168, the DeepSeek config's) with few active experts: the decode chain's
    k split grows until each CTA's prepared input slice fits in shared memory."""
    E, D, I, k, T = 4, 7168, 256, 2, 1
    bank_np = _bank(71, E, D, I, 32, 32)
    oargs, dec = dec_args(orc.CB_MCG, 16)
    x = synth.activations(72, T, D)
    inds, wts = _route(73, T, E, k)
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    y = to_f32(sx.moe(xt, _sx_bank(sx, bank_np), torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda(), dec))
    truth = _truth(bank_np, D, I, 32, 32, oargs, xt.float().cpu().numpy(), inds, wts)
    assert max_rel(y, truth) <= MAX_REL_TOL, max_rel(y, truth)
    assert sx.device_error() == 0


@pytest.mark.parametrize("k,folded", [(15, True), (16, True), (16, False), (10, True)])
def test_moe_one_token_items(sx, k, folded):
    """One token: its k slots (and a folded shared expert) are the decode chain's work items and a
    cluster of them per output block reduces in k order (up to 16 items); 17 items take the routed
    chain.  Both against the f64 truth of the routed sum plus the shared expert."""
    E, D, I, T = 40, 512, 256, 1
    bank_np = _bank(800 + k, E, D, I, 32, 32)
    sh_np = _bank(900 + k, 1, D, I, 32, 32)
    oargs, dec = dec_args(orc.CB_MCG, 16)
    x = synth.activations(k, T, D)
    inds, wts = _route(k + 1, T, E, k)
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    b, shb = _sx_bank(sx, bank_np), _sx_bank(sx, sh_np)
    ii, ww = torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda()
    xf = xt.float().cpu().numpy()
    truth = _truth(bank_np, D, I, 32, 32, oargs, xf, inds, wts)
    if folded:
        y = to_f32(sx.moe_folded(xt, b, shb, ii, ww, dec))
        sh_e = tuple(tuple(a[None] for a in proj) for proj in sh_np)  # (one-expert packs come squeezed)
        truth = truth + _truth(sh_e, D, I, 32, 32, oargs, xf, np.zeros((T, 1), np.int32), np.ones((T, 1), np.float32))
    else:
        y = to_f32(sx.moe(xt, b, ii, ww, dec))
    torch.cuda.synchronize()
    assert sx.device_error() == 0
    assert max_rel(y, truth) <= MAX_REL_TOL, max_rel(y, truth)
    assert rel_rms(y, truth) <= REL_RMS_TOL, rel_rms(y, truth)


def test_moe_one_token_skips_slots_outside_the_bank(sx):
    """A one-token layer whose slots name ids past the bank (another rank's experts, sentinels)
    leaves those slots out of the sum, as the routed chain does."""
    E, D, I, k, T = 16, 256, 128, 6, 1
    bank_np = _bank(55, E, D, I, 32, 32)
    oargs, dec = dec_args(orc.CB_MCG, 16)
    x = synth.activations(56, T, D)
    inds, wts = _route(57, T, E, k)
    inds[0, 1] = E
    inds[0, 4] = E + 100
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    y = to_f32(sx.moe(xt, _sx_bank(sx, bank_np), torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda(), dec))
    live = [j for j in range(k) if inds[0, j] < E]
    truth = _truth(bank_np, D, I, 32, 32, oargs, xt.float().cpu().numpy(), inds[:, live], wts[:, live])
    torch.cuda.synchronize()
    assert sx.device_error() == 0
    assert max_rel(y, truth) <= MAX_REL_TOL, max_rel(y, truth)


def _unfused(sx, x, bank, shb, inds, wts, dec, gate, shared_dec=None, ragged=False, clamp=0):
    """The composition sx_moe_folded replaces: the shared expert as its own one-expert layer, its
    output passed to the routed layer."""
    T = x.shape[0]
    one_i = torch.zeros((T, 1), dtype=torch.int32, device="cuda")
    one_s = torch.ones((T, 1), device="cuda")
    sh = sx.moe(x, shb, one_i, one_s, shared_dec or dec, clamp_limit=clamp)
    fn = sx.moe_ragged if ragged else sx.moe
    return fn(x, bank, inds, wts, dec, shared=sh, shared_gate=gate, clamp_limit=clamp)


@pytest.mark.parametrize(
    "T,n_sh,gated",
    [(1, 32, True), (5, 32, False), (16, 32, True),  # same rate: folded into the routed launches
     (3, 64, True),                                    # other rate, <= 16 rows: its own chain launches
     (40, 32, True),                                   # > 16 rows: tensor-core path
     (200, 32, True)],                                 # routed layer on the tensor-core path
)
def test_moe_folded_equals_unfused(sx, T, n_sh, gated):
    """moe_shared_fold.folded: the routed layer with its shared expert in one call gives the bits of
    the unfused composition (the shared expert's own layer output passed as `shared`), in each of
    the three ways the shared expert runs (at these sizes both take the same k split)."""
    E, D, I, k = (16, 256, 128, 4) if T < 100 else (8, 256, 128, 2)
    bank_np = _bank(600 + T, E, D, I, 32, 32)
    sh_np = _bank(700 + T, 1, D, I, n_sh, n_sh)
    _, dec = dec_args(orc.CB_MCG, 16)
    b, shb = _sx_bank(sx, bank_np), _sx_bank(sx, sh_np)
    x = torch.from_numpy(synth.activations(T + 5, T, D)).cuda().to(torch.bfloat16)
    inds, wts = _route(T + 6, T, E, k)
    ii, ww = torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda()
    gate = torch.randn((T,), device="cuda").to(torch.bfloat16) if gated else None
    want = _unfused(sx, x, b, shb, ii, ww, dec, gate)
    got = sx.moe_folded(x, b, shb, ii, ww, dec, shared_gate=gate)
    torch.cuda.synchronize()
    assert sx.device_error() == 0
    assert torch.equal(got, want)
    got2 = sx.moe_folded(x, b, shb, ii, ww, dec, shared_gate=gate, clamp_limit=7)
    want2 = _unfused(sx, x, b, shb, ii, ww, dec, gate, clamp=7)
    torch.cuda.synchronize()
    assert torch.equal(got2, want2)


@pytest.mark.parametrize("T", [2, 24])
def test_moe_ragged_folded_equals_unfused(sx, T):
    """The DeepSeek shape of the fold: K1/K2 rate groups with a K4 shared expert (SPEC1 w15, whose
    table has every rate), which runs as its own launches."""
    D, I, k = 256, 128, 4
    g0 = _bank(800 + T, 6, D, I, 16, 16)
    g1 = _bank(900 + T, 10, D, I, 32, 32)
    sh_np = _bank(950 + T, 1, D, I, 64, 64)
    _, dec = dec_args(orc.CB_SPEC1, 15)
    rb = sx.Ragged.from_banks([_sx_bank(sx, g0), _sx_bank(sx, g1)])
    shb = _sx_bank(sx, sh_np)
    x = torch.from_numpy(synth.activations(T + 7, T, D)).cuda().to(torch.bfloat16)
    inds, wts = _route(T + 8, T, 16, k)
    ii, ww = torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda()
    want = _unfused(sx, x, rb, shb, ii, ww, dec, None, ragged=True)
    got = sx.moe_folded(x, rb, shb, ii, ww, dec)
    torch.cuda.synchronize()
    assert sx.device_error() == 0
    assert torch.equal(got, want)


@pytest.mark.parametrize("T", [1, 9])
def test_moe_chained_layers_match_synchronised_layers(sx, T):
    """The decode chain's kernels start early (programmatic dependent launch) and wait for their
    predecessor before touching global memory: layers whose input is the previous layer's output,
    issued back to back (routing included), give the bits of the same layers with a device
    synchronisation between them, with the shared expert folded and not."""
    E, D, I, k, L = 16, 256, 128, 4, 5
    banks = [_sx_bank(sx, _bank(1000 + 10 * l, E, D, I, 32, 32)) for l in range(L)]
    shb = _sx_bank(sx, _bank(1100, 1, D, I, 32, 32))
    _, dec = dec_args(orc.CB_MCG, 16)
    wr = torch.randn((D, E), device="cuda") * 0.05
    x0 = torch.from_numpy(synth.activations(T + 11, T, D)).cuda().to(torch.bfloat16)

    def run(sync, fold):
        x = x0
        for l in range(L):
            inds, scores = sx.router_topk((x.float() @ wr), k)
            y = (sx.moe_folded(x, banks[l], shb, inds, scores, dec) if fold else sx.moe(x, banks[l], inds, scores, dec))
            x = (x.float() + y.float()).to(torch.bfloat16)
            if sync:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        return x

    for fold in (False, True):
        want = run(True, fold)
        for _ in range(3):
            assert torch.equal(run(False, fold), want), fold
    assert sx.device_error() == 0
