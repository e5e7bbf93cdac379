"""Fused EXL3 projection (sx_linear) against the f32 truth and the reference's CPU projection.

Truth: y = x . W in f64 with W the reference's dense f32 twin `decodeDense`
(src/exl3/linear.zig:406-431), as its f32-truth bars score the Metal arms
(src/exl3/f32_truth.zig:56-63).  Bar: max |y - truth| / max |truth| <= 1e-2 (BASELINE.json's
north star) and relative RMS <= 5e-3.  The reference's own CPU projection `format.project`
(src/exl3/expert_exl3.zig:546), which rounds its inner sums and output to f16, is checked
against the same bars.
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


def _x(seed, rows, in_f, dtype):
    x = synth.activations(seed, rows, in_f)
    t = torch.from_numpy(x).cuda().to(dtype)
    return t, t.float().cpu().numpy()


def _check(sx, tr, su, sv, in_f, out_f, n, cb, w, rows, dtype=None, seed=0):
    dtype = dtype or torch.bfloat16
    oargs, dec = dec_args(cb, w)
    proj = sx.Proj(dev(tr, torch), dev(su, torch), dev(sv, torch))
    xt, xv = _x(seed + rows, rows, in_f, dtype)
    y = to_f32(sx.linear(xt, proj, dec))
    W = orc.decode_dense(tr, su, sv, in_f, out_f, n, *oargs)
    truth = orc.matvec_f64(W, xv)
    assert np.isfinite(y).all()
    assert max_rel(y, truth) <= MAX_REL_TOL, max_rel(y, truth)
    assert rel_rms(y, truth) <= REL_RMS_TOL, rel_rms(y, truth)
    return y, truth, xv


def _check_reference(y, xv, tr, su, sv, in_f, out_f, n, cb, w):
    """The fused projection against the reference's CPU projection `format.project` on the same
    pack and rows: the GEMV's doubled-k products skip the f16 rounding of each weight's half sum
    that the CPU decode applies, and format.project rounds its inner sums and outputs to f16, so the
    two agree to the output bar, not bit for bit."""
    oargs, _ = dec_args(cb, w)
    ref = orc.project(xv, tr, su, sv, in_f, out_f, n, *oargs)
    assert max_rel(y, ref) <= MAX_REL_TOL, max_rel(y, ref)


@pytest.mark.parametrize("n", [16, 24, 32, 36, 40, 42, 48, 56, 64, 80, 96, 112, 128])
def test_linear_mcg_every_rate_class(sx, n):
    tr, su, sv = random_pack(n, 256, 384, n)
    y, _, xv = _check(sx, tr, su, sv, 256, 384, n, orc.CB_MCG, 16, rows=1)
    _check_reference(y, xv, tr, su, sv, 256, 384, n, orc.CB_MCG, 16)


@pytest.mark.parametrize("rows", [1, 2, 3, 4, 7, 8, 9, 16, 17, 33, 64])
def test_linear_rows(sx, rows):
    tr, su, sv = random_pack(11, 512, 256, 32)
    _check(sx, tr, su, sv, 512, 256, 32, orc.CB_MCG, 16, rows=rows)


@pytest.mark.parametrize(
    "cb,w,n",
    [(orc.CB_MUL1, 16, 32), (orc.CB_MUL1, 16, 64), (orc.CB_MCG, 12, 40), (orc.CB_MCG, 8, 48), (orc.CB_SPEC1, 15, 16),
     (orc.CB_SPEC1, 15, 32), (orc.CB_SPEC1, 15, 64), (orc.CB_SPEC1, 15, 128), (orc.CB_STD1, 15, 40),
     (orc.CB_PAIR1, 16, 24), (orc.CB_PAIR1, 16, 32), (orc.CB_PAIR1, 16, 48), (orc.CB_PAIR1, 16, 64)],
)
def test_linear_codebooks(sx, cb, w, n):
    tr, su, sv = random_pack(100 + n + cb, 384, 256, n)
    y, _, xv = _check(sx, tr, su, sv, 384, 256, n, cb, w, rows=3)
    _check_reference(y, xv, tr, su, sv, 384, 256, n, cb, w)


@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
def test_linear_dtypes(sx, dtype):
    tr, su, sv = random_pack(21, 256, 256, 32)
    _check(sx, tr, su, sv, 256, 256, 32, orc.CB_MCG, 16, rows=2, dtype=getattr(torch, dtype))


@pytest.mark.parametrize("in_f,out_f", [(128, 128), (7168, 256), (256, 7168), (2048, 1024)])
def test_linear_geometry_splits(sx, in_f, out_f):
    tr, su, sv = random_pack(in_f + out_f, in_f, out_f, 32)
    _check(sx, tr, su, sv, in_f, out_f, 32, orc.CB_MCG, 16, rows=1)


def test_linear_encoded_pack_and_reference_projection(sx):
    # A pack the quantizer restatement wrote (w12 keeps the CPU search quick), with outlier channels.
    w = synth.dense_weight(7, 512, 384, 0.02, outlier_frac=0.01)
    tr, su, sv, _ = synth.encode_weight(w, 7, "blk.0.ffn", 32, orc.CB_MCG, 12)
    y, truth, xv = _check(sx, tr, su, sv, 512, 384, 32, orc.CB_MCG, 12, rows=2)
    ref = orc.project(xv, tr, su, sv, 512, 384, 32, orc.CB_MCG, 12)
    assert max_rel(ref, truth) <= MAX_REL_TOL
    assert max_rel(y, ref) <= 2 * MAX_REL_TOL


def test_linear_grouped(sx):
    tr, su, sv = random_pack(33, 256, 128, 40, experts=3)
    proj = sx.Proj(dev(tr, torch), dev(su, torch), dev(sv, torch))
    _, dec = dec_args(orc.CB_MCG, 16)
    xs = [synth.activations(40 + g, 2, 256) for g in range(3)]
    xt = torch.from_numpy(np.stack(xs)).cuda().to(torch.bfloat16)
    y = to_f32(sx.linear_grouped(xt, proj, dec))
    for g in range(3):
        W = orc.decode_dense(tr[g], su[g], sv[g], 256, 128, 40, orc.CB_MCG, 16)
        truth = orc.matvec_f64(W, xt[g].float().cpu().numpy())
        assert max_rel(y[g], truth) <= MAX_REL_TOL


def test_linear_refusals(sx):
    tr, su, sv = random_pack(3, 256, 128, 32)
    proj = sx.Proj(dev(tr, torch), dev(su, torch), dev(sv, torch))
    _, dec = dec_args(orc.CB_MCG, 16)
    with pytest.raises(sx.Exl3Error) as e:
        sx.linear(torch.zeros((1, 128), device="cuda", dtype=torch.bfloat16), proj, dec)
    assert e.value.name == "SX_ERR_BAD_SHAPE"
    with pytest.raises(sx.Exl3Error) as e:
        sx.linear(torch.zeros((1, 256), device="cuda", dtype=torch.int32), proj, dec)
    assert e.value.name == "SX_ERR_BAD_DTYPE"
    assert sx.device_error() == 0


@pytest.mark.parametrize("rows", [1, 5, 33])
def test_linear_static_weights_overlap_matches(sx, rows):
    """sx_linear_ex with SX_LINEAR_WEIGHTS_STATIC (programmatic dependent launch) gives the same
    bits as sx_linear, over a chain where each launch reads the previous launch's output."""
    tr, su, sv = random_pack(21, 512, 512, 32)
    _, dec = dec_args(orc.CB_MCG, 16)
    proj = sx.Proj(dev(tr, torch), dev(su, torch), dev(sv, torch))
    x0, _ = _x(3, rows, 512, torch.bfloat16)
    outs = []
    for flags in (0, sx.LINEAR_WEIGHTS_STATIC):
        a = x0.clone()
        b = torch.empty_like(a)
        for _ in range(6):  # a -> b -> a ...: each launch's x is the previous launch's y
            sx.linear(a, proj, dec, flags=flags, out=b)
            a, b = b, a
        torch.cuda.synchronize()
        outs.append(a.clone())
    assert torch.equal(outs[0], outs[1])
    assert torch.isfinite(outs[0].float()).all()


@pytest.mark.parametrize("rows,cols", [(1, [0, 128, 384, 512]), (5, [0, 256, 512]), (20, [0, 128, 256, 384, 512])])
def test_linear_shared_stacked_outputs(sx, rows, cols):
    """linear.linearShared: linears stacked along the output with one suh row each; linear s's
    truth is the dense twin with suh row s, columns cols[s]..cols[s+1]."""
    in_f, out_f, n = 384, 512, 32
    count = len(cols) - 1
    tr, su0, sv = random_pack(33, in_f, out_f, n)
    rng = np.random.default_rng(4)
    suh = np.stack([su0] + [(su0.view(np.float16) * rng.choice([-1.0, 1.0], size=in_f).astype(np.float16)).view(np.uint16)
                            for _ in range(count - 1)])
    _, dec = dec_args(orc.CB_MCG, 16)
    proj = sx.Proj(dev(tr, torch), dev(suh, torch), dev(sv, torch))
    xt, xv = _x(9, rows, in_f, torch.bfloat16)
    outs = sx.linear_shared(xt, proj, cols, dec)
    for s in range(count):
        W = orc.decode_dense(tr, suh[s], sv, in_f, out_f, n, orc.CB_MCG, 16)[:, cols[s]:cols[s + 1]]
        truth = orc.matvec_f64(W, xv)
        y = to_f32(outs[s])
        assert y.shape == (rows, cols[s + 1] - cols[s])
        assert max_rel(y, truth) <= MAX_REL_TOL, (s, max_rel(y, truth))


@pytest.mark.parametrize(
    "in_f,cols,rows,dtype",
    [
        (384, [0, 256, 512], 1, torch.bfloat16),
        (384, [0, 512], 3, torch.float16),
        (1024, [0, 1536, 2048], 9, torch.bfloat16),
        (512, [0, 128, 384, 640], 16, torch.float32),
    ],
)
def test_linear_shared_normed_first_linear(sx, in_f, cols, rows, dtype):
    """linear.linearSharedNormed: linear 0 leaves as MLX's rms_norm of its finished row
    (src/exl3/project_rows.zig:394-456) in the same launch; the other linears are linear_shared's
    bytes.  Bars: the f64 truth of the normed row (1e-2), the unfused composition (linear_shared,
    then the norm in f32 with the same roundings) to one output rounding, and a second call on
    the same workspace gives the same bytes and leaves the workspace zeroed."""
    out_f, n = cols[-1], 32
    count = len(cols) - 1
    tr, su0, sv = random_pack(41, in_f, out_f, n)
    rng = np.random.default_rng(7)
    suh = np.stack([su0] + [(su0.view(np.float16) * rng.choice([-1.0, 1.0], size=in_f).astype(np.float16)).view(np.uint16)
                            for _ in range(count - 1)])
    _, dec = dec_args(orc.CB_MCG, 16)
    proj = sx.Proj(dev(tr, torch), dev(suh, torch), dev(sv, torch))
    xt, xv = _x(12, rows, in_f, dtype)
    w = torch.from_numpy(rng.uniform(0.5, 1.5, size=cols[1]).astype(np.float32)).cuda().to(dtype)
    eps = 1e-6
    ws = torch.zeros(sx.linear_shared_normed_workspace_bytes(proj), dtype=torch.uint8, device="cuda")
    outs = sx.linear_shared_normed(xt, proj, cols, dec, w, eps, workspace=ws)
    plain = sx.linear_shared(xt, proj, cols, dec)
    torch.cuda.synchronize()
    assert int(ws[:16].count_nonzero()) == 0, "the block counter is back at zero"
    for s in range(1, count):
        assert torch.equal(outs[s], plain[s]), s

    W0 = orc.decode_dense(tr, suh[0], sv, in_f, out_f, n, orc.CB_MCG, 16)[:, : cols[1]]
    truth = orc.rms_norm_truth(orc.matvec_f64(W0, xv), to_f32(w), eps)
    y = to_f32(outs[0])
    assert y.shape == (rows, cols[1])
    assert max_rel(y, truth) <= MAX_REL_TOL, max_rel(y, truth)

    o = plain[0].float()
    inv = torch.rsqrt((o * o).mean(dim=-1, keepdim=True) + eps)
    want = (w.float() * (o * inv).to(dtype).float()).to(dtype).float()
    # two output roundings apart at most (the sums' order and rsqrt may differ in the last bit)
    rtol = {torch.bfloat16: 2.0**-6, torch.float16: 2.0**-9, torch.float32: 2.0**-18}[dtype]
    assert torch.allclose(outs[0].float(), want, rtol=rtol, atol=0.0)

    again = sx.linear_shared_normed(xt, proj, cols, dec, w, eps, workspace=ws)
    torch.cuda.synchronize()
    for s in range(count):
        assert torch.equal(again[s], outs[s]), s
    assert int(ws[:16].count_nonzero()) == 0
