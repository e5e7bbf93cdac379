"""The MoE decode layer at the full size of BASELINE configs[2], as the bench runs it: 512 routed
experts of hidden 2048 / intermediate 512 at K2 (MCG), top-10 softmax routing by the library's
router over bf16 logits, and one shared expert gated by sigmoid of its gate logit, folded into the
routed call (moe_shared_fold.folded, src/moe_shared_fold.zig:24).  At one token the router also
returns the gate logit (softmax_gate, src/moe_router.zig:457); at 8 and 64 tokens it comes from a
matmul.  64 tokens touch ~370 experts through the decode chain.

Truth: the f64 routed sum of the reference's f32-truth SwiGLU slot (src/exl3/f32_truth.zig:85-98)
over the dense twins of the touched experts, with the routing the kernel used, plus
sigmoid(gate) times the shared expert's truth; bars as the other MoE parity tests (max relative
1e-2, relative RMS 5e-3).
"""

import numpy as np
import pytest

from oracle import oracle as orc
from oracle import synth
from tests.helpers import MAX_REL_TOL, REL_RMS_TOL, dev, max_rel, random_pack, rel_rms, to_f32

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

E, D, I, K, N = 512, 2048, 512, 10, 32


@pytest.fixture(scope="module")
def layer():
    import sushi_b200 as sx

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    parts_np = [random_pack(4000 + i, i_f, o_f, N, experts=E) for i, (i_f, o_f) in enumerate(((D, I), (D, I), (I, D)))]
    sh_np = [random_pack(4100 + i, i_f, o_f, N, experts=1) for i, (i_f, o_f) in enumerate(((D, I), (D, I), (I, D)))]
    bank = sx.Bank(*[sx.Proj(dev(p[0], torch), dev(p[1], torch), dev(p[2], torch)) for p in parts_np])
    shared = sx.Bank(*[sx.Proj(dev(p[0][None], torch), dev(p[1][None], torch), dev(p[2][None], torch))
                       for p in sh_np])
    gen = torch.Generator(device="cuda")
    gen.manual_seed(4200)
    wr = (torch.randn((D, E), device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    wg = (torch.randn((D, 1), device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    sh_dense = tuple(orc.decode_dense(p[0], p[1], p[2], i_f, o_f, N, orc.CB_MCG, 16)
                     for p, (i_f, o_f) in zip(sh_np, ((D, I), (D, I), (I, D))))
    return sx, parts_np, bank, shared, wr, wg, sh_dense


@pytest.mark.parametrize("T", [1, 8, 64])
def test_full_layer_against_truth(layer, T):
    sx, parts_np, bank, shared, wr, wg, sh_dense = layer
    dec = sx.Decode(sx.Codebook.MCG, 16)
    x = torch.from_numpy(synth.activations(4300 + T, T, D)).cuda().to(torch.bfloat16)
    if T == 1:
        inds, scores, gate = sx.router_topk_gate(x @ wr, K, gate=(x, wg))
    else:
        inds, scores, _ = sx.router_topk_gate(x @ wr, K)
        gate = x @ wg
    y = to_f32(sx.moe_folded(x, bank, shared, inds, scores, dec, shared_gate=gate))
    torch.cuda.synchronize()
    assert sx.device_error() == 0

    xv = x.float().cpu().numpy().astype(np.float64)
    ii = inds.cpu().numpy()
    ww = scores.cpu().numpy().astype(np.float64)
    gv = gate.float().cpu().numpy().reshape(-1).astype(np.float64)
    dense = {}
    truth = np.zeros((T, D), np.float64)
    for r in range(T):
        for j in range(K):
            e = int(ii[r, j])
            if e not in dense:
                dense[e] = tuple(orc.decode_dense(p[0][e], p[1][e], p[2][e], i_f, o_f, N, orc.CB_MCG, 16)
                                 for p, (i_f, o_f) in zip(parts_np, ((D, I), (D, I), (I, D))))
            truth[r] += ww[r, j] * orc.expert_truth(dense[e], xv[r])
        truth[r] += orc.expert_truth(sh_dense, xv[r]) / (1.0 + np.exp(-gv[r]))
    assert np.isfinite(y).all()
    assert max_rel(y, truth) <= MAX_REL_TOL, max_rel(y, truth)
    assert rel_rms(y, truth) <= REL_RMS_TOL, rel_rms(y, truth)
    if T == 64:
        assert len(dense) > 300  # the decode chain over most of the bank
