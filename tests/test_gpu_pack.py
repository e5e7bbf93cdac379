"""A pack loaded from safetensors shards and projected on the GPU: the pack order and the
pair-major order (`trellis_pm`, converted on the device to the order the kernels read) give the
same trellis and the same projection, within the bar of the f32 truth."""

import numpy as np
import pytest

from oracle import oracle as orc
from oracle import synth
from tests.helpers import MAX_REL_TOL, max_rel, random_pack, to_f32

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _tile_major(tr):
    E, IT, OT, n = tr.shape
    out = np.empty((E, OT // 2, IT, 2, n), tr.dtype)
    for pair in range(OT // 2):
        for o in range(2):
            out[:, pair, :, o] = tr[:, :, pair * 2 + o]
    return out


@pytest.mark.parametrize("pair_major", [False, True])
def test_shard_to_projection(tmp_path, pair_major):
    import sushi_b200 as sx
    from sushi_b200 import pack as P

    in_f, out_f, n = 512, 256, 32
    tr, su, sv = random_pack(91, in_f, out_f, n)  # one bank: [in/16, out/16, n], [in], [out]
    tr = tr[None]
    tensors = {"q.suh": su[None].view(np.float16), "q.svh": sv[None].view(np.float16)}
    if pair_major:
        tensors["q.trellis_pm"] = _tile_major(tr)
        meta = {"tile_order": "pair_major"}
    else:
        tensors["q.trellis"] = tr
        meta = {}
    path = str(tmp_path / "shard.safetensors")
    P.write_safetensors(path, tensors, meta)
    cfg = {"expert_quant": {"format": "exl3", "k": 2, "codebook": "mcg", **({"tile_order": "pair_major"} if pair_major else {})}}
    spec = P.parse_expert_quant(cfg)
    proj = P.SafeTensors(path).proj("q", spec)
    np.testing.assert_array_equal(proj.trellis.cpu().numpy().view(np.uint16), tr)
    x = torch.from_numpy(synth.activations(3, 4, in_f)).cuda().to(torch.bfloat16)
    y = to_f32(sx.linear(x, proj, P.decode_of(spec)))
    W = orc.decode_dense(tr[0], su, sv, in_f, out_f, n, orc.CB_MCG, 16)
    truth = orc.matvec_f64(W, x.float().cpu().numpy())
    assert max_rel(y, truth) <= MAX_REL_TOL
