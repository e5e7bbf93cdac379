"""sx_moe_static_scratch: the routed-expert layer for callers that cannot allocate device memory.

Callers recording a layer into a CUDA graph, callers whose allocator owns and bills every device
byte, and latency-critical loops that cannot take cudaMalloc's device-wide synchronisation cannot
pass sx_moe a workspace.  This entry point runs the same kernels on a scratch buffer compiled into
the library.  The test calls it twice in a row through the C ABI and holds each result to the
workspace entry point's output within the MoE bar the other parity tests use (and, since the
kernels are the same, expects the very same bits); it also checks the refusal above the buffer's
size.  Collected last (file name) so a failure here leaves every other test already run; it
depends on no state another test leaves behind.
"""

import ctypes

import numpy as np
import pytest

from tests.helpers import MAX_REL_TOL, dev, max_rel, random_pack

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _bank(sx, E, D, I, n):
    parts = []
    for seed, (i_f, o_f) in enumerate(((D, I), (D, I), (I, D))):
        tr, su, sv = random_pack(900 + seed, i_f, o_f, n, experts=E)
        parts.append(sx.Proj(dev(tr, torch), dev(su, torch), dev(sv, torch)))
    return sx.Bank(*parts)


def test_static_scratch_moe_matches_workspace_moe_twice_in_a_row():
    import sushi_b200 as sx
    from sushi_b200 import _lib

    assert torch.cuda.is_available()
    L = _lib.load()
    E, D, I, k, T = 16, 512, 256, 4, 6
    bank = _bank(sx, E, D, I, 32)
    dec = sx.Decode(sx.Codebook.MCG, 16)
    rng = np.random.default_rng(17)
    inds = torch.from_numpy(np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)).cuda()
    scores = torch.from_numpy((0.1 + rng.random((T, k)) * 0.3).astype(np.float32)).cuda()
    x = torch.randn((T, D), device="cuda").to(torch.bfloat16)

    want = sx.moe(x, bank, inds, scores, dec).float().cpu().numpy()

    b, d = bank.c(), dec.c()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.sx_moe_workspace_bytes(ctypes.byref(b), T, k) <= L.sx_moe_static_scratch_bytes()
    for _ in range(2):
        y = torch.full((T, D), float("nan"), device="cuda").to(torch.bfloat16)
        st = L.sx_moe_static_scratch(stream, ctypes.byref(b), ctypes.byref(d), x.data_ptr(), 2, T, inds.data_ptr(),
                                     scores.data_ptr(), k, None, None, 0, y.data_ptr())
        assert st == 0, L.sx_status_name(st).decode()
        got = y.float().cpu().numpy()
        assert np.isfinite(got).all()
        assert max_rel(got, want) <= MAX_REL_TOL
        np.testing.assert_array_equal(got, want)
    assert L.sx_device_error(stream) == 0


def test_static_scratch_refuses_a_layer_larger_than_its_buffer():
    from sushi_b200 import _lib

    L = _lib.load()
    fake = 0x10000  # never dereferenced: the size check returns before any launch
    g = _lib.SxProj(fake, fake, fake, 64, 2048, 512, 32, 0)
    dn = _lib.SxProj(fake, fake, fake, 64, 512, 2048, 32, 0)
    bank = _lib.SxBank(g, g, dn)
    dec = _lib.SxDecode(1, 16, -1)
    rows, topk = 256, 8
    assert L.sx_moe_workspace_bytes(ctypes.byref(bank), rows, topk) > L.sx_moe_static_scratch_bytes()
    st = L.sx_moe_static_scratch(None, ctypes.byref(bank), ctypes.byref(dec), fake, 2, rows, fake, fake, topk, None, None,
                                 0, fake)
    assert L.sx_status_name(st).decode() == "SX_ERR_STATIC_SCRATCH_TOO_SMALL"
