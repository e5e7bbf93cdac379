"""sx_moe_static_scratch: the routed-expert layer for callers that cannot allocate device memory.

Callers whose allocator owns and bills every device byte, and latency-critical loops that cannot
take cudaMalloc's device-wide synchronisation, cannot pass sx_moe a workspace.  This entry point
runs the same kernels on a scratch buffer compiled into the library.  The tests call it through
the C ABI twice in a row and hold each result to the workspace entry point's output within the MoE
bar the other parity tests use (and, since the kernels are the same, expect the very same bits);
at the decode sizes of BASELINE configs[2] (512 experts, hidden 2048, intermediate 512, K2, top-10,
one and 64 tokens, which fit the buffer) they also hold it to the oracle's f64 truth.  They check
the refusal above the buffer's size and that a malformed call gets sx_moe's own refusal, and they
capture the call into a CUDA graph and replay it over new inputs.
Collected last (file name) so a failure here leaves every other test already run; it depends on
no state another test leaves behind.
"""

import ctypes

import numpy as np
import pytest

from oracle import oracle as orc
from oracle import synth
from tests.helpers import MAX_REL_TOL, REL_RMS_TOL, dev, max_rel, random_pack, rel_rms

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _bank(sx, E, D, I, n, seed=900):
    parts, host = [], []
    for i, (i_f, o_f) in enumerate(((D, I), (D, I), (I, D))):
        tr, su, sv = random_pack(seed + i, i_f, o_f, n, experts=E)
        host.append((tr, su, sv))
        parts.append(sx.Proj(dev(tr, torch), dev(su, torch), dev(sv, torch)))
    return sx.Bank(*parts), host


def _static(L, b, d, x, inds, scores, T, k, D):
    """Two calls in a row of sx_moe_static_scratch; returns both outputs as f32 arrays."""
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    outs = []
    for _ in range(2):
        y = torch.full((T, D), float("nan"), device="cuda").to(torch.bfloat16)
        st = L.sx_moe_static_scratch(stream, ctypes.byref(b), ctypes.byref(d), x.data_ptr(), 2, T, inds.data_ptr(),
                                     scores.data_ptr(), k, None, None, 0, y.data_ptr())
        assert st == 0, L.sx_status_name(st).decode()
        outs.append(y.float().cpu().numpy())
    assert L.sx_device_error(stream) == 0
    return outs


def test_static_scratch_moe_matches_workspace_moe_twice_in_a_row():
    import sushi_b200 as sx
    from sushi_b200 import _lib

    assert torch.cuda.is_available()
    L = _lib.load()
    E, D, I, k, T = 16, 512, 256, 4, 6
    bank, _ = _bank(sx, E, D, I, 32)
    dec = sx.Decode(sx.Codebook.MCG, 16)
    rng = np.random.default_rng(17)
    inds = torch.from_numpy(np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)).cuda()
    scores = torch.from_numpy((0.1 + rng.random((T, k)) * 0.3).astype(np.float32)).cuda()
    x = torch.randn((T, D), device="cuda").to(torch.bfloat16)

    want = sx.moe(x, bank, inds, scores, dec).float().cpu().numpy()
    b, d = bank.c(), dec.c()
    assert L.sx_moe_workspace_bytes(ctypes.byref(b), T, k) <= L.sx_moe_static_scratch_bytes()
    for got in _static(L, b, d, x, inds, scores, T, k, D):
        assert np.isfinite(got).all()
        assert max_rel(got, want) <= MAX_REL_TOL
        np.testing.assert_array_equal(got, want)


def test_static_scratch_moe_replays_from_a_cuda_graph():
    """The use the entry point exists for: one warm call, the layer captured into a CUDA graph
    (no allocation, no host read inside), then replays over new inputs written into the captured
    buffers; each replay gives sx_moe's bits for the inputs of that replay."""
    import sushi_b200 as sx
    from sushi_b200 import _lib

    L = _lib.load()
    E, D, I, k, T = 16, 512, 256, 4, 5
    bank, _ = _bank(sx, E, D, I, 32, seed=940)
    dec = sx.Decode(sx.Codebook.MCG, 16)
    b, d = bank.c(), dec.c()
    rng = np.random.default_rng(41)

    def route():
        ii = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
        return torch.from_numpy(ii).cuda(), torch.from_numpy((0.1 + rng.random((T, k)) * 0.3).astype(np.float32)).cuda()

    x = torch.randn((T, D), device="cuda").to(torch.bfloat16)
    inds, scores = route()
    y = torch.empty((T, D), device="cuda", dtype=torch.bfloat16)
    stream = torch.cuda.Stream()

    def call():
        h = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        st = L.sx_moe_static_scratch(h, ctypes.byref(b), ctypes.byref(d), x.data_ptr(), 2, T, inds.data_ptr(),
                                     scores.data_ptr(), k, None, None, 0, y.data_ptr())
        assert st == 0, L.sx_status_name(st).decode()

    with torch.cuda.stream(stream):
        call()  # warm: kernel attributes are set outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        call()
    for rep in range(2):
        x.copy_(torch.randn((T, D), device="cuda").to(torch.bfloat16))
        ni, ns = route()
        inds.copy_(ni)
        scores.copy_(ns)
        y.fill_(float("nan"))
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
        want = sx.moe(x, bank, inds, scores, dec)
        assert torch.equal(y, want), rep
    del g
    assert L.sx_device_error(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0


@pytest.fixture(scope="module")
def qwen_layer():
    """The configs[2] routed bank (512 experts, 2048/512, K2 MCG) and its router matrix."""
    import sushi_b200 as sx

    assert torch.cuda.is_available()
    E, D, I = 512, 2048, 512
    bank, host = _bank(sx, E, D, I, 32, seed=5100)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5200)
    wr = (torch.randn((D, E), device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    return bank, host, wr


@pytest.mark.parametrize("T", [1, 64])
def test_static_scratch_decode_layer_at_config_size(qwen_layer, T):
    import sushi_b200 as sx
    from sushi_b200 import _lib

    L = _lib.load()
    bank, host, wr = qwen_layer
    E, D, I, k, n = 512, 2048, 512, 10, 32
    dec = sx.Decode(sx.Codebook.MCG, 16)
    x = torch.from_numpy(synth.activations(5300 + T, T, D)).cuda().to(torch.bfloat16)
    inds, scores, _ = sx.router_topk_gate(x @ wr, k)
    inds = inds.to(torch.int32).contiguous()
    scores = scores.float().contiguous()
    b, d = bank.c(), dec.c()
    assert L.sx_moe_workspace_bytes(ctypes.byref(b), T, k) <= L.sx_moe_static_scratch_bytes()
    want = sx.moe(x, bank, inds, scores, dec).float().cpu().numpy()
    outs = _static(L, b, d, x, inds, scores, T, k, D)

    xv = x.float().cpu().numpy().astype(np.float64)
    ii = inds.cpu().numpy()
    ww = scores.cpu().numpy().astype(np.float64)
    dense = {}
    truth = np.zeros((T, D), np.float64)
    for r in range(T):
        for j in range(k):
            e = int(ii[r, j])
            if e not in dense:
                dense[e] = tuple(orc.decode_dense(p[0][e], p[1][e], p[2][e], i_f, o_f, n, orc.CB_MCG, 16)
                                 for p, (i_f, o_f) in zip(host, ((D, I), (D, I), (I, D))))
            truth[r] += ww[r, j] * orc.expert_truth(dense[e], xv[r])
    for got in outs:
        assert np.isfinite(got).all()
        assert max_rel(got, truth) <= MAX_REL_TOL, max_rel(got, truth)
        assert rel_rms(got, truth) <= REL_RMS_TOL, rel_rms(got, truth)
        assert max_rel(got, want) <= MAX_REL_TOL
        np.testing.assert_array_equal(got, want)


def test_static_scratch_refuses_a_layer_larger_than_its_buffer():
    from sushi_b200 import _lib

    L = _lib.load()
    fake = 0x10000  # never dereferenced: the checks return before any launch
    g = _lib.SxProj(fake, fake, fake, 64, 2048, 512, 32, 0)
    dn = _lib.SxProj(fake, fake, fake, 64, 512, 2048, 32, 0)
    bank = _lib.SxBank(g, g, dn)
    dec = _lib.SxDecode(1, 16, -1)
    rows, topk = 256, 8
    assert L.sx_moe_workspace_bytes(ctypes.byref(bank), rows, topk) > L.sx_moe_static_scratch_bytes()
    st = L.sx_moe_static_scratch(None, ctypes.byref(bank), ctypes.byref(dec), fake, 2, rows, fake, fake, topk, None, None,
                                 0, fake)
    assert L.sx_status_name(st).decode() == "SX_ERR_STATIC_SCRATCH_TOO_SMALL"


def test_static_scratch_gives_a_malformed_call_sx_moes_refusal():
    from sushi_b200 import _lib

    L = _lib.load()
    fake = 0x10000
    g = _lib.SxProj(fake, fake, fake, 64, 2048, 512, 32, 0)
    dn = _lib.SxProj(fake, fake, fake, 64, 512, 2048, 32, 0)
    bank = _lib.SxBank(g, g, dn)
    dec = _lib.SxDecode(1, 16, -1)
    rows, topk = 256, 8  # too large for the buffer as well: the malformed part is refused first
    st = L.sx_moe_static_scratch(None, ctypes.byref(bank), ctypes.byref(dec), fake, 2, rows, fake, fake, topk, None, None,
                                 500, fake)
    assert L.sx_status_name(st).decode() == "SX_ERR_INVALID_CLAMP"
    bad = _lib.SxProj(fake, fake, fake, 64, 2000, 512, 32, 0)  # hidden not a multiple of 128
    st = L.sx_moe_static_scratch(None, ctypes.byref(_lib.SxBank(bad, bad, dn)), ctypes.byref(dec), fake, 2, 4, fake, fake,
                                 topk, None, None, 0, fake)
    assert L.sx_status_name(st).decode() == "SX_ERR_BAD_SHAPE"
