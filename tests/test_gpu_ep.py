"""Expert-parallel routed layer (sx_ep_moe) on the GPU, over both transports (NVLink peer buffers,
the default, and NCCL all-to-alls).

One GPU: a world-1 communicator sends every row to itself, so sx_ep_moe must give the same bits
as sx_moe (the partial is the same k-order f32 sum; the combine adds it to 0), over either
transport.  Two GPUs (skipped
on one): each rank holds half of the experts and its own rows; its output must match the
single-GPU sx_moe over the full bank within the stated bar (the partials of two ranks are added
in rank order instead of k order, so a few outputs differ in their last bit) and the f32 truth.
"""

import os

import numpy as np
import pytest

from oracle import oracle as orc
from oracle import synth
from tests.helpers import MAX_REL_TOL, REL_RMS_TOL, dec_args, dev, max_rel, rel_rms, random_pack, to_f32

pytestmark = pytest.mark.gpu

TRANSPORTS = ["peer", "nccl"]

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def sx():
    import sushi_b200

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return sushi_b200


def _bank_np(seed, E, D, I, n):
    return (random_pack(seed, D, I, n, experts=E), random_pack(seed + 1, D, I, n, experts=E),
            random_pack(seed + 2, I, D, n, experts=E, suh_mag=0.05))


def _bank(sx, bank_np, e0=None, e1=None):
    sl = slice(e0, e1)
    return sx.Bank(*[sx.Proj(dev(np.ascontiguousarray(p[0][sl]), torch), dev(np.ascontiguousarray(p[1][sl]), torch),
                             dev(np.ascontiguousarray(p[2][sl]), torch)) for p in bank_np])


def _route(seed, T, E, k):
    rng = np.random.default_rng(seed)
    inds = np.stack([rng.choice(E, size=k, replace=False) for _ in range(T)]).astype(np.int32)
    wts = (0.05 + rng.random((T, k)) * 0.25).astype(np.float32)
    return inds, wts


@pytest.mark.parametrize("T", [1, 6, 19])
@pytest.mark.parametrize("transport", TRANSPORTS)
def test_ep_world1_is_bit_identical_to_moe(sx, transport, T):
    E, D, I, k = 16, 256, 128, 4
    bank_np = _bank_np(40 + T, E, D, I, 32)
    _, dec = dec_args(orc.CB_MCG, 16)
    b = _bank(sx, bank_np)
    xt = torch.from_numpy(synth.activations(T, T, D)).cuda().to(torch.bfloat16)
    inds, wts = _route(T, T, E, k)
    ii, ww = torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda()
    shared = torch.randn((T, D), device="cuda").to(torch.bfloat16)
    gate = torch.randn((T,), device="cuda").to(torch.bfloat16)
    ep = sx.ExpertParallel(sx.ExpertParallel.unique_id(), 1, 0, transport)
    try:
        for kw in ({}, {"shared": shared}, {"shared": shared, "shared_gate": gate}):
            want = sx.moe(xt, b, ii, ww, dec, **kw)
            got = ep.moe(xt, b, E, ii, ww, dec, rows_cap=T, **kw)
            torch.cuda.synchronize()
            assert torch.equal(want, got), kw
        assert sx.device_error() == 0
    finally:
        ep.destroy()


@pytest.mark.parametrize("transport", TRANSPORTS)
def test_ep_world1_spare_capacity_and_skipped_ids(sx, transport):
    """rows_cap above rows (unused places carry sentinel slots) and ids >= E (skipped)."""
    E, D, I, k, T = 8, 256, 128, 3, 5
    bank_np = _bank_np(7, E, D, I, 32)
    _, dec = dec_args(orc.CB_MCG, 16)
    b = _bank(sx, bank_np)
    xt = torch.from_numpy(synth.activations(3, T, D)).cuda().to(torch.float32)
    inds, wts = _route(9, T, E, k)
    inds[1, 2] = E + 5
    ep = sx.ExpertParallel(sx.ExpertParallel.unique_id(), 1, 0, transport)
    try:
        got = to_f32(ep.moe(xt, b, E, torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda(), dec, rows_cap=16))
        want = to_f32(sx.moe(xt, b, torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda(), dec))
    finally:
        ep.destroy()
    assert np.isfinite(got).all()
    assert max_rel(got, want) <= 1e-5


@pytest.mark.parametrize("transport", TRANSPORTS)
def test_ep_refusals(sx, transport):
    E, D, I = 8, 256, 128
    b = _bank(sx, _bank_np(1, E, D, I, 32))
    _, dec = dec_args(orc.CB_MCG, 16)
    ep = sx.ExpertParallel(sx.ExpertParallel.unique_id(), 1, 0, transport)
    x = torch.zeros((4, D), device="cuda", dtype=torch.bfloat16)
    ii = torch.zeros((4, 2), device="cuda", dtype=torch.int32)
    ww = torch.zeros((4, 2), device="cuda")
    try:
        with pytest.raises(sx.Exl3Error) as e:
            ep.moe(x, b, E + 1, ii, ww, dec, rows_cap=4)  # experts_total != world * local experts
        assert e.value.name == "SX_ERR_BAD_SHAPE"
        with pytest.raises(sx.Exl3Error) as e:
            ep.moe(x, b, E, ii, ww, dec, rows_cap=3)  # rows > rows_cap
        assert e.value.name == "SX_ERR_BAD_SHAPE"
        with pytest.raises(sx.Exl3Error) as e:
            ep.moe(x, b, E, ii, ww, dec, rows_cap=4, clamp_limit=200)
        assert e.value.name == "SX_ERR_INVALID_CLAMP"
    finally:
        ep.destroy()


def _ragged_np(seed, D, I):
    """A two-rate layer as the DeepSeek config's routed experts: 6 experts at K1 (n16), 10 at K2."""
    return [(_bank_np(seed, 6, D, I, 16), 16), (_bank_np(seed + 10, 10, D, I, 32), 32)]


def _ragged_slice(sx, groups, e0, e1):
    """The Ragged layer of experts [e0, e1) of a grouped layer (groups cut at the range's ends)."""
    banks, lo = [], 0
    for bank_np, _ in groups:
        E = bank_np[0][0].shape[0]
        a, b = max(e0, lo), min(e1, lo + E)
        if a < b:
            banks.append(_bank(sx, bank_np, a - lo, b - lo))
        lo += E
    return sx.Ragged.from_banks(banks)


@pytest.mark.parametrize("T", [3, 40])
@pytest.mark.parametrize("transport", TRANSPORTS)
def test_ep_ragged_world1_is_bit_identical_to_moe_ragged(sx, transport, T):
    """sx_ep_moe_ragged over a world of one: the same bits as sx_moe_ragged (T=40 takes the
    decode chain per group in both)."""
    D, I, k = 256, 128, 4
    groups = _ragged_np(300 + T, D, I)
    _, dec = dec_args(orc.CB_SPEC1, 15)  # spec1-w15: the table with K1 rows
    rb = _ragged_slice(sx, groups, 0, 16)
    xt = torch.from_numpy(synth.activations(T + 1, T, D)).cuda().to(torch.bfloat16)
    inds, wts = _route(T + 2, T, 16, k)
    ii, ww = torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda()
    shared = torch.randn((T, D), device="cuda").to(torch.bfloat16)
    ep = sx.ExpertParallel(sx.ExpertParallel.unique_id(), 1, 0, transport)
    try:
        for kw in ({}, {"shared": shared}):
            want = sx.moe_ragged(xt, rb, ii, ww, dec, **kw)
            got = ep.moe(xt, rb, 16, ii, ww, dec, rows_cap=T, **kw)
            torch.cuda.synchronize()
            assert torch.equal(want, got), kw
        assert sx.device_error() == 0
    finally:
        ep.destroy()


@pytest.mark.parametrize("T", [1, 6, 20])
@pytest.mark.parametrize("transport", TRANSPORTS)
def test_ep_folded_world1_equals_unfused(sx, transport, T):
    """sx_ep_moe_folded over a world of one: the shared expert, run on the side stream over the
    rank's rows, gives the bits of the unfused composition (its own layer output passed as
    `shared` to sx_ep_moe), gated and ungated; the caller's stream sees the result."""
    E, D, I, k = 16, 256, 128, 4
    bank_np = _bank_np(140 + T, E, D, I, 32)
    sh_np = _bank_np(150 + T, 1, D, I, 32)
    _, dec = dec_args(orc.CB_MCG, 16)
    b, shb = _bank(sx, bank_np), _bank(sx, sh_np)
    xt = torch.from_numpy(synth.activations(T + 2, T, D)).cuda().to(torch.bfloat16)
    inds, wts = _route(T + 3, T, E, k)
    ii, ww = torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda()
    gate = torch.randn((T,), device="cuda").to(torch.bfloat16)
    one_i = torch.zeros((T, 1), dtype=torch.int32, device="cuda")
    one_s = torch.ones((T, 1), device="cuda")
    ep = sx.ExpertParallel(sx.ExpertParallel.unique_id(), 1, 0, transport)
    try:
        for g in (None, gate):
            sh = sx.moe(xt, shb, one_i, one_s, dec)
            want = ep.moe(xt, b, E, ii, ww, dec, rows_cap=T, shared=sh, shared_gate=g)
            got = ep.moe(xt, b, E, ii, ww, dec, rows_cap=T, shared_gate=g, shared_bank=shb)
            torch.cuda.synchronize()
            assert torch.equal(want, got), g is None
        assert sx.device_error() == 0
    finally:
        ep.destroy()


def test_ep_peer_world1_tensor_core_path_matches_nccl(sx):
    """200 tokens on 16 experts take the tensor-core path; 256 places per rank leave 56 unused ones
    that the peer transport's routing skips: the peer and NCCL transports give the same bits, and
    both match sx_moe to its last bit."""
    E, D, I, k, T = 16, 256, 128, 4, 200
    bank_np = _bank_np(500, E, D, I, 32)
    _, dec = dec_args(orc.CB_MCG, 16)
    b = _bank(sx, bank_np)
    xt = torch.from_numpy(synth.activations(501, T, D)).cuda().to(torch.bfloat16)
    inds, wts = _route(502, T, E, k)
    ii, ww = torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda()
    gate = torch.randn((T,), device="cuda").to(torch.bfloat16)
    shb = _bank(sx, _bank_np(503, 1, D, I, 32))
    outs = {}
    for transport in TRANSPORTS:
        ep = sx.ExpertParallel(sx.ExpertParallel.unique_id(), 1, 0, transport)
        try:
            outs[transport] = ep.moe(xt, b, E, ii, ww, dec, rows_cap=256, shared_gate=gate, shared_bank=shb)
            torch.cuda.synchronize()
        finally:
            ep.destroy()
    assert torch.equal(outs["peer"], outs["nccl"])
    want = to_f32(sx.moe_folded(xt, b, shb, ii, ww, dec, shared_gate=gate))
    got = to_f32(outs["peer"])
    assert np.abs(got - want).max() <= 2 ** -7 * np.abs(want).max()
    assert sx.device_error() == 0


def test_ep_peer_world1_host_sized_call(sx):
    """rows_cap >= 1024: the peer transport reads the received counts back and sizes the chain's
    launches to them (the tensor-core path here); the bits equal the NCCL transport's and sx_moe's
    to the last bit."""
    E, D, I, k, T = 16, 256, 128, 4, 1100
    bank_np = _bank_np(800, E, D, I, 32)
    _, dec = dec_args(orc.CB_MCG, 16)
    b = _bank(sx, bank_np)
    xt = torch.from_numpy(synth.activations(801, T, D)).cuda().to(torch.bfloat16)
    inds, wts = _route(802, T, E, k)
    inds[7, 1] = E + 3  # a skipped id
    ii, ww = torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda()
    outs = {}
    for transport in TRANSPORTS:
        ep = sx.ExpertParallel(sx.ExpertParallel.unique_id(), 1, 0, transport)
        try:
            outs[transport] = ep.moe(xt, b, E, ii, ww, dec, rows_cap=1200)
            torch.cuda.synchronize()
        finally:
            ep.destroy()
    assert torch.equal(outs["peer"], outs["nccl"])
    want = to_f32(sx.moe(xt, b, ii, ww, dec))
    got = to_f32(outs["peer"])
    assert np.abs(got - want).max() <= 2 ** -7 * np.abs(want).max()
    assert sx.device_error() == 0


@pytest.mark.parametrize("D,I", [(512, 256), (7168, 2048)])
def test_ep_peer_world1_host_sized_ragged_with_shared(sx, D, I):
    """A host-sized call (rows_cap >= 1024) over a rate-grouped layer (K1 and K2 SPEC1 groups, the
    DeepSeek config's routed layout) with a K4 shared expert on the side stream: the peer and NCCL
    transports give the same bits, and both match the one-GPU folded layer to its last bit."""
    k, T = 8, 1100
    groups = [(_bank_np(900 + D, 4, D, I, 16), 16), (_bank_np(910 + D, 12, D, I, 32), 32)]
    _, dec = dec_args(orc.CB_SPEC1, 15)
    rb = _ragged_slice(sx, groups, 0, 16)
    shb = _bank(sx, _bank_np(920 + D, 1, D, I, 64))
    xt = torch.from_numpy(synth.activations(921, T, D)).cuda().to(torch.bfloat16)
    inds, wts = _route(922, T, 16, k)
    ii, ww = torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda()
    outs = {}
    for transport in TRANSPORTS:
        ep = sx.ExpertParallel(sx.ExpertParallel.unique_id(), 1, 0, transport)
        try:
            outs[transport] = ep.moe(xt, rb, 16, ii, ww, dec, rows_cap=T, shared_bank=shb)
            torch.cuda.synchronize()
        finally:
            ep.destroy()
    assert torch.equal(outs["peer"], outs["nccl"])
    want = to_f32(sx.moe_folded(xt, rb, shb, ii, ww, dec))
    got = to_f32(outs["peer"])
    assert np.abs(got - want).max() <= 2 ** -7 * np.abs(want).max()
    assert sx.device_error() == 0


def test_ep_peer_world1_graph_replays(sx):
    """The peer transport recorded in a CUDA graph after a warm call: every replay (each a new call
    of the communicator, its flags raised anew) gives sx_moe's bits for the inputs of that replay."""
    E, D, I, k, T = 16, 256, 128, 4, 8
    bank_np = _bank_np(600, E, D, I, 32)
    _, dec = dec_args(orc.CB_MCG, 16)
    b = _bank(sx, bank_np)
    inds, wts = _route(601, T, E, k)
    ii, ww = torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda()
    x = torch.zeros((T, D), device="cuda", dtype=torch.bfloat16)
    ep = sx.ExpertParallel(sx.ExpertParallel.unique_id(), 1, 0, "peer")
    stream = torch.cuda.Stream()
    try:
        with torch.cuda.stream(stream):
            ep.moe(x, b, E, ii, ww, dec, rows_cap=T)  # reserves the peer buffer, warms the kernels
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                y = ep.moe(x, b, E, ii, ww, dec, rows_cap=T)
            for rep in range(3):
                x.copy_(torch.from_numpy(synth.activations(610 + rep, T, D)).cuda().to(torch.bfloat16))
                g.replay()
                want = sx.moe(x, b, ii, ww, dec)
                torch.cuda.synchronize()
                assert torch.equal(y, want), rep
            del g
        assert sx.device_error() == 0
    finally:
        torch.cuda.synchronize()
        ep.destroy()


def test_ep_phase_timing_eager_and_in_a_graph(sx):
    """sx_ep_phase_timing: an eager call records its phase events as plain records, a captured call
    as the graph's external records; either way sx_ep_phase_ms gives six finite, non-negative
    durations and the results stay sx_moe's."""
    E, D, I, k, T = 16, 256, 128, 4, 2
    bank_np = _bank_np(620, E, D, I, 32)
    _, dec = dec_args(orc.CB_MCG, 16)
    b = _bank(sx, bank_np)
    inds, wts = _route(621, T, E, k)
    ii, ww = torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda()
    x = torch.from_numpy(synth.activations(622, T, D)).cuda().to(torch.bfloat16)
    ep = sx.ExpertParallel(sx.ExpertParallel.unique_id(), 1, 0, "peer")
    stream = torch.cuda.Stream()
    try:
        with torch.cuda.stream(stream):
            ep.phase_timing(True)
            y = ep.moe(x, b, E, ii, ww, dec, rows_cap=T)
            eager = ep.phase_ms()
            assert torch.equal(y, sx.moe(x, b, ii, ww, dec))
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                y2 = ep.moe(x, b, E, ii, ww, dec, rows_cap=T)
            g.replay()
            graphed = ep.phase_ms()
            torch.cuda.synchronize()
            assert torch.equal(y2, sx.moe(x, b, ii, ww, dec))
            ep.phase_timing(False)
            del g
        for ph in (eager, graphed):
            assert set(ph) == set(sx.ExpertParallel.PHASES)
            assert all(np.isfinite(v) and v >= 0.0 for v in ph.values()), ph
        assert sx.device_error() == 0
    finally:
        torch.cuda.synchronize()
        ep.destroy()


def test_ep_peer_reservation_grows_and_releases(sx):
    """A call larger than the reservation grows it (a collective step of the communicator); a
    reservation of 0 returns the communicator to the NCCL transport; results stay sx_moe's."""
    from sushi_b200 import _lib

    E, D, I, k = 8, 256, 128, 3
    bank_np = _bank_np(700, E, D, I, 32)
    _, dec = dec_args(orc.CB_MCG, 16)
    b = _bank(sx, bank_np)
    ep = sx.ExpertParallel(sx.ExpertParallel.unique_id(), 1, 0, "peer")
    L = _lib.load()
    try:
        sizes = []
        for T in (2, 40):
            xt = torch.from_numpy(synth.activations(701 + T, T, D)).cuda().to(torch.bfloat16)
            inds, wts = _route(702 + T, T, E, k)
            ii, ww = torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda()
            got = ep.moe(xt, b, E, ii, ww, dec, rows_cap=T)
            assert torch.equal(got, sx.moe(xt, b, ii, ww, dec)), T
            sizes.append(ep.peer_reserved())
        assert 0 < sizes[0] <= sizes[1]
        assert L.sx_ep_peer_bytes(ep._h, 40, D, k, 2) <= sizes[1]
        assert L.sx_ep_reserve_peer(ep._h, 0) == 0
        assert ep.peer_reserved() == 0
        ep.transport = "nccl"
        got = ep.moe(xt, b, E, ii, ww, dec, rows_cap=T)
        assert torch.equal(got, sx.moe(xt, b, ii, ww, dec))
        assert sx.device_error() == 0
    finally:
        torch.cuda.synchronize()
        ep.destroy()


# ------------------------------------------------------------------ two GPUs
def _rank_main(rank, world, port, out_dir, transport):
    import torch.distributed as dist

    import sushi_b200 as sx

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        E, D, I, k, T = 16, 256, 128, 4, 7 + 3 * rank
        bank_np = _bank_np(123, E, D, I, 32)
        _, dec = dec_args(orc.CB_MCG, 16)
        El = E // world
        local = _bank(sx, bank_np, rank * El, (rank + 1) * El)
        full = _bank(sx, bank_np)
        xt = torch.from_numpy(synth.activations(50 + rank, T, D)).cuda().to(torch.bfloat16)
        inds, wts = _route(60 + rank, T, E, k)
        ii, ww = torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda()
        ep = sx.ExpertParallel.from_process_group(transport=transport)
        got = to_f32(ep.moe(xt, local, E, ii, ww, dec, rows_cap=16))
        torch.cuda.synchronize()
        ep.destroy()
        want = to_f32(sx.moe(xt, full, ii, ww, dec))
        np.save(os.path.join(out_dir, f"got{rank}.npy"), got)
        np.save(os.path.join(out_dir, f"want{rank}.npy"), want)
        np.save(os.path.join(out_dir, f"x{rank}.npy"), xt.float().cpu().numpy())
        np.save(os.path.join(out_dir, f"inds{rank}.npy"), inds)
        np.save(os.path.join(out_dir, f"wts{rank}.npy"), wts)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("transport", TRANSPORTS)
def test_ep_two_gpus_match_single_gpu(tmp_path, transport):
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_rank_main, args=(2, port, str(tmp_path), transport), nprocs=2, start_method="spawn", join=True)
    E, D, I = 16, 256, 128
    bank_np = _bank_np(123, E, D, I, 32)
    oargs, _ = dec_args(orc.CB_MCG, 16)
    for rank in range(2):
        got = np.load(tmp_path / f"got{rank}.npy")
        want = np.load(tmp_path / f"want{rank}.npy")
        assert np.isfinite(got).all()
        assert np.abs(got - want).max() <= 2 ** -7 * np.abs(want).max(), rank  # a last-bit bf16 difference
        inds, wts = np.load(tmp_path / f"inds{rank}.npy"), np.load(tmp_path / f"wts{rank}.npy")
        x = np.load(tmp_path / f"x{rank}.npy")
        truth = np.zeros((x.shape[0], D))
        for r in range(x.shape[0]):
            for j in range(inds.shape[1]):
                e = int(inds[r, j])
                dense = tuple(orc.decode_dense(p[0][e], p[1][e], p[2][e], a, b_, 32, *oargs)
                              for p, a, b_ in zip(bank_np, (D, D, I), (I, I, D)))
                truth[r] += wts[r, j] * orc.expert_truth(dense, x[r])
        assert max_rel(got, truth) <= MAX_REL_TOL
        assert rel_rms(got, truth) <= REL_RMS_TOL


def _ragged_rank_main(rank, world, port, out_dir, transport):
    import torch.distributed as dist

    import sushi_b200 as sx

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        D, I, k, T = 256, 128, 4, 9 + 4 * rank
        groups = _ragged_np(777, D, I)
        _, dec = dec_args(orc.CB_MCG, 16)
        El = 16 // world
        local = _ragged_slice(sx, groups, rank * El, (rank + 1) * El)  # rank 0: K1 and K2 experts; rank 1: K2
        full = _ragged_slice(sx, groups, 0, 16)
        xt = torch.from_numpy(synth.activations(80 + rank, T, D)).cuda().to(torch.bfloat16)
        inds, wts = _route(90 + rank, T, 16, k)
        ii, ww = torch.from_numpy(inds).cuda(), torch.from_numpy(wts).cuda()
        ep = sx.ExpertParallel.from_process_group(transport=transport)
        got = to_f32(ep.moe(xt, local, 16, ii, ww, dec, rows_cap=16))
        torch.cuda.synchronize()
        ep.destroy()
        want = to_f32(sx.moe_ragged(xt, full, ii, ww, dec))
        np.save(os.path.join(out_dir, f"got{rank}.npy"), got)
        np.save(os.path.join(out_dir, f"want{rank}.npy"), want)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("transport", TRANSPORTS)
def test_ep_ragged_two_gpus_match_single_gpu(tmp_path, transport):
    """A rate-grouped layer split over two GPUs whose local layers differ (rank 0 holds K1 and K2
    experts, rank 1 only K2): each rank's rows match sx_moe_ragged over the full layer to the last
    bf16 bit (rank-order versus k-order sums)."""
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_ragged_rank_main, args=(2, port, str(tmp_path), transport), nprocs=2, start_method="spawn", join=True)
    for rank in range(2):
        got = np.load(tmp_path / f"got{rank}.npy")
        want = np.load(tmp_path / f"want{rank}.npy")
        assert np.isfinite(got).all()
        assert np.abs(got - want).max() <= 2 ** -7 * np.abs(want).max(), rank
