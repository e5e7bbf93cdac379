"""Expert-parallel host logic on the CPU, as world-size-2 gloo process groups.

* share_unique_id: rank 0's sx_ep_unique_id reaches every rank intact (the library call runs on
  the host; sx_ep_init itself needs GPUs and runs in tests/test_gpu_ep.py).
* The dispatch / combine protocol of sx_ep_moe (sushi_b200/csrc/sx_ep.cu), restated in numpy
  with the blocks exchanged by gloo all-to-alls of the same fixed size (rows_cap rows per peer):
  each rank lists, per destination, its rows with a slot there (pos[r][d] = place or -1), sends
  the rows with destination-local ids and the sentinel elsewhere, the destination runs its
  experts over every received place, and the owner adds the returned partials in rank order.
  The result must equal the single-process routed sum over the full expert set.
* sx_ep_* argument refusals that happen before any device work.
"""

import ctypes
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
dist = pytest.importorskip("torch.distributed")

SENTINEL = 0xFFFFFFFF


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(fn, world, *args):
    import torch.multiprocessing as mp

    mp.start_processes(fn, args=(world, _free_port()) + args, nprocs=world, start_method="spawn", join=True)


def _init(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)


# ------------------------------------------------------------------ unique id
def _id_main(rank, world, port, out_dir):
    import sushi_b200 as sx

    _init(rank, world, port)
    try:
        uid = sx.share_unique_id()
        with open(os.path.join(out_dir, f"id{rank}"), "wb") as f:
            f.write(uid)
    finally:
        dist.destroy_process_group()


def test_share_unique_id_gloo(tmp_path):
    _spawn(_id_main, 2, str(tmp_path))
    ids = [open(tmp_path / f"id{r}", "rb").read() for r in range(2)]
    assert len(ids[0]) == 128 and ids[0] == ids[1] and any(ids[0])


# ------------------------------------------------------------------ protocol
E, D, K, WORLD = 12, 16, 3, 2


def _experts():
    rng = np.random.default_rng(5)
    return rng.standard_normal((E, D, D)) / np.sqrt(D)


def _rows(rank):
    rng = np.random.default_rng(100 + rank)
    T = 4 + 3 * rank
    x = rng.standard_normal((T, D))
    inds = np.stack([rng.choice(E, size=K, replace=False) for _ in range(T)]).astype(np.uint32)
    inds[0, 1] = E + 2  # an id past the experts: skipped
    scores = rng.random((T, K))
    return x, inds, scores


def _routed(W, x, inds, scores, e_lo=0, e_hi=E):
    """k-order sum of score * expert(x) over the slots whose expert lies in [e_lo, e_hi)."""
    y = np.zeros_like(x)
    for r in range(x.shape[0]):
        for k in range(inds.shape[1]):
            e = int(inds[r, k])
            if e_lo <= e < e_hi:
                y[r] += scores[r, k] * (W[e] @ x[r])
    return y


def _ep_main(rank, world, port, cap, out_dir):
    _init(rank, world, port)
    try:
        W = _experts()
        El = E // world
        x, inds, scores = _rows(rank)
        T = x.shape[0]
        # plan + gather (ep_plan_kernel, ep_gather_kernel)
        pos = np.full((T, world), -1)
        send_x = np.zeros((world, cap, D))
        send_i = np.full((world, cap, K), SENTINEL, np.int64)
        send_s = np.zeros((world, cap, K))
        for d in range(world):
            place = 0
            for r in range(T):
                here = [(int(e) < E and int(e) // El == d) for e in inds[r]]
                if any(here):
                    pos[r, d] = place
                    send_x[d, place] = x[r]
                    send_i[d, place] = [int(e) - d * El if h else SENTINEL for e, h in zip(inds[r], here)]
                    send_s[d, place] = np.where(here, scores[r], 0.0)
                    place += 1
            assert place <= cap
        # dispatch: fixed-size all-to-alls
        recv = []
        for a in (send_x, send_i, send_s):
            t_in = torch.from_numpy(np.ascontiguousarray(a))
            t_out = torch.empty_like(t_in)
            dist.all_to_all_single(t_out, t_in)
            recv.append(t_out.numpy())
        rx, ri, rs = recv
        # local experts over every place: partial = k-order sum over the place's local slots
        Wl = W[rank * El:(rank + 1) * El]
        part = _routed(Wl, rx.reshape(-1, D), ri.reshape(-1, K), rs.reshape(-1, K), 0, El).reshape(world, cap, D)
        # combine: partials back, added in rank order by the owner
        t_in = torch.from_numpy(np.ascontiguousarray(part))
        back = torch.empty_like(t_in)
        dist.all_to_all_single(back, t_in)
        back = back.numpy()
        y = np.zeros((T, D))
        for r in range(T):
            for d in range(world):
                if pos[r, d] >= 0:
                    y[r] += back[d, pos[r, d]]
        np.save(os.path.join(out_dir, f"y{rank}.npy"), y)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("cap", [10, 16])
def test_ep_protocol_matches_single_process(tmp_path, cap):
    _spawn(_ep_main, WORLD, cap, str(tmp_path))
    W = _experts()
    for rank in range(WORLD):
        x, inds, scores = _rows(rank)
        want = _routed(W, x, inds, scores)
        got = np.load(tmp_path / f"y{rank}.npy")
        np.testing.assert_allclose(got, want, rtol=1e-12, atol=1e-12)


# ------------------------------------------------------------------ refusals before device work
@pytest.fixture(scope="module")
def L():
    from sushi_b200 import _lib

    return _lib.load()


def test_ep_init_refuses_bad_rank(L):
    buf = (ctypes.c_uint8 * 128)()
    h = ctypes.c_void_p()
    for world, rank in ((0, 0), (2, 2), (2, -1)):
        assert L.sx_status_name(L.sx_ep_init(buf, world, rank, ctypes.byref(h))).decode() == "SX_ERR_BAD_SHAPE"
    assert L.sx_status_name(L.sx_ep_init(None, 1, 0, ctypes.byref(h))).decode() == "SX_ERR_NULL_POINTER"


def test_ep_calls_refuse_null_handles(L):
    for name in ("sx_ep_destroy", "sx_ep_abort"):
        assert L.sx_status_name(getattr(L, name)(None)).decode() == "SX_ERR_NULL_POINTER"
    assert L.sx_ep_workspace_bytes(None, None, 4, 2, 2) == 0
    st = L.sx_ep_moe(None, None, None, 8, None, None, 2, 1, 1, None, None, 1, None, None, 0, None, None, 0)
    assert L.sx_status_name(st).decode() == "SX_ERR_NULL_POINTER"
    assert L.sx_status_name(L.sx_ep_unique_id(None)).decode() == "SX_ERR_NULL_POINTER"
