"""The C ABI on the host (no GPU): the library loads, exports every symbol include/sushi_exl3.h
declares, names every status, holds the reference's codebook tables (pinned by their sha256
digests, src/exl3/codebook_tables.zig:281-460), and refuses bad calls by name before touching the
device (src/exl3/root.zig:98-135 admission)."""

import ctypes
import hashlib
import os
import re

import pytest

from sushi_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FAKE = 0x10000  # an aligned, never-dereferenced device address: refusals return before any access


@pytest.fixture(scope="module")
def L():
    return _lib.load()


def test_every_declared_symbol_is_exported(L):
    header = open(os.path.join(ROOT, "include", "sushi_exl3.h")).read()
    declared = set(re.findall(r"^\w[\w\s\*]*?\b(sx_\w+)\(", header, re.M))
    assert {"sx_linear", "sx_moe", "sx_router_topk", "sx_dequant_inner"} <= declared
    for name in declared:
        assert hasattr(L, name), name
    assert set(declared) <= set(_lib.SIGNATURES), "the ctypes binding covers every declared function"


def test_status_names(L):
    names = {i: L.sx_status_name(i).decode() for i in range(0, 20)}
    assert names[0] == "SX_OK"
    assert names[1] == "SX_ERR_BAD_SHAPE"
    assert names[4] == "SX_ERR_TOPK_EXCEEDS_REDUCE_BANK"
    assert names[12] == "SX_ERR_ROUTER_DECLINED"
    assert len(set(names.values())) == 20
    assert L.sx_status_name(999).decode() == "SX_ERR_UNKNOWN"
    assert b"sushi" in L.sx_version()


def _digest(fields, ns, rows):
    h = hashlib.sha256()
    for n, r in zip(ns, rows):
        h.update((str(n) + "".join("," + format(v, "08x") for v in r[:fields]) + "\n").encode())
    return h.hexdigest()[:8]


PINNED = {"pair1-w16-v1": "c089b4eb", "spec1-w15": "37f72431", "spec1-w16": "753ffa03", "std1": "c5dba171",
          "spec1-test-per-rate": "a2f2fe40"}


def test_library_tables_keep_the_reference_digests():
    import sushi_b200 as sx

    for t in range(5):
        info = sx.table_info(t)
        ns = [info["n_lo"] + 2 * i for i in range(info["rows"])]
        rows = [sx.table_row(t, n) for n in ns]
        assert all(r is not None for r in rows)
        assert _digest(info["fields"], ns, rows) == PINNED[info["name"]] == info["digest"], info["name"]
    assert sx.table_row(1, 14) is None and sx.table_row(3, 16) is None and sx.table_row(0, 66) is None


def _proj(in_f=256, out_f=128, n=32, experts=1):
    return _lib.SxProj(FAKE, FAKE, FAKE, experts, in_f, out_f, n, 0)


def _dec(cb=1, w=16, table=-1):
    return _lib.SxDecode(cb, w, table)


@pytest.mark.parametrize(
    "proj,dec,dtype,rows,want",
    [
        (_proj(in_f=200), _dec(), 2, 1, "SX_ERR_BAD_SHAPE"),
        (_proj(out_f=130), _dec(), 2, 1, "SX_ERR_BAD_SHAPE"),
        (_proj(n=31), _dec(), 2, 1, "SX_ERR_TRELLIS_GEOMETRY"),
        (_proj(n=130), _dec(), 2, 1, "SX_ERR_TRELLIS_GEOMETRY"),
        (_proj(), _dec(), 7, 1, "SX_ERR_BAD_DTYPE"),
        (_proj(), _dec(), 2, 0, "SX_ERR_BAD_SHAPE"),
        (_proj(), _dec(w=7), 2, 1, "SX_ERR_WINDOW_UNSUPPORTED"),
        (_proj(), _dec(cb=2), 2, 1, "SX_ERR_CODEBOOK_TABLE_UNKNOWN"),
        (_proj(n=16), _dec(cb=4, table=3), 2, 1, "SX_ERR_CODEBOOK_TABLE_RATE_MISSING"),
        (_proj(), _dec(cb=3, w=15), 2, 1, "SX_ERR_CODEBOOK_TABLE_WINDOW_MISMATCH"),
        (_proj(), _dec(cb=9), 2, 1, "SX_ERR_CODEBOOK_UNSUPPORTED"),
        (_proj(experts=2), _dec(), 2, 1, "SX_ERR_BAD_SHAPE"),
    ],
)
def test_linear_refusals_before_launch(L, proj, dec, dtype, rows, want):
    st = L.sx_linear(None, ctypes.byref(proj), ctypes.byref(dec), FAKE, dtype, rows, FAKE)
    assert L.sx_status_name(st).decode() == want


def test_linear_ex_refuses_unknown_flags(L):
    st = L.sx_linear_ex(None, ctypes.byref(_proj()), ctypes.byref(_dec()), FAKE, 2, 1, FAKE, 2)
    assert L.sx_status_name(st).decode() == "SX_ERR_BAD_SHAPE"


def test_misaligned_trellis_is_refused(L):
    p = _lib.SxProj(FAKE + 2, FAKE, FAKE, 1, 256, 128, 32, 0)
    st = L.sx_linear(None, ctypes.byref(p), ctypes.byref(_dec()), FAKE, 2, 1, FAKE)
    assert L.sx_status_name(st).decode() == "SX_ERR_BAD_SHAPE"


def test_moe_refusals_before_launch(L):
    g = _lib.SxProj(FAKE, FAKE, FAKE, 8, 256, 128, 32, 0)
    d = _lib.SxProj(FAKE, FAKE, FAKE, 8, 128, 256, 32, 0)
    bank = _lib.SxBank(g, g, d)
    dec = _dec()
    call = lambda topk=4, clamp=0, ws=1 << 30, bank=bank: L.sx_status_name(L.sx_moe(
        None, ctypes.byref(bank), ctypes.byref(dec), FAKE, 2, 3, FAKE, FAKE, topk, None, None, clamp, FAKE, FAKE,
        ws)).decode()
    assert call(topk=33) == "SX_ERR_TOPK_EXCEEDS_REDUCE_BANK"
    assert call(topk=9) == "SX_ERR_TOPK_EXCEEDS_EXPERTS"
    assert call(clamp=129) == "SX_ERR_INVALID_CLAMP"
    assert call(ws=16) == "SX_ERR_WORKSPACE_TOO_SMALL"
    bad = _lib.SxBank(g, g, _lib.SxProj(FAKE, FAKE, FAKE, 8, 256, 256, 32, 0))
    assert call(bank=bad) == "SX_ERR_BAD_SHAPE"
    assert L.sx_moe_workspace_bytes(ctypes.byref(bank), 3, 4) > 3 * 4 * (128 * 2 + 256 * 4)


def test_router_declines_before_launch(L):
    st = L.sx_router_topk(None, FAKE, None, 1, 64, 33, 0, 1, 1.0, 0, 0, FAKE, FAKE)
    assert L.sx_status_name(st).decode() == "SX_ERR_ROUTER_DECLINED"
    st = L.sx_router_topk(None, FAKE, None, 1, 4096, 8, 0, 1, 1.0, 0, 0, FAKE, FAKE)
    assert L.sx_status_name(st).decode() == "SX_ERR_ROUTER_DECLINED"
    st = L.sx_router_topk(None, FAKE, None, 1, 64, 8, 1, 1, 1.0, 0, 0, FAKE, FAKE)  # sigmoid without bias
    assert L.sx_status_name(st).decode() == "SX_ERR_ROUTER_DECLINED"
    st = L.sx_router_topk(None, FAKE, FAKE, 1, 64, 8, 2, 1, 1.0, 3, 1, FAKE, FAKE)  # 64 % 3 != 0
    assert L.sx_status_name(st).decode() == "SX_ERR_ROUTER_DECLINED"


def test_router_gate_declines_before_launch(L):
    gate = lambda rows=1, gk=2048, gdt=2, ldt=2: L.sx_status_name(L.sx_router_topk_gate(
        None, FAKE, ldt, None, rows, 512, 10, 0, 1, 1.0, 0, 0, FAKE, FAKE, gk, gdt, FAKE, FAKE, FAKE)).decode()
    assert gate(rows=2) == "SX_ERR_ROUTER_DECLINED"  # src/moe_router.zig:503: one row
    assert gate(gk=12) == "SX_ERR_ROUTER_DECLINED"
    assert gate(gk=16392) == "SX_ERR_ROUTER_DECLINED"
    assert gate(gdt=0) == "SX_ERR_ROUTER_DECLINED"  # F32 gate
    assert gate(ldt=7) == "SX_ERR_ROUTER_DECLINED"  # unknown logits dtype
    st = L.sx_router_topk_gate(None, FAKE, 2, None, 1, 512, 10, 0, 1, 1.0, 0, 0, FAKE, None, 2048, 2, FAKE, FAKE, FAKE)
    assert L.sx_status_name(st).decode() == "SX_ERR_NULL_POINTER"


def test_router_gate_logit_oracle_is_a_dot():
    """The restated MLX order is a dot product: within f32 rounding of the f64 sum."""
    import numpy as np

    from oracle import oracle as orc

    rng = np.random.default_rng(3)
    for gk in (8, 1032, 2048, 7168):
        x = rng.standard_normal(gk).astype(np.float32)
        w = rng.standard_normal(gk).astype(np.float32)
        got = float(orc.router_gate_logit(x, w))
        want = float(np.dot(x.astype(np.float64), w.astype(np.float64)))
        bound = gk * 2.0 ** -23 * float(np.abs(x.astype(np.float64) * w).sum())
        assert abs(got - want) <= bound


class SxRaggedMeta:
    """A host meta table for sx_ragged (8 u32 words per expert)."""

    def __init__(self, rows):
        import numpy as np

        self.arr = np.ascontiguousarray(np.array(rows, np.uint32))


def _ragged(meta_rows, experts=None, hidden=256, inter=128):
    m = SxRaggedMeta(meta_rows)
    r = _lib.SxRagged()
    for p in range(3):
        r.trellis[p] = FAKE
        r.suh[p] = FAKE
        r.svh[p] = FAKE
    r.meta = m.arr.ctypes.data
    r.experts = len(meta_rows) if experts is None else experts
    r.hidden, r.inter = hidden, inter
    return r, m


def test_ragged_meta_admission(L):
    """sx_moe_ragged reads the groups from the host meta table before any device work: groups must
    be runs of experts with one rate per projection and tiles at the rate's stride."""
    tiles = (256 // 16) * (128 // 16)
    good = [[16, 16, 32, 0, e * tiles * 16 // 2, e * tiles * 16 // 2, e * tiles * 32 // 2, e] for e in range(2)]
    good += [[32, 32, 32, 1, 2 * tiles * 8 + e * tiles * 16, 2 * tiles * 8 + e * tiles * 16,
              2 * tiles * 16 + e * tiles * 16, e] for e in range(3)]
    r, keep = _ragged(good)
    assert L.sx_moe_ragged_workspace_bytes(ctypes.byref(r), 4, 2) > 0
    bad_stride = [row[:] for row in good]
    bad_stride[1][4] += 2
    bad_rate = [row[:] for row in good]
    bad_rate[3][2] = 48
    bad_local = [row[:] for row in good]
    bad_local[2][7] = 1
    for rows in (bad_stride, bad_rate, bad_local):
        r, keep = _ragged(rows)
        assert L.sx_moe_ragged_workspace_bytes(ctypes.byref(r), 4, 2) == 0
        st = L.sx_moe_ragged(None, ctypes.byref(r), ctypes.byref(_dec()), FAKE, 2, 4, FAKE, FAKE, 2, None, None, 0,
                             FAKE, FAKE, 1 << 30)
        assert L.sx_status_name(st).decode() == "SX_ERR_GROUP_GEOMETRY"
    mixed = [row[:] for row in good]
    for row in mixed[:2]:
        row[1] = 24  # up rate differs from gate within the group
        row[5] = row[7] * tiles * 24 // 2
    r, keep = _ragged(mixed)
    st = L.sx_moe_ragged(None, ctypes.byref(r), ctypes.byref(_dec()), FAKE, 2, 4, FAKE, FAKE, 2, None, None, 0, FAKE,
                         FAKE, 1 << 30)
    assert L.sx_status_name(st).decode() == "SX_ERR_TRELLIS_GEOMETRY"


def test_selftest_limit_is_checked_before_launch(L):
    for bad in (0, -5, 2001):
        assert L.sx_status_name(L.sx_selftest_wait_timeout(None, bad)).decode() == "SX_ERR_BAD_SHAPE"


def test_linear_shared_normed_admission(L):
    """linearSharedNormed serves one bank, <= 16 rows, out <= 4096 (project_rows.zig:914-919) and
    needs its counter workspace; each refusal comes before any launch."""
    cols = (ctypes.c_int32 * 3)(0, 128, 256)
    ys = (ctypes.c_void_p * 2)(FAKE, FAKE)
    p = _proj(in_f=256, out_f=256)
    need = L.sx_linear_shared_normed_workspace_bytes(ctypes.byref(p))
    assert need == 16 + 16 * 2 * 4

    def call(proj=p, rows=1, w=FAKE, eps=1e-6, ws=FAKE, wsb=need, c=cols, count=2):
        st = L.sx_linear_shared_normed(None, ctypes.byref(proj), c, count, ctypes.byref(_dec()), FAKE, 2, rows, ys, w,
                                       eps, ws, wsb)
        return L.sx_status_name(st).decode()

    assert call(rows=17) == "SX_ERR_BAD_SHAPE"
    assert call(w=None) == "SX_ERR_NULL_POINTER"
    assert call(ws=None) == "SX_ERR_NULL_POINTER"
    assert call(wsb=need - 1) == "SX_ERR_WORKSPACE_TOO_SMALL"
    assert call(ws=FAKE + 8) == "SX_ERR_BAD_SHAPE"
    assert call(eps=-1.0) == "SX_ERR_BAD_SHAPE"
    assert call(eps=float("nan")) == "SX_ERR_BAD_SHAPE"
    assert call(proj=_proj(in_f=256, out_f=256, experts=2)) == "SX_ERR_BAD_SHAPE"
    wide = _proj(in_f=256, out_f=4224)
    wcols = (ctypes.c_int32 * 2)(0, 4224)
    assert call(proj=wide, c=wcols, count=1, wsb=1 << 20) == "SX_ERR_BAD_SHAPE"
    bad = (ctypes.c_int32 * 3)(0, 100, 256)
    assert call(c=bad) == "SX_ERR_BAD_SHAPE"


def test_moe_folded_refusals_before_launch(L):
    """The shared expert of sx_moe_folded is one SwiGLU expert over the layer's hidden size."""
    g = _lib.SxProj(FAKE, FAKE, FAKE, 8, 256, 128, 32, 0)
    d = _lib.SxProj(FAKE, FAKE, FAKE, 8, 128, 256, 32, 0)
    bank = _lib.SxBank(g, g, d)
    sg = _lib.SxProj(FAKE, FAKE, FAKE, 1, 256, 128, 32, 0)
    sd = _lib.SxProj(FAKE, FAKE, FAKE, 1, 128, 256, 32, 0)
    shared = _lib.SxBank(sg, sg, sd)
    dec = _dec()
    need = L.sx_moe_folded_workspace_bytes(ctypes.byref(bank), ctypes.byref(shared), ctypes.byref(dec), None, 4, 2)
    assert need > L.sx_moe_workspace_bytes(ctypes.byref(bank), 4, 2)

    def call(sh=shared, wsb=need):
        st = L.sx_moe_folded(None, ctypes.byref(bank), ctypes.byref(sh) if sh is not None else None,
                             ctypes.byref(dec), None, FAKE, 2, 4, FAKE, FAKE, 2, None, 0, FAKE, FAKE, wsb)
        return L.sx_status_name(st).decode()

    assert call(sh=None) == "SX_ERR_NULL_POINTER"
    two = _lib.SxBank(_lib.SxProj(FAKE, FAKE, FAKE, 2, 256, 128, 32, 0), _lib.SxProj(FAKE, FAKE, FAKE, 2, 256, 128, 32, 0),
                      _lib.SxProj(FAKE, FAKE, FAKE, 2, 128, 256, 32, 0))
    assert call(sh=two) == "SX_ERR_BAD_SHAPE"
    wide = _lib.SxBank(_lib.SxProj(FAKE, FAKE, FAKE, 1, 512, 128, 32, 0), _lib.SxProj(FAKE, FAKE, FAKE, 1, 512, 128, 32, 0),
                       _lib.SxProj(FAKE, FAKE, FAKE, 1, 128, 512, 32, 0))
    assert call(sh=wide) == "SX_ERR_BAD_SHAPE"
    assert call(wsb=need - 1) == "SX_ERR_WORKSPACE_TOO_SMALL"
