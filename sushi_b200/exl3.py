"""Host-side mirror of the reference's `sushi_exl3` module surface, over the CUDA C ABI.

Names, argument meaning and refusals follow the reference (beamivalice/sushi 1.7.2):
  Decode / Codebook / Rate          src/exl3/expert_exl3.zig:54-226
  Proj / Bank                       src/exl3/root.zig:30-39
  linear / linear_grouped           src/exl3/linear.zig:27-54
  moe / moe_with_shared / moe_with_gated_shared / moe_clamped
                                    src/exl3/root.zig:51-125
  router_topk                       src/moe_router.zig:442 (moeRouterTopK)
  dequant_inner                     src/exl3/expert_exl3.zig:416 (reconstructInner)
A refusal raises `Exl3Error` whose `.name` is the status name mirroring the reference's error
(e.g. "SX_ERR_BAD_SHAPE" for error.BadExl3Shape).  Tensors are torch CUDA tensors: torch is the
device-memory plumbing here, the arithmetic runs in libsushi_exl3_cuda.so.
"""

import ctypes
import enum
from dataclasses import dataclass
from typing import Optional

import numpy as np

import torch

from . import _lib

TILE = 16
HAD_DIM = 128


class Codebook(enum.IntEnum):
    MUL1 = 0
    MCG = 1
    SPEC1 = 2
    PAIR1 = 3
    STD1 = 4

    @classmethod
    def from_name(cls, name):
        return {"mul1": cls.MUL1, "mcg": cls.MCG, "spec1": cls.SPEC1, "pair1": cls.PAIR1, "std1": cls.STD1}.get(name)

    def tabled_hash_mask(self):
        return self in (Codebook.SPEC1, Codebook.STD1)

    def has_table(self):
        return self.tabled_hash_mask() or self == Codebook.PAIR1


TABLES = ("pair1-w16-v1", "spec1-w15", "spec1-w16", "std1", "spec1-test-per-rate")


def table_index(name):
    return TABLES.index(name)


@dataclass(frozen=True)
class Decode:
    """format.Decode: codebook, codeword window (8..16; 16 masks nothing) and the STQ table."""

    codebook: Codebook
    window_bits: int = 16
    table: Optional[int] = None

    @staticmethod
    def tabled(codebook, window_bits=16):
        """Decode.tabled (src/exl3/expert_exl3.zig:152): SPEC1 under spec1-w15, STD1 under std1."""
        t = {Codebook.SPEC1: table_index("spec1-w15"), Codebook.STD1: table_index("std1")}.get(Codebook(codebook))
        return Decode(Codebook(codebook), window_bits, t)

    def c(self):
        return _lib.SxDecode(int(self.codebook), int(self.window_bits), -1 if self.table is None else int(self.table))


class TileOrder(enum.IntEnum):
    PACK = 0
    PAIR_MAJOR = 1


@dataclass
class Proj:
    """root.Proj: trellis U16 [E, in/16, out/16, n], suh F16 [E, in], svh F16 [E, out] (torch CUDA).
    A 3-D trellis / 1-D scales are a one-bank projection."""

    trellis: torch.Tensor
    suh: torch.Tensor
    svh: torch.Tensor
    tile_order: TileOrder = TileOrder.PACK

    def dims(self):
        t = self.trellis
        if self.tile_order == TileOrder.PAIR_MAJOR:
            if t.dim() != 5 or t.shape[3] != 2:
                raise Exl3Error(19)
            return t.shape[0], t.shape[2] * 16, t.shape[1] * 32, t.shape[4]
        if t.dim() == 3:
            return 1, t.shape[0] * 16, t.shape[1] * 16, t.shape[2]
        if t.dim() != 4:
            raise Exl3Error(1)
        return t.shape[0], t.shape[1] * 16, t.shape[2] * 16, t.shape[3]

    def c(self, suh_rows: int = 1):
        """The C struct; `suh_rows` suh rows per bank (stacked linears carry one per linear)."""
        experts, in_f, out_f, n = self.dims()
        for a in (self.trellis, self.suh, self.svh):
            if not a.is_cuda or not a.is_contiguous():
                raise Exl3Error(1)
        if self.trellis.dtype not in (torch.uint16, torch.int16) or self.suh.dtype not in (torch.float16, torch.uint16, torch.int16) \
                or self.svh.dtype not in (torch.float16, torch.uint16, torch.int16):
            raise Exl3Error(2)
        if self.suh.numel() != experts * in_f * suh_rows or self.svh.numel() != experts * out_f:
            raise Exl3Error(1)
        return _lib.SxProj(self.trellis.data_ptr(), self.suh.data_ptr(), self.svh.data_ptr(), experts, in_f, out_f, n,
                           int(self.tile_order))


@dataclass
class Bank:
    gate: Proj
    up: Proj
    down: Proj

    def c(self):
        return _lib.SxBank(self.gate.c(), self.up.c(), self.down.c())


class Exl3Error(RuntimeError):
    def __init__(self, status):
        self.status = int(status)
        L = _lib.load()
        self.name = L.sx_status_name(self.status).decode()
        detail = L.sx_last_error_detail().decode() if self.name in ("SX_ERR_CUDA", "SX_ERR_NCCL") else ""
        super().__init__(f"{self.name} ({detail})" if detail else self.name)


_DT = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def _check(status):
    if status != 0:
        raise Exl3Error(status)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def lib():
    return _lib.load()


LINEAR_WEIGHTS_STATIC = 1


def linear(x, proj: Proj, dec: Decode, flags: int = 0, out=None):
    """linear.linear: x [rows, in] (bf16/f16/f32) through the one-bank proj -> [rows, out] in x's dtype.

    flags: LINEAR_WEIGHTS_STATIC when nothing queued just before this call writes the projection's
    weights (the launch may then stream them while the previous kernel finishes).  out: an optional
    preallocated [rows, out] tensor of x's dtype."""
    if x.dim() != 2 or not x.is_contiguous():
        raise Exl3Error(1)
    if x.dtype not in _DT:
        raise Exl3Error(2)
    _, in_f, out_f, _ = proj.dims()
    if x.shape[1] != in_f:
        raise Exl3Error(1)
    if out is None:
        y = torch.empty((x.shape[0], out_f), dtype=x.dtype, device=x.device)
    else:
        if out.shape != (x.shape[0], out_f) or out.dtype != x.dtype or not out.is_contiguous():
            raise Exl3Error(1)
        y = out
    p, d = proj.c(), dec.c()
    if flags:
        _check(lib().sx_linear_ex(_stream(), ctypes.byref(p), ctypes.byref(d), x.data_ptr(), _DT[x.dtype], x.shape[0],
                                  y.data_ptr(), flags))
    else:
        _check(lib().sx_linear(_stream(), ctypes.byref(p), ctypes.byref(d), x.data_ptr(), _DT[x.dtype], x.shape[0],
                               y.data_ptr()))
    return y


def linear_gemm(x, proj: Proj, dec: Decode, workspace=None):
    """sx_linear_gemm: the many-row projection on the tensor cores (tcgen05), same result bar as
    linear; x [rows, in] -> [rows, out] in x's dtype."""
    if x.dim() != 2 or not x.is_contiguous():
        raise Exl3Error(1)
    if x.dtype not in _DT:
        raise Exl3Error(2)
    _, in_f, out_f, _ = proj.dims()
    if x.shape[1] != in_f:
        raise Exl3Error(1)
    y = torch.empty((x.shape[0], out_f), dtype=x.dtype, device=x.device)
    p, d = proj.c(), dec.c()
    need = lib().sx_linear_gemm_workspace_bytes(ctypes.byref(p), x.shape[0])
    ws = workspace if workspace is not None else _workspace(need, x.device)
    _check(lib().sx_linear_gemm(_stream(), ctypes.byref(p), ctypes.byref(d), x.data_ptr(), _DT[x.dtype], x.shape[0],
                                y.data_ptr(), ws.data_ptr(), ws.numel()))
    return y


def linear_shared(x, proj: Proj, cols, dec: Decode):
    """linear.linearShared: the linears stacked along the output of `proj` (suh holds one row per
    linear) over the same rows x [rows, in]; linear s owns columns cols[s]..cols[s+1].  Returns the
    list of [rows, cols[s+1]-cols[s]] outputs in x's dtype."""
    if x.dim() != 2 or not x.is_contiguous():
        raise Exl3Error(1)
    if x.dtype not in _DT:
        raise Exl3Error(2)
    count = len(cols) - 1
    outs = [torch.empty((x.shape[0], cols[i + 1] - cols[i]), dtype=x.dtype, device=x.device) for i in range(count)]
    c = (ctypes.c_int32 * len(cols))(*cols)
    ys = (ctypes.c_void_p * count)(*[o.data_ptr() for o in outs])
    p, d = proj.c(count), dec.c()
    _check(lib().sx_linear_shared(_stream(), ctypes.byref(p), c, count, ctypes.byref(d), x.data_ptr(), _DT[x.dtype],
                                  x.shape[0], ys))
    return outs


def linear_shared_normed(x, proj: Proj, cols, dec: Decode, norm_w, eps: float, workspace=None):
    """linear.linearSharedNormed: linear_shared whose first linear leaves RMS-normed with weight
    norm_w [cols[1]] (x's dtype) and epsilon eps, in the same launch.  rows 1..16, out <= 4096.
    `workspace` (optional): a zeroed uint8 device tensor of
    linear_shared_normed_workspace_bytes(proj) bytes, reused across calls on one stream (each call
    leaves it zeroed)."""
    if x.dim() != 2 or not x.is_contiguous():
        raise Exl3Error(1)
    if x.dtype not in _DT:
        raise Exl3Error(2)
    if norm_w.dtype != x.dtype or not norm_w.is_contiguous() or norm_w.numel() != cols[1]:
        raise Exl3Error(1)
    count = len(cols) - 1
    p, d = proj.c(count), dec.c()
    need = lib().sx_linear_shared_normed_workspace_bytes(ctypes.byref(p))
    if workspace is None:
        workspace = torch.zeros(need, dtype=torch.uint8, device=x.device)
    outs = [torch.empty((x.shape[0], cols[i + 1] - cols[i]), dtype=x.dtype, device=x.device) for i in range(count)]
    c = (ctypes.c_int32 * len(cols))(*cols)
    ys = (ctypes.c_void_p * count)(*[o.data_ptr() for o in outs])
    _check(lib().sx_linear_shared_normed(_stream(), ctypes.byref(p), c, count, ctypes.byref(d), x.data_ptr(),
                                         _DT[x.dtype], x.shape[0], ys, norm_w.data_ptr(), float(eps),
                                         workspace.data_ptr(), workspace.numel()))
    return outs


def linear_shared_normed_workspace_bytes(proj: Proj) -> int:
    p = proj.c(proj.suh.numel() // max(1, proj.dims()[1]))
    return lib().sx_linear_shared_normed_workspace_bytes(ctypes.byref(p))


def linear_grouped(x, proj: Proj, dec: Decode):
    """linear.linearGrouped: x [G, rows, in] through the G-bank proj (bank g serves x[g]) -> [G, rows, out]."""
    if x.dim() != 3 or not x.is_contiguous():
        raise Exl3Error(1)
    if x.dtype not in _DT:
        raise Exl3Error(2)
    experts, in_f, out_f, _ = proj.dims()
    if x.shape[0] != experts or x.shape[2] != in_f:
        raise Exl3Error(1)
    y = torch.empty((x.shape[0], x.shape[1], out_f), dtype=x.dtype, device=x.device)
    p, d = proj.c(), dec.c()
    _check(lib().sx_linear_grouped(_stream(), ctypes.byref(p), ctypes.byref(d), x.data_ptr(), _DT[x.dtype],
                                   x.shape[1], y.data_ptr()))
    return y


def dequant_inner(proj: Proj, expert: int, dec: Decode):
    """reconstructInner on the device: the [in, out] f16 inner matrix of one expert, as int16 bits."""
    _, in_f, out_f, _ = proj.dims()
    out = torch.empty((in_f, out_f), dtype=torch.int16, device=proj.trellis.device)
    p, d = proj.c(), dec.c()
    _check(lib().sx_dequant_inner(_stream(), ctypes.byref(p), expert, ctypes.byref(d), out.data_ptr()))
    return out


def tile_order_convert(trellis, to_order: "TileOrder", from_order: "TileOrder" = None):
    """layout.tileMajor / tileMajorInverse on the device: a [E, IT, OT, n] pack-order trellis to the
    pair-major order (stored as [E, OT/2, IT, 2, n]) or back; returns a new tensor."""
    from_order = TileOrder.PACK if from_order is None else TileOrder(from_order)
    t = trellis.contiguous()
    if t.dim() == 4:
        E, IT, OT, n = t.shape
    elif t.dim() == 5:
        E, P, IT, two, n = t.shape
        OT = 2 * P
    else:
        raise Exl3Error(1)
    out_shape = (E, OT // 2, IT, 2, n) if TileOrder(to_order) == TileOrder.PAIR_MAJOR else (E, IT, OT, n)
    dst = torch.empty(out_shape, dtype=t.dtype, device=t.device)
    _check(lib().sx_tile_order_convert(_stream(), t.data_ptr(), dst.data_ptr(), E, IT * 16, OT * 16, n, int(from_order),
                                       int(to_order)))
    return dst


def decode_codewords(n: int, dec: Decode, device="cuda"):
    """Every codeword's decode at rate n (int32: weight bits low, PAIR1's partner high)."""
    out = torch.empty(65536, dtype=torch.int32, device=device)
    d = dec.c()
    _check(lib().sx_decode_codewords(_stream(), n, ctypes.byref(d), out.data_ptr()))
    return out


class RouterMode(enum.IntEnum):
    SOFTMAX = 0
    SIGMOID_BIAS = 1
    SIGMOID_BIAS_GROUPED = 2


def router_topk(logits, k, mode=RouterMode.SOFTMAX, bias=None, route_norm=True, route_scale=1.0, n_group=0,
                topk_group=0):
    """moeRouterTopK: logits [..., E] f32 -> (inds [..., k] int32, scores [..., k] f32), or None where the
    reference's fused kernel declines (the caller keeps its own chain)."""
    lg = logits.reshape(-1, logits.shape[-1]).contiguous()
    if lg.dtype != torch.float32:
        lg = lg.float()
    rows, experts = lg.shape
    inds = torch.empty((rows, k), dtype=torch.int32, device=lg.device)
    scores = torch.empty((rows, k), dtype=torch.float32, device=lg.device)
    b = None if bias is None else bias.float().contiguous()
    st = lib().sx_router_topk(_stream(), lg.data_ptr(), None if b is None else b.data_ptr(), rows, experts, k, int(mode),
                              1 if route_norm else 0, float(route_scale), n_group, topk_group, inds.data_ptr(),
                              scores.data_ptr())
    if st == 12:  # SX_ERR_ROUTER_DECLINED
        return None
    _check(st)
    shape = tuple(logits.shape[:-1]) + (k,)
    return inds.reshape(shape), scores.reshape(shape)


def router_topk_gate(logits, k, gate=None, mode=RouterMode.SOFTMAX, bias=None, route_norm=True, route_scale=1.0,
                     n_group=0, topk_group=0):
    """moeRouterTopKGate: router_topk over logits [..., E] of any activation dtype and, in the softmax
    mode with `gate` = (x [K], w [K]) of one F16/BF16 dtype, the shared-expert gate's logit computed
    in the same launch (the reference's softmax_gate).  Returns (inds, scores, gate_logit [1] in the
    gate's dtype, or None without a gate), or None where the reference's kernel declines."""
    if logits.dtype not in _DT:
        raise TypeError(f"BadExl3Dtype: router logits dtype {logits.dtype}")
    lg = logits.reshape(-1, logits.shape[-1]).contiguous()
    rows, experts = lg.shape
    inds = torch.empty((rows, k), dtype=torch.int32, device=lg.device)
    scores = torch.empty((rows, k), dtype=torch.float32, device=lg.device)
    b = None if bias is None else bias.float().contiguous()
    gx = gw = glog = None
    gk, gdt = 0, 2
    if gate is not None and mode == RouterMode.SOFTMAX:
        gx, gw = (t.reshape(-1).contiguous() for t in gate)
        if gx.dtype not in (torch.float16, torch.bfloat16) or gw.dtype != gx.dtype:
            return None
        gk, gdt = gx.numel(), _DT[gx.dtype]
        glog = torch.empty((1,), dtype=gx.dtype, device=lg.device)
    st = lib().sx_router_topk_gate(_stream(), lg.data_ptr(), _DT[lg.dtype], None if b is None else b.data_ptr(), rows,
                                   experts, k, int(mode), 1 if route_norm else 0, float(route_scale), n_group,
                                   topk_group, None if gx is None else gx.data_ptr(),
                                   None if gw is None else gw.data_ptr(), gk, gdt,
                                   None if glog is None else glog.data_ptr(), inds.data_ptr(), scores.data_ptr())
    if st == 12:  # SX_ERR_ROUTER_DECLINED
        return None
    _check(st)
    shape = tuple(logits.shape[:-1]) + (k,)
    return inds.reshape(shape), scores.reshape(shape), glog


_WS_CACHE = {}


def _workspace(nbytes, device):
    key = (str(device),)
    ws = _WS_CACHE.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
        _WS_CACHE[key] = ws
    return ws


def moe(x, bank: Bank, inds, scores, dec: Decode, shared=None, shared_gate=None, clamp_limit=0, workspace=None):
    """root.moe (and its shared / gated-shared / clamped forms): routed SwiGLU experts over x [..., D]
    for top-k inds/scores [..., K]; returns x's shape and dtype."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]).contiguous()
    rows = x2.shape[0]
    ix = inds.reshape(rows, -1).to(torch.int32).contiguous()
    sc = scores.reshape(rows, -1).float().contiguous()
    topk = ix.shape[1]
    if sc.shape != ix.shape:
        raise Exl3Error(1)
    if x2.dtype not in _DT:
        raise Exl3Error(2)
    b = bank.c()
    need = lib().sx_moe_workspace_bytes(ctypes.byref(b), rows, topk)
    ws = workspace if workspace is not None else _workspace(need, x.device)
    y = torch.empty_like(x2)
    d = dec.c()
    sh = None if shared is None else shared.reshape(rows, -1).to(x2.dtype).contiguous()
    sg = None if shared_gate is None else shared_gate.reshape(rows).to(x2.dtype).contiguous()
    _check(lib().sx_moe(_stream(), ctypes.byref(b), ctypes.byref(d), x2.data_ptr(), _DT[x2.dtype], rows, ix.data_ptr(),
                        sc.data_ptr(), topk, None if sh is None else sh.data_ptr(),
                        None if sg is None else sg.data_ptr(), int(clamp_limit), y.data_ptr(), ws.data_ptr(),
                        ws.numel()))
    return y.reshape(shape)


class Ragged:
    """rate_groups.Ragged (src/exl3/rate_groups.zig:23-130): a layer of rate groups held as one flat
    trellis per projection, scales concatenated over all experts, and the 8-word per-expert meta
    table (gate/up/down n, group, tile offsets in u32 words, index in group).  `from_banks` builds it
    from the groups' Banks in order, as Ragged.init does; expert ids run over the groups in order."""

    def __init__(self, trellis, suh, svh, meta, hidden, inter):
        self.trellis, self.suh, self.svh = list(trellis), list(suh), list(svh)
        self.meta = meta.astype(np.uint32).reshape(-1, 8)  # host table
        self.hidden, self.inter = int(hidden), int(inter)
        self.experts = self.meta.shape[0]

    @classmethod
    def from_banks(cls, banks):
        hidden = banks[0].gate.trellis.shape[1] * 16
        inter = banks[0].gate.trellis.shape[2] * 16
        tiles = (hidden // 16) * (inter // 16)
        meta, words = [], [0, 0, 0]
        for g, b in enumerate(banks):
            projs = (b.gate, b.up, b.down)
            rates = [int(p.trellis.shape[3]) for p in projs]
            E = int(b.gate.trellis.shape[0])
            for local in range(E):
                meta.append(rates + [g] + [words[p] + local * tiles * rates[p] // 2 for p in range(3)] + [local])
            for p in range(3):
                words[p] += E * tiles * rates[p] // 2
        flat = [torch.cat([(b.gate, b.up, b.down)[p].trellis.reshape(-1) for b in banks]) for p in range(3)]
        suh = [torch.cat([(b.gate, b.up, b.down)[p].suh.reshape(-1) for b in banks]) for p in range(3)]
        svh = [torch.cat([(b.gate, b.up, b.down)[p].svh.reshape(-1) for b in banks]) for p in range(3)]
        return cls(flat, suh, svh, np.array(meta, np.uint32), hidden, inter)

    def c(self):
        r = _lib.SxRagged()
        for p in range(3):
            r.trellis[p] = self.trellis[p].data_ptr()
            r.suh[p] = self.suh[p].data_ptr()
            r.svh[p] = self.svh[p].data_ptr()
        r.meta = self.meta.ctypes.data
        r.experts, r.hidden, r.inter = self.experts, self.hidden, self.inter
        return r


def moe_ragged(x, ragged: Ragged, inds, scores, dec: Decode, shared=None, shared_gate=None, clamp_limit=0,
               workspace=None):
    """root.moeRagged: routed SwiGLU experts over a rate-grouped layer; returns x's shape and dtype."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]).contiguous()
    rows = x2.shape[0]
    ix = inds.reshape(rows, -1).to(torch.int32).contiguous()
    sc = scores.reshape(rows, -1).float().contiguous()
    topk = ix.shape[1]
    if sc.shape != ix.shape:
        raise Exl3Error(1)
    if x2.dtype not in _DT:
        raise Exl3Error(2)
    r = ragged.c()
    need = lib().sx_moe_ragged_workspace_bytes(ctypes.byref(r), rows, topk)
    if need == 0:
        raise Exl3Error(19)
    ws = workspace if workspace is not None else _workspace(need, x.device)
    y = torch.empty_like(x2)
    d = dec.c()
    sh = None if shared is None else shared.reshape(rows, -1).to(x2.dtype).contiguous()
    sg = None if shared_gate is None else shared_gate.reshape(rows).to(x2.dtype).contiguous()
    _check(lib().sx_moe_ragged(_stream(), ctypes.byref(r), ctypes.byref(d), x2.data_ptr(), _DT[x2.dtype], rows,
                               ix.data_ptr(), sc.data_ptr(), topk, None if sh is None else sh.data_ptr(),
                               None if sg is None else sg.data_ptr(), int(clamp_limit), y.data_ptr(), ws.data_ptr(),
                               ws.numel()))
    return y.reshape(shape)


def moe_folded(x, bank, shared_bank: Bank, inds, scores, dec: Decode, shared_gate=None, clamp_limit=0,
               shared_dec: Decode = None, workspace=None):
    """moe_shared_fold.folded: the routed layer (a Bank, or a Ragged layer) plus its shared expert
    `shared_bank` (one SwiGLU expert), optionally sigmoid-gated by shared_gate [rows], in one call;
    the shared expert rides the routed launches where its rates and decode match.  Returns x's
    shape and dtype; the arithmetic of moe(..., shared=<the shared expert's own output>,
    shared_gate=...), up to the k split of the shared expert's products."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]).contiguous()
    rows = x2.shape[0]
    ix = inds.reshape(rows, -1).to(torch.int32).contiguous()
    sc = scores.reshape(rows, -1).float().contiguous()
    topk = ix.shape[1]
    if sc.shape != ix.shape:
        raise Exl3Error(1)
    if x2.dtype not in _DT:
        raise Exl3Error(2)
    ragged = isinstance(bank, Ragged)
    b, shb, d = bank.c(), shared_bank.c(), dec.c()
    sd = shared_dec.c() if shared_dec is not None else None
    sdp = ctypes.byref(sd) if sd is not None else None
    L = lib()
    wsfn = L.sx_moe_ragged_folded_workspace_bytes if ragged else L.sx_moe_folded_workspace_bytes
    need = wsfn(ctypes.byref(b), ctypes.byref(shb), ctypes.byref(d), sdp, rows, topk)
    if need == 0:
        raise Exl3Error(19 if ragged else 1)
    ws = workspace if workspace is not None else _workspace(need, x.device)
    y = torch.empty_like(x2)
    sg = None if shared_gate is None else shared_gate.reshape(rows).to(x2.dtype).contiguous()
    fn = L.sx_moe_ragged_folded if ragged else L.sx_moe_folded
    _check(fn(_stream(), ctypes.byref(b), ctypes.byref(shb), ctypes.byref(d), sdp, x2.data_ptr(), _DT[x2.dtype], rows,
              ix.data_ptr(), sc.data_ptr(), topk, None if sg is None else sg.data_ptr(), int(clamp_limit), y.data_ptr(),
              ws.data_ptr(), ws.numel()))
    return y.reshape(shape)


def moe_with_shared(x, bank, inds, scores, dec, shared):
    return moe(x, bank, inds, scores, dec, shared=shared)


def moe_with_gated_shared(x, bank, inds, scores, dec, down, gate):
    return moe(x, bank, inds, scores, dec, shared=down, shared_gate=gate)


def moe_clamped(x, bank, inds, scores, dec, limit):
    if limit <= 0 or limit > 128:
        raise Exl3Error(3)
    return moe(x, bank, inds, scores, dec, clamp_limit=limit)


def share_unique_id(group=None) -> bytes:
    """The NCCL unique id for sx_ep_init, made on the group's rank 0 (sx_ep_unique_id) and handed
    to every rank by the group's broadcast (any torch.distributed backend, gloo included)."""
    import torch.distributed as dist

    box = [ExpertParallel.unique_id() if dist.get_rank(group) == 0 else None]
    dist.broadcast_object_list(box, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
    if not isinstance(box[0], bytes) or len(box[0]) != 128:
        raise Exl3Error(17)
    return box[0]


class ExpertParallel:
    """An expert-parallel communicator (sx_ep_*): rank `rank` of `world` holds experts
    [rank*E/world, (rank+1)*E/world) of each E-expert layer as a local Bank of E/world experts.

    transport "peer" (the default): dispatch and combine store the routed rows and partials straight
    into the owning ranks' peer buffers over NVLink (sx_ep_reserve_peer; the buffer is reserved, a
    collective step, the first time a call needs more than is reserved, so every rank must make the
    same calls); "nccl": fixed-size NCCL all-to-alls."""

    def __init__(self, unique_id: bytes, world: int, rank: int, transport: str = "peer"):
        if len(unique_id) != 128:
            raise Exl3Error(1)
        if transport not in ("peer", "nccl"):
            raise ValueError(f"transport {transport!r}")
        self.world, self.rank = int(world), int(rank)
        self.transport = transport
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(unique_id)
        h = ctypes.c_void_p()
        _check(lib().sx_ep_init(buf, self.world, self.rank, ctypes.byref(h)))
        self._h = h
        self._ws = None

    def reserve(self, rows_cap: int, hidden: int, topk: int, dtype=torch.bfloat16):
        """Collective: the peer buffers for calls up to these sizes (no-op when already reserved or
        with the NCCL transport)."""
        if self.transport != "peer":
            return
        need = int(lib().sx_ep_peer_bytes(self._h, int(rows_cap), int(hidden), int(topk), _DT[dtype]))
        if need == 0:
            raise Exl3Error(1)
        if need > int(lib().sx_ep_peer_reserved(self._h)):
            _check(lib().sx_ep_reserve_peer(self._h, need))

    def peer_reserved(self) -> int:
        return int(lib().sx_ep_peer_reserved(self._h))

    PHASES = ("plan_dispatch", "wait_rows", "local_experts", "reduce_push", "shared_join", "combine")

    def phase_timing(self, enable: bool = True):
        """sx_ep_phase_timing: CUDA events at each call's phase boundaries (recorded at each graph
        replay when the call is captured)."""
        _check(lib().sx_ep_phase_timing(self._h, 1 if enable else 0))

    def phase_ms(self) -> dict:
        """The last call's phase durations in ms (sx_ep_phase_ms; waits for the call's end)."""
        out = (ctypes.c_float * 6)()
        _check(lib().sx_ep_phase_ms(self._h, out))
        return {name: float(v) for name, v in zip(self.PHASES, out)}

    @staticmethod
    def unique_id() -> bytes:
        buf = (ctypes.c_uint8 * 128)()
        _check(lib().sx_ep_unique_id(buf))
        return bytes(buf)

    @classmethod
    def from_process_group(cls, group=None, transport: str = "peer"):
        """Every rank of a torch.distributed group joins one communicator (share_unique_id)."""
        import torch.distributed as dist

        return cls(share_unique_id(group), dist.get_world_size(group), dist.get_rank(group), transport)

    def workspace_bytes(self, local_bank, rows_cap: int, topk: int, dtype=torch.bfloat16, shared_bank=None) -> int:
        """Workspace bytes for a local Bank (sx_ep_workspace_bytes) or Ragged layer
        (sx_ep_ragged_workspace_bytes); with a shared expert, the *_folded_* variants.  With the
        peer transport this reserves the peer buffers for these sizes first (collective)."""
        b = local_bank.c()
        ragged = isinstance(local_bank, Ragged)
        self.reserve(rows_cap, local_bank.hidden if ragged else local_bank.gate.dims()[1], topk, dtype)
        if shared_bank is not None:
            sb = shared_bank.c()
            fn = lib().sx_ep_ragged_folded_workspace_bytes if ragged else lib().sx_ep_folded_workspace_bytes
            return int(fn(self._h, ctypes.byref(b), ctypes.byref(sb), int(rows_cap), int(topk), _DT[dtype]))
        fn = lib().sx_ep_ragged_workspace_bytes if ragged else lib().sx_ep_workspace_bytes
        return int(fn(self._h, ctypes.byref(b), int(rows_cap), int(topk), _DT[dtype]))

    def moe(self, x, local_bank, experts_total: int, inds, scores, dec: Decode, rows_cap: int,
            shared=None, shared_gate=None, clamp_limit=0, workspace=None, shared_bank=None, shared_dec=None):
        """sx_ep_moe (local_bank a Bank) or sx_ep_moe_ragged (a Ragged layer of this rank's
        experts): this rank's rows x [rows, D] with GLOBAL expert ids inds [rows, K]; every rank
        calls it with the same rows_cap, K, experts_total and dtype.  Returns y [rows, D].  With
        `shared_bank` (the layer's shared expert, replicated on every rank) the *_folded entries run
        it over this rank's rows alongside the exchange and add it in the combine."""
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        rows = x2.shape[0]
        if x2.dtype not in _DT:
            raise Exl3Error(2)
        ix = inds.reshape(rows, -1).to(torch.int32).contiguous()
        sc = scores.reshape(rows, -1).float().contiguous()
        topk = ix.shape[1]
        if sc.shape != ix.shape:
            raise Exl3Error(1)
        ragged = isinstance(local_bank, Ragged)
        b = local_bank.c()
        need = self.workspace_bytes(local_bank, rows_cap, topk, x2.dtype, shared_bank)
        if need == 0 and ragged:
            raise Exl3Error(19)
        if workspace is None:
            if self._ws is None or self._ws.numel() < need:
                self._ws = torch.empty(max(need, 1), dtype=torch.uint8, device=x2.device)
            ws = self._ws
        else:
            ws = workspace
        y = torch.empty_like(x2)
        d = dec.c()
        sh = None if shared is None else shared.reshape(rows, -1).to(x2.dtype).contiguous()
        sg = None if shared_gate is None else shared_gate.reshape(rows).to(x2.dtype).contiguous()
        if shared_bank is not None:
            sb = shared_bank.c()
            sd = shared_dec.c() if shared_dec is not None else None
            fn = lib().sx_ep_moe_ragged_folded if ragged else lib().sx_ep_moe_folded
            _check(fn(self._h, _stream(), ctypes.byref(b), ctypes.byref(sb), int(experts_total), ctypes.byref(d),
                      ctypes.byref(sd) if sd is not None else None, x2.data_ptr(), _DT[x2.dtype], rows,
                      int(rows_cap), ix.data_ptr(), sc.data_ptr(), topk, None if sg is None else sg.data_ptr(),
                      int(clamp_limit), y.data_ptr(), ws.data_ptr(), ws.numel()))
            return y.reshape(x.shape)
        fn = lib().sx_ep_moe_ragged if ragged else lib().sx_ep_moe
        _check(fn(self._h, _stream(), ctypes.byref(b), int(experts_total), ctypes.byref(d), x2.data_ptr(),
                  _DT[x2.dtype], rows, int(rows_cap), ix.data_ptr(), sc.data_ptr(), topk,
                  None if sh is None else sh.data_ptr(), None if sg is None else sg.data_ptr(),
                  int(clamp_limit), y.data_ptr(), ws.data_ptr(), ws.numel()))
        return y.reshape(x.shape)

    def destroy(self):
        if self._h:
            _check(lib().sx_ep_destroy(self._h))
            self._h = None


def device_error():
    """The latched code of a bounded device wait that gave up (0 = none); clears it."""
    return lib().sx_device_error(_stream())


def table_row(table, n):
    out = (ctypes.c_uint32 * 4)()
    if lib().sx_table_row(table, n, out) != 0:
        return None
    return tuple(int(v) for v in out)


def table_info(table):
    name, digest = ctypes.c_char_p(), ctypes.c_char_p()
    cb, win, fields, n_lo, rows = (ctypes.c_int32() for _ in range(5))
    _check(lib().sx_table_info(table, ctypes.byref(name), ctypes.byref(cb), ctypes.byref(win), ctypes.byref(digest),
                               ctypes.byref(fields), ctypes.byref(n_lo), ctypes.byref(rows)))
    return {"name": name.value.decode(), "codebook": Codebook(cb.value), "window_bits": win.value,
            "digest": digest.value.decode(), "fields": fields.value, "n_lo": n_lo.value, "rows": rows.value}
