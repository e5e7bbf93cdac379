"""ctypes wrapper over the CPU oracle (oracle/_build/liboracle.so).  TEST INFRASTRUCTURE ONLY.

The oracle restates the reference's host decoder and CPU encoder (see exl3_oracle.cpp and
exl3_encoder.cpp for the file:line each function follows).  Only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline leg use it, and only as the checker; the product library never calls
it.  The numpy helpers at the bottom restate the reference's f32-truth MoE slot
(src/exl3/f32_truth.zig:56-98) and its routing chain (src/moe_router.zig:16-65, with the fused
kernel's lowest-id tie break, src/moe_router.zig:130-150).
"""

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

CB_MUL1, CB_MCG, CB_SPEC1, CB_PAIR1, CB_STD1 = 0, 1, 2, 3, 4
# Table indices follow the reference's `tables` order (src/exl3/codebook_tables.zig:101-106).
TABLE_NONE, TABLE_PAIR1_W16_V1, TABLE_SPEC1_W15, TABLE_SPEC1_W16, TABLE_STD1, TABLE_SPEC1_TEST = -1, 0, 1, 2, 3, 4

_lib = None


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = ctypes.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


_u16p = ctypes.POINTER(ctypes.c_uint16)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i64p = ctypes.POINTER(ctypes.c_int64)
_sz = ctypes.c_size_t


def _declare(L):
    sig = {
        "orc_f32_to_f16": (ctypes.c_uint16, [ctypes.c_float]),
        "orc_f16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
        "orc_f32_to_f16_n": (None, [_f32p, _u16p, _sz]),
        "orc_f16_to_f32_n": (None, [_u16p, _f32p, _sz]),
        "orc_f32_to_bf16_n": (None, [_f32p, _u16p, _sz]),
        "orc_bit_end": (_sz, [ctypes.c_uint32, _sz]),
        "orc_fresh_bits": (_sz, [ctypes.c_uint32, _sz]),
        "orc_decode_mcg": (ctypes.c_uint16, [ctypes.c_uint16]),
        "orc_decode_mul1": (ctypes.c_uint16, [ctypes.c_uint16]),
        "orc_decode_hash_mask": (ctypes.c_uint16, [ctypes.c_uint16, ctypes.c_uint32, ctypes.c_uint32]),
        "orc_pair1_row": (ctypes.c_int, [ctypes.c_uint32, _u32p]),
        "orc_hash_row": (ctypes.c_int, [ctypes.c_int, ctypes.c_uint32, _u32p]),
        "orc_decode_pair": (ctypes.c_int, [ctypes.c_uint16, ctypes.c_uint32, _u16p]),
        "orc_unpack_tile": (None, [_u16p, ctypes.c_uint32, _u16p]),
        "orc_decode_all": (ctypes.c_int, [ctypes.c_int, ctypes.c_uint32, ctypes.c_int, ctypes.c_int, _u32p]),
        "orc_tensor_core_perm": (None, [_i64p]),
        "orc_decode_tile": (ctypes.c_int, [_u16p, ctypes.c_uint32, ctypes.c_int, ctypes.c_int, ctypes.c_int, _u16p]),
        "orc_hadamard128": (None, [_f32p]),
        "orc_reconstruct_inner": (ctypes.c_int, [_u16p, _sz, _sz, ctypes.c_uint32, ctypes.c_int, ctypes.c_int, ctypes.c_int, _u16p]),
        "orc_reconstruct_public": (ctypes.c_int, [_u16p, _u16p, _u16p, _sz, _sz, ctypes.c_uint32, ctypes.c_int, ctypes.c_int, ctypes.c_int, _u16p]),
        "orc_decode_dense": (ctypes.c_int, [_u16p, _u16p, _u16p, _sz, _sz, ctypes.c_uint32, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p]),
        "orc_prepare_input": (None, [_f32p, _u16p, _sz, _f32p]),
        "orc_inner_gemv": (ctypes.c_int, [_u16p, _f32p, _sz, _sz, ctypes.c_uint32, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p]),
        "orc_finish_output": (None, [_f32p, _u16p, _sz, _f32p]),
        "orc_project": (ctypes.c_int, [_f32p, _u16p, _u16p, _u16p, _sz, _sz, ctypes.c_uint32, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p]),
        "orc_project_rows": (ctypes.c_int, [_f32p, _sz, _u16p, _u16p, _u16p, _sz, _sz, ctypes.c_uint32, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p]),
        "orc_project_mt": (ctypes.c_int, [_f32p, _u16p, _u16p, _u16p, _sz, _sz, ctypes.c_uint32, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p]),
        "orc_num_threads": (ctypes.c_int, []),
        "orc_set_num_threads": (None, [ctypes.c_int]),
        "orc_tile_major": (None, [_u16p, _u16p, _sz, _sz, _sz]),
        "orc_encode_tile": (ctypes.c_double, [_f32p, ctypes.c_uint32, ctypes.c_int, ctypes.c_int, _u16p, _f32p]),
        "orc_encode_tiles": (ctypes.c_int, [_f32p, _sz, ctypes.c_uint32, ctypes.c_int, ctypes.c_int, _u16p, _f64p]),
        "orc_signs": (None, [ctypes.c_uint64, ctypes.c_char_p, _sz, _f32p]),
        "orc_regularize": (ctypes.c_int, [_f32p, _sz, _sz, _f32p, _f32p, ctypes.c_int, _f32p, _f32p, _f32p, _f32p]),
        "orc_ldl_factor": (ctypes.c_int, [_f32p, _sz, _f32p]),
        "orc_quantize_tensor": (ctypes.c_int, [_f32p, _f32p, _sz, _sz, _f32p, _f32p, ctypes.c_uint32, ctypes.c_int, ctypes.c_int, ctypes.c_int, _u16p, _u16p, _u16p, _f32p]),
        "orc_quantize_named": (ctypes.c_int, [_f32p, _f32p, _sz, _sz, ctypes.c_uint64, ctypes.c_char_p, ctypes.c_uint32, ctypes.c_int, ctypes.c_int, ctypes.c_int, _u16p, _u16p, _u16p, _f32p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _p(a, t):
    return a.ctypes.data_as(t)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ------------------------------------------------------------------ scalar decode
def f16_bits(x):
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_f16_n(_p(x, _f32p), _p(out, _u16p), x.size)
    return out


def f16_value(bits):
    bits = _c(bits, np.uint16)
    out = np.empty(bits.shape, np.float32)
    lib().orc_f16_to_f32_n(_p(bits, _u16p), _p(out, _f32p), bits.size)
    return out


def bf16_bits(x):
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_bf16_n(_p(x, _f32p), _p(out, _u16p), x.size)
    return out


def bf16_value(bits):
    return (_c(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def decode_mcg(cw):
    return lib().orc_decode_mcg(cw)


def decode_mul1(cw):
    return lib().orc_decode_mul1(cw)


def decode_hash_mask(cw, mult, mask):
    return lib().orc_decode_hash_mask(cw, mult, mask)


def pair1_row(n):
    out = np.zeros(4, np.uint32)
    return None if lib().orc_pair1_row(n, _p(out, _u32p)) else tuple(int(v) for v in out)


def hash_row(table, n):
    out = np.zeros(2, np.uint32)
    return None if lib().orc_hash_row(table, n, _p(out, _u32p)) else tuple(int(v) for v in out)


def decode_pair(cw, n):
    out = np.zeros(2, np.uint16)
    if lib().orc_decode_pair(cw, n, _p(out, _u16p)):
        raise ValueError(f"no PAIR1 row at n={n}")
    return int(out[0]), int(out[1])


def bit_end(n, t):
    return lib().orc_bit_end(n, t)


def fresh_bits(n, t):
    return lib().orc_fresh_bits(n, t)


def unpack_tile(words, n):
    words = _c(words, np.uint16)
    out = np.empty(256, np.uint16)
    lib().orc_unpack_tile(_p(words, _u16p), n, _p(out, _u16p))
    return out


def decode_all(codebook, n, window_bits=16, table=TABLE_NONE):
    """Every codeword's decode (u32 per codeword; PAIR1 packs the pair)."""
    out = np.empty(1 << 16, np.uint32)
    if lib().orc_decode_all(codebook, n, window_bits, table, _p(out, _u32p)):
        raise ValueError("decode without a codebook row at this rate")
    return out


def tensor_core_perm():
    out = np.empty(256, np.int64)
    lib().orc_tensor_core_perm(_p(out, _i64p))
    return out


def decode_tile(words, n, codebook, window_bits=16, table=TABLE_NONE):
    words = _c(words, np.uint16)
    out = np.empty(256, np.uint16)
    if lib().orc_decode_tile(_p(words, _u16p), n, codebook, window_bits, table, _p(out, _u16p)):
        raise ValueError("decode without a codebook row at this rate")
    return out


def hadamard128(v):
    v = _c(v, np.float32).copy()
    lib().orc_hadamard128(_p(v, _f32p))
    return v


# ------------------------------------------------------------------ whole projections
def reconstruct_inner(trellis, in_f, out_f, n, codebook, window_bits=16, table=TABLE_NONE):
    trellis = _c(trellis, np.uint16)
    out = np.empty((in_f, out_f), np.uint16)
    if lib().orc_reconstruct_inner(_p(trellis, _u16p), in_f, out_f, n, codebook, window_bits, table, _p(out, _u16p)):
        raise ValueError("decode without a codebook row at this rate")
    return out


def reconstruct_public(trellis, suh, svh, in_f, out_f, n, codebook, window_bits=16, table=TABLE_NONE):
    trellis, suh, svh = _c(trellis, np.uint16), _c(suh, np.uint16), _c(svh, np.uint16)
    out = np.empty((in_f, out_f), np.uint16)
    rc = lib().orc_reconstruct_public(_p(trellis, _u16p), _p(suh, _u16p), _p(svh, _u16p), in_f, out_f, n, codebook,
                                      window_bits, table, _p(out, _u16p))
    if rc:
        raise ValueError("decode without a codebook row at this rate")
    return out


def decode_dense(trellis, suh, svh, in_f, out_f, n, codebook, window_bits=16, table=TABLE_NONE):
    """The dense f32 twin W [in, out] of one bank (src/exl3/linear.zig:406-431)."""
    trellis, suh, svh = _c(trellis, np.uint16), _c(suh, np.uint16), _c(svh, np.uint16)
    out = np.empty((in_f, out_f), np.float32)
    rc = lib().orc_decode_dense(_p(trellis, _u16p), _p(suh, _u16p), _p(svh, _u16p), in_f, out_f, n, codebook,
                                window_bits, table, _p(out, _f32p))
    if rc:
        raise ValueError("decode without a codebook row at this rate")
    return out


def project(x, trellis, suh, svh, in_f, out_f, n, codebook, window_bits=16, table=TABLE_NONE, threads=None):
    """The reference's CPU projection `format.project` (src/exl3/expert_exl3.zig:546) per row."""
    x = _c(np.atleast_2d(x), np.float32)
    trellis, suh, svh = _c(trellis, np.uint16), _c(suh, np.uint16), _c(svh, np.uint16)
    y = np.empty((x.shape[0], out_f), np.float32)
    L = lib()
    if threads is not None:
        L.orc_set_num_threads(threads)
    if x.shape[0] == 1:
        rc = L.orc_project_mt(_p(x, _f32p), _p(trellis, _u16p), _p(suh, _u16p), _p(svh, _u16p), in_f, out_f, n,
                              codebook, window_bits, table, _p(y, _f32p))
    else:
        rc = L.orc_project_rows(_p(x, _f32p), x.shape[0], _p(trellis, _u16p), _p(suh, _u16p), _p(svh, _u16p), in_f,
                                out_f, n, codebook, window_bits, table, _p(y, _f32p))
    if rc:
        raise ValueError("decode without a codebook row at this rate")
    return y


def project_single_thread(x, trellis, suh, svh, in_f, out_f, n, codebook, window_bits=16, table=TABLE_NONE):
    x = _c(x, np.float32).reshape(-1)
    trellis, suh, svh = _c(trellis, np.uint16), _c(suh, np.uint16), _c(svh, np.uint16)
    y = np.empty(out_f, np.float32)
    rc = lib().orc_project(_p(x, _f32p), _p(trellis, _u16p), _p(suh, _u16p), _p(svh, _u16p), in_f, out_f, n, codebook,
                           window_bits, table, _p(y, _f32p))
    if rc:
        raise ValueError("decode without a codebook row at this rate")
    return y


def num_threads():
    return lib().orc_num_threads()


def set_num_threads(n):
    lib().orc_set_num_threads(n)


def tile_major(trellis, it, ot, n):
    src = _c(trellis, np.uint16)
    dst = np.empty_like(src)
    lib().orc_tile_major(_p(src, _u16p), _p(dst, _u16p), it, ot, n)
    return dst


# ------------------------------------------------------------------ encoder
def encode_tile(tile, n, codebook, window_bits):
    tile = _c(tile, np.float32).reshape(256)
    packed = np.empty(n, np.uint16)
    recon = np.empty(256, np.float32)
    cost = lib().orc_encode_tile(_p(tile, _f32p), n, codebook, window_bits, _p(packed, _u16p), _p(recon, _f32p))
    if cost < 0:
        raise ValueError(f"encoder refused: {cost}")
    return packed, cost, recon


def encode_tiles(tiles, n, codebook, window_bits):
    tiles = _c(tiles, np.float32).reshape(-1, 256)
    packed = np.empty((tiles.shape[0], n), np.uint16)
    costs = np.empty(tiles.shape[0], np.float64)
    rc = lib().orc_encode_tiles(_p(tiles, _f32p), tiles.shape[0], n, codebook, window_bits, _p(packed, _u16p),
                                _p(costs, _f64p))
    if rc:
        raise ValueError(f"encoder refused: {rc}")
    return packed, costs


def signs(seed, name, length):
    out = np.empty(length, np.float32)
    lib().orc_signs(seed, name.encode(), length, _p(out, _f32p))
    return out


MODES = {"auto": 0, "always": 1, "never": 2}


def regularize(w, in_f, out_f, sign_in, sign_out, mode, hdiag):
    w, si, so = _c(w, np.float32), _c(sign_in, np.float32), _c(sign_out, np.float32)
    hd = None if hdiag is None else _c(hdiag, np.float32)
    inner = np.empty((in_f, out_f), np.float32)
    suh = np.empty(in_f, np.float32)
    svh = np.empty(out_f, np.float32)
    rc = lib().orc_regularize(_p(w, _f32p), in_f, out_f, _p(si, _f32p), _p(so, _f32p), MODES[mode],
                              None if hd is None else _p(hd, _f32p), _p(inner, _f32p), _p(suh, _f32p), _p(svh, _f32p))
    if rc:
        raise ValueError(f"regularize refused: {rc}")
    return inner, suh, svh


def ldl_factor(h, n):
    h = _c(h, np.float32)
    out = np.empty((n, n), np.float32)
    rc = lib().orc_ldl_factor(_p(h, _f32p), n, _p(out, _f32p))
    if rc:
        raise ValueError(f"ldl refused: {rc}")
    return out


def quantize_tensor(w, h, in_f, out_f, sign_in, sign_out, n, codebook, window_bits, mode):
    w, h, si, so = _c(w, np.float32), _c(h, np.float32), _c(sign_in, np.float32), _c(sign_out, np.float32)
    packed = np.empty((in_f // 16, out_f // 16, n), np.uint16)
    suh = np.empty(in_f, np.uint16)
    svh = np.empty(out_f, np.uint16)
    g = np.zeros(1, np.float32)
    rc = lib().orc_quantize_tensor(_p(w, _f32p), _p(h, _f32p), in_f, out_f, _p(si, _f32p), _p(so, _f32p), n, codebook,
                                   window_bits, MODES[mode], _p(packed, _u16p), _p(suh, _u16p), _p(svh, _u16p),
                                   _p(g, _f32p))
    if rc:
        raise ValueError(f"quantize refused: {rc}")
    return packed, suh, svh, float(g[0])


def quantize_named(w, h, in_f, out_f, seed, name, n, codebook, window_bits, mode="auto"):
    """`quantize.quantizeNamed` (src/encoder/quantize.zig:593): the pack one named weight encodes to."""
    w, h = _c(w, np.float32), _c(h, np.float32)
    packed = np.empty((in_f // 16, out_f // 16, n), np.uint16)
    suh = np.empty(in_f, np.uint16)
    svh = np.empty(out_f, np.uint16)
    g = np.zeros(1, np.float32)
    rc = lib().orc_quantize_named(_p(w, _f32p), _p(h, _f32p), in_f, out_f, seed, name.encode(), n, codebook,
                                  window_bits, MODES[mode], _p(packed, _u16p), _p(suh, _u16p), _p(svh, _u16p),
                                  _p(g, _f32p))
    if rc:
        raise ValueError(f"quantize refused: {rc}")
    return packed, suh, svh, float(g[0])


# ------------------------------------------------------------------ f32 truth (numpy, f64)
def matvec_f64(w, x):
    """y = x . W in f64 over a dense f32 [in, out] (src/exl3/f32_truth.zig:56-63)."""
    return np.asarray(x, np.float64) @ np.asarray(w, np.float64)


def expert_truth(dense, x, limit=0.0):
    """The (clamped) SwiGLU expert in f64 over its dense gate/up/down twins
    (src/exl3/f32_truth.zig:85-98): act is rounded to f32 before the down product."""
    g = matvec_f64(dense[0], x)
    u = matvec_f64(dense[1], x)
    if limit > 0:
        g = np.minimum(g, limit)
        u = np.clip(u, -limit, limit)
    act = (g / (1.0 + np.exp(-g)) * u).astype(np.float32)
    return matvec_f64(dense[2], act)


def rms_norm_truth(y, w, eps):
    """MLX's rms_norm of each row, as the normed stacked finish applies it to a linear's finished
    output (src/exl3/project_rows.zig:394-456): y * rsqrt(mean(y^2) + eps) * w, in f64."""
    y = np.asarray(y, np.float64)
    inv = 1.0 / np.sqrt(np.mean(y * y, axis=-1, keepdims=True) + eps)
    return y * inv * np.asarray(w, np.float64)


def router_gate_logit(x, w):
    """The softmax_gate router's shared-expert gate logit (src/moe_router.zig:200-218, :328-332),
    in f32 with the order MLX's dot_product uses as that kernel restates it: virtual group vs of
    1024 elements; lane l keeps a float4 c over its 8-element chunks at 1024 vs + 8 l + 256 i
    (i = 0..3; chunks past the end skipped), c[q] += x * w element by element; then
    c0 + c1 + c2 + c3, a butterfly sum over the 32 lanes (xor 16, 8, 4, 2, 1), and a butterfly
    over the groups' partials in 16 lanes (xor 8, 4, 2, 1; zeros past the last group).  Products
    and sums rounded separately.  x and w are the (already rounded) f16/bf16 values as float32;
    returns the f32 sum (the caller rounds it to the gate dtype)."""
    x = np.asarray(x, np.float32)
    w = np.asarray(w, np.float32)
    gk = x.shape[0]
    f = np.float32

    def butterfly(vals, widths):
        v = list(vals)
        for m in widths:
            v = [f(v[i] + v[i ^ m]) for i in range(len(v))]
        return v[0]

    parts = []
    for vs in range((gk + 1023) // 1024):
        lanes = []
        for lane in range(32):
            c = [f(0.0)] * 4
            for i in range(0, 32, 8):
                idx = vs * 1024 + lane * 8 + i * 32
                if idx + 8 <= gk:
                    for j in range(8):
                        c[j & 3] = f(c[j & 3] + f(x[idx + j] * w[idx + j]))
            lanes.append(f(f(f(c[0] + c[1]) + c[2]) + c[3]))
        parts.append(butterfly(lanes, (16, 8, 4, 2, 1)))
    parts = parts + [f(0.0)] * (16 - len(parts))
    return butterfly(parts, (8, 4, 2, 1))


def router_truth(logits, k, mode="softmax", bias=None, renorm=True, scale=1.0, n_group=0, topk_group=0):
    """Top-k routing (src/moe_router.zig:16-65 chain semantics with the fused kernel's lowest-id
    tie break, :130-150; sigmoid_bias and its group limit :200-290).  Returns (inds, weights)."""
    logits = np.asarray(logits, np.float64)
    T, E = logits.shape
    inds = np.zeros((T, k), np.int64)
    wts = np.zeros((T, k), np.float64)
    for t in range(T):
        l = logits[t]
        if mode == "softmax":
            key = l.copy()
            p = np.exp(l - l.max())
            p = p / p.sum()
        else:
            sig = 1.0 / (1.0 + np.exp(-l))
            key = sig + np.asarray(bias, np.float64)
            p = sig
            if mode == "sigmoid_bias_grouped":
                gsz = E // n_group
                gs = np.array([np.sort(key[g * gsz:(g + 1) * gsz])[-2:].sum() for g in range(n_group)])
                keep = np.argsort(-gs, kind="stable")[:topk_group]
                mask = np.zeros(E, bool)
                for g in keep:
                    mask[g * gsz:(g + 1) * gsz] = True
                key = np.where(mask, key, -1.0e4)
        order = np.argsort(-key, kind="stable")[:k]
        inds[t] = order
        w = p[order]
        if mode == "softmax":
            w = w / w.sum()
        else:
            if renorm and k > 1:
                w = w / (w.sum() + 1e-20)
            w = w * scale
        wts[t] = w
    return inds, wts
