"""Seeded synthetic inputs for the parity tests and the bench.  TEST INFRASTRUCTURE ONLY.

The reference measures on real packs; BASELINE.json's configs name seeded synthetic weights of
the benchmark shapes instead.  Weights are splitmix64-seeded Box-Muller normals (rounded to bf16
as a checkpoint would hold them), encoded by the oracle's restatement of the reference quantizer
(`quantizeNamed`, src/encoder/quantize.zig:593) with an identity Hessian.  Expert banks for the
MoE configs use random trellis words with sign-only scales, the reference's own synthetic-bank
recipe (`synth.makeBank`, src/exl3/synth.zig:16-41).
"""

import os

import numpy as np

from oracle import oracle as orc

MASK64 = (1 << 64) - 1


def splitmix_stream(seed, count):
    """`count` splitmix64 outputs from `seed`, vectorised (state_i = seed + (i+1) * golden)."""
    i = np.arange(1, count + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + i * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return z


def normal(seed, count, std=1.0):
    """Box-Muller normals from a splitmix64 stream: two uniforms per pair of outputs."""
    pairs = (count + 1) // 2
    z = splitmix_stream(seed, 2 * pairs)
    u = ((z >> np.uint64(11)).astype(np.float64) + 0.5) * (1.0 / (1 << 53))
    u1, u2 = u[0::2], u[1::2]
    r = np.sqrt(-2.0 * np.log(u1))
    out = np.empty(2 * pairs, np.float64)
    out[0::2] = r * np.cos(2 * np.pi * u2)
    out[1::2] = r * np.sin(2 * np.pi * u2)
    return (out[:count] * std).astype(np.float32)


def bf16_round(x):
    return orc.bf16_value(orc.bf16_bits(x))


def dense_weight(seed, in_f, out_f, std=0.02, outlier_frac=0.0, outlier_scale=8.0):
    """W [in, out] ~ N(0, std) rounded to bf16; optionally ceil(frac * in) seeded input channels x scale."""
    w = normal(seed, in_f * out_f, std).reshape(in_f, out_f)
    if outlier_frac > 0:
        k = int(np.ceil(outlier_frac * in_f))
        rng = np.random.default_rng(seed ^ 0x5EED)
        rows = rng.choice(in_f, size=k, replace=False)
        w[rows] *= outlier_scale
    return bf16_round(w)


def activations(seed, rows, in_f, std=1.0):
    """x [rows, in] ~ N(0, std) as bf16 values (f32 holding bf16)."""
    return bf16_round(normal(seed, rows * in_f, std).reshape(rows, in_f))


def outlier_activations(seed, rows, in_f, std=1.0):
    """x [rows, in] as bf16 values: N(0, std) with every channel i where i % 997 == 3 scaled x30,
    the normed-residual stand-in of the reference's f32 truth (`activations`,
    src/exl3/f32_truth.zig:42-54)."""
    x = normal(seed, rows * in_f, std).reshape(rows, in_f)
    x[:, np.arange(in_f) % 997 == 3] *= 30.0
    return bf16_round(x)


def encode_weight(w, seed, name, n, codebook, window_bits):
    """(trellis, suh, svh, g) for public weight w [in, out] with an identity Hessian."""
    in_f, out_f = w.shape
    h = np.eye(in_f, dtype=np.float32)
    return orc.quantize_named(w, h, in_f, out_f, seed, name, n, codebook, window_bits, "auto")


def random_bank(seed, experts, in_f, out_f, n, suh_mag=0.02, svh_mag=1.0):
    """Random trellis words with sign-only scales (src/exl3/synth.zig:16-41): trellis
    [E, in/16, out/16, n] u16, suh [E, in] and svh [E, out] f16 bits."""
    rng = np.random.default_rng(seed)
    trellis = rng.integers(0, 1 << 16, size=(experts, in_f // 16, out_f // 16, n), dtype=np.uint16)
    su = np.where(rng.random((experts, in_f)) < 0.5, -suh_mag, suh_mag).astype(np.float32)
    sv = np.where(rng.random((experts, out_f)) < 0.5, -svh_mag, svh_mag).astype(np.float32)
    return trellis, orc.f16_bits(su), orc.f16_bits(sv)


CONFIG1_SEED = 0xC0F1
CONFIG1_NAME = "model.layers.0.self_attn.o_proj"


def config1_pack(cache_dir=None):
    """W [4096, 4096] ~ N(0, 0.02) bf16, encoded MCG K2 (n32) window 16 by the
    quantizer restatement with an identity Hessian and name-seeded signs.  Cached as .npz in
    `cache_dir` when given (the encode takes minutes on 8 cores)."""
    path = None
    if cache_dir:
        path = os.path.join(cache_dir, "config1_mcg_n32_w16.npz")
        if os.path.exists(path):
            with np.load(path) as z:
                return {k: z[k] for k in z.files}
    w = dense_weight(CONFIG1_SEED, 4096, 4096, 0.02)
    trellis, suh, svh, g = encode_weight(w, CONFIG1_SEED, CONFIG1_NAME, 32, orc.CB_MCG, 16)
    pack = {"trellis": trellis, "suh": suh, "svh": svh, "g": np.float32(g)}
    if path:
        os.makedirs(cache_dir, exist_ok=True)
        np.savez(path, **pack)
    return pack


CONFIG2_SEED = 0xC0F2
CONFIG2_NAME = "model.layers.0.mlp.up_proj"


def config2_pack(cache_dir=None):
    """BASELINE configs[1]'s encoded weight at the sweep shape 7168x2048 (out x in): W [2048, 7168]
    ~ N(0, 0.02) bf16 with ceil(1% of 2048) seeded input channels x8 (outlier channels), encoded
    MCG K2 (n32) at window 12 by the quantizer restatement with an identity Hessian.  Cached as
    .npz in `cache_dir` when given (about 15 s of encode on 8 cores)."""
    path = None
    if cache_dir:
        path = os.path.join(cache_dir, "config2_mcg_n32_w12_outliers.npz")
        if os.path.exists(path):
            with np.load(path) as z:
                return {k: z[k] for k in z.files}
    w = dense_weight(CONFIG2_SEED, 2048, 7168, 0.02, outlier_frac=0.01, outlier_scale=8.0)
    trellis, suh, svh, g = encode_weight(w, CONFIG2_SEED, CONFIG2_NAME, 32, orc.CB_MCG, 12)
    pack = {"trellis": trellis, "suh": suh, "svh": svh, "g": np.float32(g)}
    if path:
        os.makedirs(cache_dir, exist_ok=True)
        np.savez(path, **pack)
    return pack
