"""Pins the CPU oracle to the reference's own golden vectors and known-answer tests.

Every case here restates one of the reference's host tests (file:line cited per test) and runs it
against tests/golden/*.npz, the reference's committed fixtures (tests/golden/make_golden.py).
"""

import hashlib

import numpy as np
import pytest

from oracle import oracle as orc


def test_f16_conversion_matches_ieee_rne():
    # Every f16 bit pattern round-trips, and random f32 values round as numpy's IEEE RNE does.
    bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    finite = (bits & 0x7C00) != 0x7C00
    vals = orc.f16_value(bits)
    np.testing.assert_array_equal(vals[finite], bits[finite].view(np.float16).astype(np.float32))
    np.testing.assert_array_equal(orc.f16_bits(vals[finite]), bits[finite])
    rng = np.random.default_rng(1)
    for scale in (1e-8, 1e-6, 1e-4, 1.0, 1e3, 6e4, 7e4):
        x = (rng.standard_normal(200000) * scale).astype(np.float32)
        x = x[np.abs(x) < 65520]
        want = x.astype(np.float16).view(np.uint16)
        np.testing.assert_array_equal(orc.f16_bits(x), want)
    # ties at the subnormal boundary and overflow boundary
    edge = np.array([2.0**-25, 3 * 2.0**-25, 65504.0, 65519.0, 65520.0, -65520.0, 2.0**-24 * 1.5], np.float32)
    np.testing.assert_array_equal(orc.f16_bits(edge), edge.astype(np.float16).view(np.uint16))


def test_bf16_conversion_rne():
    rng = np.random.default_rng(2)
    x = rng.standard_normal(100000).astype(np.float32)
    b = orc.bf16_bits(x)
    u = x.view(np.uint32)
    want = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    np.testing.assert_array_equal(b, want)


# src/exl3/expert_exl3.zig:661-697
@pytest.mark.parametrize(
    "n,ends,fresh",
    [
        (40, [2, 5, 7, 10, 12, 15, 17, 20], [2, 3] * 8),
        (44, [2, 5, 8, 11, 13, 16, 19, 22], [2, 3, 3, 3] * 4),
        (48, [3, 6, 9, 12, 15, 18, 21, 24], [3] * 16),
        (64, [4, 8, 12, 16, 20, 24, 28, 32], [4] * 16),
    ],
)
def test_bit_ends_hand_table(n, ends, fresh):
    assert [orc.bit_end(n, i) for i in range(8)] == ends
    assert [orc.fresh_bits(n, i) for i in range(16)] == fresh
    assert orc.bit_end(n, 255) == 16 * n
    assert sum(orc.fresh_bits(n, i) for i in range(256)) == 16 * n


def test_mul1_and_mcg_codeword_pins():
    # src/exl3/expert_exl3.zig:699-704, :839-862
    assert orc.decode_mul1(0) == 49896
    assert orc.decode_mul1(1) == 14625
    assert orc.decode_mul1(7) == 47511
    pair = 0x3B603B60
    want = orc.f16_bits(np.array([orc.f16_value(np.uint16(pair & 0xFFFF)) + orc.f16_value(np.uint16(pair >> 16))], np.float32))[0]
    assert orc.decode_mcg(0) == int(want)


def test_hash_mask_codeword_pins():
    # src/exl3/expert_exl3.zig:728-739 (sashimi's bits, rounded half sums included)
    mult, mask = 0x840C1F37, 0x8FFE8FD0
    pins = {0: 0x0000, 1: 0x3E0D, 7: 0xBF94, 0x15: 0xC060, 0x3E: 0xC164, 0x1234: 0xBAD0, 0xFFFF: 0xBB8A}
    for cw, want in pins.items():
        assert orc.decode_hash_mask(cw, mult, mask) == want, hex(cw)


def test_std1_is_one_pair_at_every_rate_and_spec1_needs_a_table():
    # src/exl3/expert_exl3.zig:716-747
    for n in (24, 32, 40, 48, 64):
        assert orc.hash_row(orc.TABLE_STD1, n) == (0x840C1F37, 0x8FFE8FD0)
    assert orc.hash_row(orc.TABLE_NONE, 40) is None
    assert orc.hash_row(orc.TABLE_SPEC1_W15, 40) is not None


def test_pair1_rows_exist_only_at_even_n_24_to_64():
    # src/exl3/expert_exl3.zig:749-767
    for n in range(16, 73):
        assert (orc.pair1_row(n) is not None) == (n % 2 == 0 and 24 <= n <= 64)
    assert orc.pair1_row(24) == (0x58F41BF3, 3, 0x8ED78C13, 0x8EEE8C03)
    assert orc.pair1_row(32) == (0x3B22BE15, 3, 0x8ED78C13, 0x8ECE8C03)
    assert orc.pair1_row(48) == (0xF75D60FF, 19, 0x8E6E8F9A, 0x8E258FFE)
    assert orc.pair1_row(56) == (0x82439F67, 19, 0x8E6E8F9A, 0x8E258FAE)
    assert orc.pair1_row(64) == (0xE2C7FC0D, 19, 0x8F408FA0, 0x8F118FC9)
    for n in (34, 36, 38, 40):
        assert orc.pair1_row(n)[2] == (0x8E6E8F9A if n == 38 else 0x8F9A8E6E)


# src/exl3/expert_exl3.zig:770-795 (sashimi's numpy v2rot_tables bits)
PAIR1_PINS = [
    (24, 0x1, (0x3C74, 0xBDAA)), (24, 0x1234, (0x3A7C, 0xB8CB)), (32, 0x0, (0x0000, 0x0000)),
    (32, 0x1, (0xB440, 0xB804)), (32, 0x1234, (0x3822, 0xB086)), (32, 0xFFFF, (0xB19E, 0x3DA0)),
    (38, 0x1, (0x3FA4, 0x3610)), (38, 0x1234, (0x3A99, 0xB898)), (40, 0x1, (0x3FA6, 0x3610)),
    (40, 0x1234, (0x3A6D, 0xB898)), (48, 0x1, (0xB5B2, 0xB7AF)), (48, 0x15, (0x37C6, 0xA9D0)),
    (48, 0x8000, (0xA6E0, 0xB3EE)), (56, 0x1, (0xBF92, 0xB91E)), (56, 0x1234, (0xBCF0, 0xBAD6)),
    (58, 0x1, (0xBC90, 0x3608)), (58, 0x1234, (0x3CB0, 0xB102)), (64, 0x7, (0xAA00, 0xBA80)),
    (64, 0x15, (0xC010, 0x34F7)), (64, 0xFFFF, (0x3B10, 0x3C0C)),
]


@pytest.mark.parametrize("n,cw,want", PAIR1_PINS)
def test_pair1_codeword_pins(n, cw, want):
    assert orc.decode_pair(cw, n) == want


def test_pair1_tiles_match_upstream_numpy_decode(golden):
    # src/exl3/expert_exl3.zig:797-815 against fixtures/exl3_pair1_tiles.safetensors
    g = golden("exl3_pair1_tiles")
    for n in range(24, 65, 2):
        tr = g[f"trellis_n{n}"]
        want = g[f"decoded_n{n}"]
        for t in range(tr.shape[0]):
            got = orc.decode_tile(tr[t], n, orc.CB_PAIR1)
            np.testing.assert_array_equal(got, want[t], err_msg=f"n{n} tile {t}")


LINEAR_FIXTURES = [
    ("exl3_k4_linear", 64, orc.CB_MUL1, 16),
    ("exl3_k3_linear", 48, orc.CB_MUL1, 16),
    ("exl3_k2_linear", 32, orc.CB_MUL1, 16),
    ("exl3_k2p5_mcg_linear", 40, orc.CB_MCG, 16),
    ("exl3_k3_mcg_linear", 48, orc.CB_MCG, 16),
    ("exl3_k2p5_mcg_w12_linear", 40, orc.CB_MCG, 12),
]


@pytest.mark.parametrize("stem,n,cb,w", LINEAR_FIXTURES)
def test_packed_fixture_decodes_to_library_inner_and_public(golden, stem, n, cb, w):
    # src/exl3/expert_exl3.zig:864-997
    g = golden(stem)
    tr, suh, svh = g["trellis"], g["suh"], g["svh"]
    assert tr.shape == (8, 8, n)
    inner = orc.reconstruct_inner(tr, 128, 128, n, cb, w)
    np.testing.assert_array_equal(inner, g["inner"])
    public = orc.reconstruct_public(tr, suh, svh, 128, 128, n, cb, w)
    np.testing.assert_array_equal(public, g["public"])


def test_w12_fixture_is_a_different_matrix_at_w16(golden):
    # src/exl3/expert_exl3.zig:987-996
    g = golden("exl3_k2p5_mcg_w12_linear")
    wide = orc.reconstruct_inner(g["trellis"], 128, 128, 40, orc.CB_MCG, 16)
    assert not np.array_equal(wide, g["inner"])


def test_k4_projection_matches_dense_public(golden):
    # src/exl3/expert_exl3.zig:890-914: project() within 2% relative RMS of x . public
    g = golden("exl3_k4_linear")
    rng = np.random.default_rng(7)
    x = (rng.random(128, dtype=np.float32) * 2 - 1).astype(np.float32)
    y = orc.project_single_thread(x, g["trellis"], g["suh"], g["svh"], 128, 128, 64, orc.CB_MUL1)
    dense = x.astype(np.float32) @ orc.f16_value(g["public"])
    rel = np.sqrt(((y - dense) ** 2).sum() / max((dense**2).sum(), 1e-20))
    assert rel < 0.02


def test_narrowed_window_is_masked_codeword(golden):
    # src/exl3/expert_exl3.zig:1015-1039
    g = golden("exl3_k2p5_mcg_linear")
    tile = g["trellis"].reshape(-1, 40)[0]
    cws = orc.unpack_tile(tile, 40)
    perm = orc.tensor_core_perm()
    wide = orc.decode_tile(tile, 40, orc.CB_MCG, 16)
    for wbits in (8, 10):
        got = orc.decode_tile(tile, 40, orc.CB_MCG, wbits)
        want = np.empty(256, np.uint16)
        for i, cw in enumerate(cws):
            want[perm[i]] = orc.decode_mcg(int(cw) & ((1 << wbits) - 1))
        np.testing.assert_array_equal(got, want)
        assert not np.array_equal(got, wide)


def _circular_codewords(words, n):
    # src/exl3/expert_exl3.zig:1062-1068: independent bit-at-a-time extraction.
    want = np.zeros(256, np.uint16)
    for slot in range(256):
        cw = 0
        for bit in range(16):
            at = ((slot + 1) * n // 16 + 16 * n - 16 + bit) % (16 * n)
            v = (int(words[2 * (at // 32) + (1 - (at % 32) // 16)]) >> (15 - at % 16)) & 1
            cw = (cw << 1) | v
        want[slot] = cw
    return want


def test_scalar_tiles_match_circular_bit_extraction_every_rate():
    # src/exl3/expert_exl3.zig:1051-1089 (every n 16..128, every codebook, windows 8..16)
    rng = np.random.default_rng(0x51555348)
    perm = orc.tensor_core_perm()
    for n in range(16, 129, 2):
        for rep in range(2):
            words = rng.integers(0, 1 << 16, n, dtype=np.uint16)
            want = _circular_codewords(words, n)
            np.testing.assert_array_equal(orc.unpack_tile(words, n), want, err_msg=f"n{n}")
            for cb, table in ((orc.CB_MCG, -1), (orc.CB_MUL1, -1), (orc.CB_SPEC1, orc.TABLE_SPEC1_W15),
                              (orc.CB_STD1, orc.TABLE_STD1), (orc.CB_PAIR1, -1)):
                if cb == orc.CB_PAIR1 and orc.pair1_row(n) is None:
                    continue
                if cb in (orc.CB_SPEC1, orc.CB_STD1) and orc.hash_row(table, n) is None:
                    continue
                for wbits in (8, 12, 15, 16) if rep == 0 else (9, 16):
                    mask = (1 << wbits) - 1
                    got = orc.decode_tile(words, n, cb, wbits, table)
                    for slot in range(0, 256, 7):
                        if cb == orc.CB_PAIR1:
                            v = orc.decode_pair(int(want[slot | 1]) & mask, n)[slot & 1]
                        elif cb in (orc.CB_SPEC1, orc.CB_STD1):
                            m, k = orc.hash_row(table, n)
                            v = orc.decode_hash_mask(int(want[slot]) & mask, m, k)
                        elif cb == orc.CB_MCG:
                            v = orc.decode_mcg(int(want[slot]) & mask)
                        else:
                            v = orc.decode_mul1(int(want[slot]) & mask)
                        assert got[perm[slot]] == v, (n, cb, wbits, slot)


def _digest(fields, ns, rows):
    # src/exl3/codebook_tables.zig:243-257
    h = hashlib.sha256()
    for n, r in zip(ns, rows):
        line = str(n) + "".join("," + format(v, "08x") for v in r[:fields]) + "\n"
        h.update(line.encode())
    return h.hexdigest()[:8]


def test_digest_fixed_vector():
    # src/exl3/codebook_tables.zig:281-285
    assert _digest(4, [24, 64], [(1, 2, 3, 4), (0xFFFFFFFF, 0, 0x80000000, 0x7FFFFFFF)]) == "72fc0906"


def test_oracle_tables_keep_their_pinned_digests():
    # src/exl3/codebook_tables.zig:287-307, :418-460
    ns = list(range(24, 65, 2))
    assert _digest(4, ns, [orc.pair1_row(n) for n in ns]) == "c089b4eb"
    ns15 = list(range(16, 129, 2))
    assert _digest(2, ns15, [orc.hash_row(orc.TABLE_SPEC1_W15, n) for n in ns15]) == "37f72431"
    assert _digest(2, ns, [orc.hash_row(orc.TABLE_SPEC1_W15, n) for n in ns]) == "2ac2594d"
    assert _digest(2, ns, [orc.hash_row(orc.TABLE_SPEC1_W16, n) for n in ns]) == "753ffa03"
    assert _digest(2, ns, [orc.hash_row(orc.TABLE_STD1, n) for n in ns]) == "c5dba171"
    assert _digest(2, ns15, [orc.hash_row(orc.TABLE_SPEC1_TEST, n) for n in ns15]) == "a2f2fe40"


# ------------------------------------------------------------------ encoder
TILE_FIXTURE_CONFIGS = [
    ("mcg_n24_w12", orc.CB_MCG, 12, 24), ("mcg_n32_w12", orc.CB_MCG, 12, 32),
    ("mcg_n40_w15", orc.CB_MCG, 15, 40), ("mcg_n40_w16", orc.CB_MCG, 16, 40),
    ("mcg_n48_w12", orc.CB_MCG, 12, 48), ("mcg_n56_w15", orc.CB_MCG, 15, 56),
    ("mcg_n64_w16", orc.CB_MCG, 16, 64), ("mcg_n36_w12", orc.CB_MCG, 12, 36),
    ("mul1_n24_w15", orc.CB_MUL1, 15, 24), ("mul1_n32_w12", orc.CB_MUL1, 12, 32),
    ("mul1_n40_w16", orc.CB_MUL1, 16, 40), ("mul1_n44_w12", orc.CB_MUL1, 12, 44),
    ("mul1_n64_w15", orc.CB_MUL1, 15, 64),
]


@pytest.mark.parametrize("name,cb,w,n", TILE_FIXTURE_CONFIGS)
def test_encoder_matches_reference_search_code_for_code(golden, name, cb, w, n):
    # src/encoder/encode.zig:464-485
    g = golden("exl3_encode_tiles")
    xs = g[f"{name}.x"]
    want = g[f"{name}.packed"]
    costs = g[f"{name}.cost"]
    for i in range(costs.shape[0]):
        packed, cost, _ = orc.encode_tile(xs[i], n, cb, w)
        np.testing.assert_array_equal(packed, want[i], err_msg=f"{name} tile {i}")
        assert abs(cost - costs[i]) <= 1e-12 * abs(costs[i])


def test_encoder_codes_decode_to_scored_values():
    # src/encoder/encode.zig:302-335
    rng = np.random.default_rng(7)
    for cb, w, n in ((orc.CB_MCG, 12, 24), (orc.CB_MCG, 15, 40), (orc.CB_MUL1, 12, 44), (orc.CB_MUL1, 16, 64)):
        for _ in range(2):
            tile = rng.standard_normal(256).astype(np.float32)
            packed, cost, recon = orc.encode_tile(tile, n, cb, w)
            dec = orc.decode_tile(packed, n, cb, w)
            np.testing.assert_array_equal(orc.f16_bits(recon), dec)
            sse = ((tile.astype(np.float64) - orc.f16_value(dec).astype(np.float64)) ** 2).sum()
            assert abs(sse - cost) <= 1e-9 * abs(cost)


def test_encoder_refuses_rates_and_windows():
    # src/encoder/encode.zig:487-503
    for n, w in ((41, 16), (8, 16), (128, 8), (32, 11)):
        with pytest.raises(ValueError):
            orc.encode_tile(np.zeros(256, np.float32), n, orc.CB_MCG, w)


TENSOR_CONFIGS = [
    ("mcg_n32_w12_r256_auto", orc.CB_MCG, 12, 32, 256, "auto"),
    ("mul1_n40_w12_r256_always", orc.CB_MUL1, 12, 40, 256, "always"),
    ("mcg_n24_w12_r256_never", orc.CB_MCG, 12, 24, 256, "never"),
    ("mcg_n40_w15_r128_auto", orc.CB_MCG, 15, 40, 128, "auto"),
    ("mul1_n64_w12_r128_always", orc.CB_MUL1, 12, 64, 128, "always"),
]


def _tensor_inputs(golden, rows):
    g = golden("exl3_encode_tensor")
    w = orc.f16_value(g["W"])[:rows]
    h = orc.f16_value(g["H"])[:rows, :rows]
    sign_in = g["sign_in_r256"] if rows == 256 else g["sign_in_r128"]
    return g, np.ascontiguousarray(w), np.ascontiguousarray(h), sign_in, g["sign_out"]


@pytest.mark.parametrize("rows,mode", [(256, "always"), (256, "never"), (256, "auto"), (128, "auto"), (128, "always")])
def test_regularize_matches_reference_scales(golden, rows, mode):
    # src/encoder/quantize.zig:683-712
    g, w, h, sign_in, sign_out = _tensor_inputs(golden, rows)
    hdiag = np.diag(h).copy()
    inner, suh, svh = orc.regularize(w, rows, 128, sign_in, sign_out, mode, hdiag)
    for name, got in (("suh", suh), ("svh", svh)):
        want = g[f"reg_r{rows}_{mode}.{name}"]
        assert np.all(np.abs(want - got) <= 2e-6 * np.abs(want) + 1e-9), name
    if rows == 256 and mode == "always":
        want = orc.f16_value(g["reg_r256_always.inner"])
        assert np.all(np.abs(want - inner) <= 1.5e-3 * np.abs(want) + 1e-5)


@pytest.mark.parametrize("name,cb,w,n,rows,mode", TENSOR_CONFIGS)
def test_whole_tensor_quantize_matches_reference(golden, name, cb, w, n, rows, mode):
    # src/encoder/quantize.zig:770-790
    g, wt, h, sign_in, sign_out = _tensor_inputs(golden, rows)
    packed, suh, svh, gs = orc.quantize_tensor(wt, h, rows, 128, sign_in, sign_out, n, cb, w, mode)
    np.testing.assert_array_equal(packed, g[f"{name}.packed"])
    lo, hi = (0.4, 1.2) if cb == orc.CB_MUL1 else (0.5, 1.5)
    assert lo < gs < hi
    assert abs(gs - float(g[f"{name}.g"][0])) <= 1e-5
    np.testing.assert_array_equal(suh, g[f"{name}.suh"])
    np.testing.assert_array_equal(svh, g[f"{name}.svh"])


def test_signs_pure_function_of_seed_and_name():
    # src/encoder/quantize.zig:792-808
    a = orc.signs(7, "language_model.model.layers.0.mlp.switch_mlp.gate_proj", 128)
    b = orc.signs(7, "language_model.model.layers.0.mlp.switch_mlp.gate_proj", 128)
    o = orc.signs(7, "language_model.model.layers.0.mlp.switch_mlp.up_proj", 128)
    r = orc.signs(8, "language_model.model.layers.0.mlp.switch_mlp.gate_proj", 128)
    np.testing.assert_array_equal(a, b)
    assert set(np.unique(a)) <= {-1.0, 1.0}
    assert not np.array_equal(a, o) and not np.array_equal(a, r)


def test_ldl_factor_carries_h10_equals_l10_h00():
    # src/encoder/quantize.zig:744-768
    n = 32
    rng = np.random.default_rng(5)
    a = rng.standard_normal((n, n)).astype(np.float32)
    h = (a @ a.T / n).astype(np.float32)
    l = orc.ldl_factor(h, n)
    mean = np.float32(np.diag(h).astype(np.float64).mean())
    for i in range(n):
        for j in range(n):
            if i // 16 == j // 16 or j > i:
                assert l[i, j] == 0
    h00 = h[:16, :16].astype(np.float64) + np.eye(16) * float(np.float32(np.float64(np.float32(0.025)) * np.float64(mean)))
    s = l[16:, :16].astype(np.float64) @ h00
    assert np.abs(s - h[16:, :16]).max() < 2e-4
