"""Pack admission on the host: the reference's config cases (src/exl3/root.zig:294-533 tests, read
as golden cases) against sushi_b200.pack, and safetensors shards written and read back."""

import json

import numpy as np
import pytest

from sushi_b200 import exl3
from sushi_b200 import pack as P

SPEC1_TABLE = {"codebook_table": "spec1-w15", "codebook_digest": "37f72431"}
PAIR1_TABLE = {"codebook_table": "pair1-w16-v1", "codebook_digest": "c089b4eb"}
STD1_TABLE = {"codebook_table": "std1", "codebook_digest": "c5dba171"}


def spec(**block):
    return P.parse_expert_quant({"expert_quant": block})


def refused(name, **block):
    with pytest.raises(P.Exl3ConfigError) as e:
        spec(**block)
    assert e.value.name == name, e.value.name


def test_window_is_16_unless_the_config_names_a_decodable_one():
    base = dict(format="exl3", k=2.5, codebook="mcg")
    assert spec(**base).window == 16 and spec(**base, window=16).window == 16
    for w in (12, 11, 10, 8):
        assert spec(**base, window=w).window == w
    for bad in (17, 7, "12"):
        refused("Exl3WindowUnsupported", **base, window=bad)


def test_tile_order():
    base = dict(format="exl3", k=2.5, codebook="mcg")
    assert spec(**base).tile_order == exl3.TileOrder.PACK
    assert spec(**base, tile_order="pair_major").tile_order == exl3.TileOrder.PAIR_MAJOR
    for bad in ("pack", "Pair_Major", "", 1, None, True):
        refused("Exl3TileOrderUnsupported", **base, tile_order=bad)


def test_unknown_codebook_and_format():
    refused("ExpertLayoutUnsupported", format="exl3", k=2.5, codebook="mul2", window=12)
    refused("ExpertLayoutUnsupported", format="stq", k=2.5, codebook="mcg")
    refused("ExpertLayoutUnsupported", format="exl3", k=2.5, codebook="std1", window=15, **STD1_TABLE)
    refused("ExpertLayoutUnsupported", format="exq", k=2.5, codebook="mcg")
    with pytest.raises(P.Exl3ConfigError):
        P.parse_expert_quant({})


def test_stq_tables_and_their_rates():
    s1 = spec(format="stq", k=2.5, codebook="spec1", window=15, **SPEC1_TABLE)
    assert s1.codebook == exl3.Codebook.SPEC1 and s1.n == 40
    p1 = spec(format="stq", k=3, codebook="pair1", window=16, **PAIR1_TABLE)
    assert p1.codebook == exl3.Codebook.PAIR1
    assert all(n in p1.rates for n in (24, 32, 36, 48, 64))
    assert not any(n in p1.rates for n in (16, 22, 66, 128))
    assert all(n in s1.rates for n in (16, 22, 66, 128)) and 14 not in s1.rates and 130 not in s1.rates
    assert spec(format="exl3", k=3, codebook="mcg").rates is None  # no table: every rate


def test_spec1_decodes_at_every_window_pair1_only_at_its_own():
    for w in P.WINDOWS:
        s = spec(format="stq", k=2.5, codebook="spec1", window=w, **SPEC1_TABLE)
        assert s.window == w and s.table == 1
    assert spec(format="stq", k=2, codebook="spec1", **SPEC1_TABLE).window == 16
    named = spec(format="stq", k=3, codebook="spec1", window=8, codebook_table="spec1-test-per-rate",
                 codebook_digest="a2f2fe40")
    assert named.table == 4
    refused("Exl3WindowUnsupported", format="stq", k=2, codebook="spec1", window=7, **SPEC1_TABLE)
    refused("Exl3CodebookTableWindowMismatch", format="stq", k=2, codebook="pair1", window=15, **PAIR1_TABLE)
    for w in P.WINDOWS:
        s = spec(format="stq", k=2.5, codebook="std1", window=w, **STD1_TABLE)
        assert s.codebook == exl3.Codebook.STD1 and s.table == 3


def test_missing_foreign_or_legacy_table():
    head = dict(format="stq", k=2, codebook="spec1", window=15)
    refused("Exl3CodebookTableUnknown", **head)
    refused("Exl3CodebookTableUnknown", **head, codebook_table="spec1-w15-v2", codebook_digest="c5dba171")
    refused("Exl3CodebookTableDigestMismatch", **head, codebook_table="spec1-w15", codebook_digest="00000000")
    refused("Exl3CodebookTableCodebookMismatch", **head, **STD1_TABLE)
    refused("Exl3CodebookTableCodebookMismatch", **head, **PAIR1_TABLE)
    refused("Exl3CodebookTableWindowMismatch", format="stq", k=2, codebook="pair1", window=15, **PAIR1_TABLE)
    refused("Exl3CodebookTableLegacyConfig", **head, codebook_table="spec1-w15", codebook_digest="2ac2594d")
    refused("Exl3CodebookTableRateMissing", format="stq", k=1, codebook="pair1", **PAIR1_TABLE)
    refused("Exl3CodebookTableRateMissing", format="stq", k=4.5, codebook="std1", window=15, **STD1_TABLE)
    refused("Exl3CodebookTableCodebookMismatch", format="exl3", k=2, codebook="mcg", **SPEC1_TABLE)


@pytest.mark.parametrize("k,n", [(2, 32), (2.5, 40), (2.75, 44), (3, 48), (3.5, 56), (4, 64)])
def test_integer_and_fractional_k_under_every_codebook(k, n):
    keys = {"spec1": dict(window=15, **SPEC1_TABLE), "std1": dict(window=15, **STD1_TABLE), "pair1": PAIR1_TABLE}
    for name, cb in P.CODEBOOK_NAMES.items():
        fmt = "stq" if cb in P.TABLED else "exl3"
        s = spec(format=fmt, k=k, codebook=name, **keys.get(name, {}))
        assert s.n == n and s.codebook == cb


def test_k_off_the_rate_grid_is_refused():
    for bad in (2.3, 8.125, 9, 0.875, 2.0625):
        refused("ExpertLayoutUnsupported", format="exl3", k=bad, codebook="mul1")
    refused("ExpertLayoutUnsupported", format="exl3", k=4, codebook="mul2")


def test_shard_stamps():
    s = spec(format="exl3", k=2.5, codebook="mcg", window=12)
    P.shard_stamp_agrees(s, "2.5", "mcg", "12")
    P.shard_stamp_agrees(s, "2", None, None)  # a narrower k is over-billed, not wrong
    for k, cb, w in (("3", None, None), (None, "mul1", None), (None, None, "16"), ("2.3", None, None), ("inf", None, None)):
        with pytest.raises(P.Exl3ConfigError):
            P.shard_stamp_agrees(s, k, cb, w)
    P.shard_tile_order_agrees(exl3.TileOrder.PACK, None)
    P.shard_tile_order_agrees(exl3.TileOrder.PAIR_MAJOR, "pair_major")
    for order, stamp in ((exl3.TileOrder.PACK, "pair_major"), (exl3.TileOrder.PAIR_MAJOR, None), (exl3.TileOrder.PACK, "x")):
        with pytest.raises(P.Exl3ConfigError):
            P.shard_tile_order_agrees(order, stamp)


def test_trellis_admitted_below_the_billed_rate():
    assert P.trellis_admitted((4, 8, 16, 32), 4, 128, 256, 40)
    assert P.trellis_admitted((4, 8, 16, 40), 4, 128, 256, 40)
    assert not P.trellis_admitted((4, 8, 16, 48), 4, 128, 256, 40)
    assert not P.trellis_admitted((4, 8, 16, 33), 4, 128, 256, 40)
    assert not P.trellis_admitted((3, 8, 16, 32), 4, 128, 256, 40)


def test_safetensors_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    tr = rng.integers(0, 1 << 16, size=(2, 8, 8, 32), dtype=np.uint16)
    su = rng.standard_normal((2, 128)).astype(np.float16)
    sv = rng.standard_normal((2, 128)).astype(np.float16)
    path = str(tmp_path / "model-00001.safetensors")
    P.write_safetensors(path, {"mlp.gate_proj.trellis": tr, "mlp.gate_proj.suh": su, "mlp.gate_proj.svh": sv},
                        {"k": "2", "codebook": "mcg"})
    st = P.SafeTensors(path)
    assert st.metadata == {"k": "2", "codebook": "mcg"}
    assert st.shape("mlp.gate_proj.trellis") == (2, 8, 8, 32)
    np.testing.assert_array_equal(st.numpy("mlp.gate_proj.trellis"), tr)
    np.testing.assert_array_equal(st.numpy("mlp.gate_proj.suh"), su)
    s = spec(format="exl3", k=2, codebook="mcg")
    P.shard_stamp_agrees(s, st.metadata.get("k"), st.metadata.get("codebook"), st.metadata.get("window"))
    proj = st.proj("mlp.gate_proj", s, device="cpu")
    assert proj.dims() == (2, 128, 128, 32)
    raw = json.loads(open(path, "rb").read()[8:8 + int.from_bytes(open(path, "rb").read(8), "little")])
    assert raw["mlp.gate_proj.trellis"]["dtype"] == "U16"
