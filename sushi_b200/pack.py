"""EXL3 / STQ pack admission and loading on the host (the reference's `root.parseExpertQuant`,
`codebook_tables.resolve`, shard stamps and `trellisAdmitted`, src/exl3/root.zig:189-297, :449;
src/exl3/codebook_tables.zig:266-280; pack layout docs/pack-format.md).

A pack's `config.json` carries an `expert_quant` block: format (`exl3`, or `stq` for the tabled
codebooks), rate `k`, codebook, codeword window, the STQ table by name and digest, and the routed
experts' tile order.  `parse_expert_quant` turns it into a Spec or refuses by the reference's error
name; `decode_of(spec)` is the `sushi_b200.Decode` the kernels take.  `SafeTensors` reads a shard's
header and tensors (trellis `U16`, scales `F16`) without copying the file, and `load` puts a
tensor on the device.
"""

import json
import math
import struct
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from . import exl3

MIN_N, MAX_N = 16, 128  # format.Rate bounds: K1 .. K8 (src/exl3/expert_exl3.zig:180-241)
WINDOWS = range(8, 17)  # format.Window: the codeword widths this build decodes
TABLED = {exl3.Codebook.SPEC1, exl3.Codebook.STD1, exl3.Codebook.PAIR1}  # Codebook.hasTable
HASH_MASK = {exl3.Codebook.SPEC1, exl3.Codebook.STD1}  # Codebook.tabledHashMask
CODEBOOK_NAMES = {"mcg": exl3.Codebook.MCG, "mul1": exl3.Codebook.MUL1, "std1": exl3.Codebook.STD1,
                  "spec1": exl3.Codebook.SPEC1, "pair1": exl3.Codebook.PAIR1}
# Digests a table replaced (codebook_tables.zig:103): a config stamped with one is a legacy pack.
SUPERSEDED = {"spec1-w15": ("2ac2594d",)}


class Exl3ConfigError(ValueError):
    """A pack refused by name: `name` is the reference's error (`ExpertLayoutUnsupported`, ...)."""

    def __init__(self, name: str):
        super().__init__(name)
        self.name = name


@dataclass
class Spec:
    n: int                               # packed halfwords per tile (rate K = n / 16)
    codebook: "exl3.Codebook"
    window: int = 16
    rates: Optional[frozenset] = None    # the rates the pack's table has rows for; None admits all
    table: Optional[int] = None          # the STQ table's index (SX_TABLE_*)
    tile_order: "exl3.TileOrder" = field(default=exl3.TileOrder.PACK)


def _tables():
    out = {}
    for i in range(5):
        info = exl3.table_info(i)
        info["index"] = i
        info["rates"] = frozenset(info["n_lo"] + 2 * r for r in range(info["rows"]))
        out[info["name"]] = info
    return out


def rate_from_config_k(k) -> Optional[int]:
    """rateFromConfigK (root.zig:205): k integer or fractional with 16k an even whole number of
    halfwords in 16..128; else None."""
    if isinstance(k, bool) or not isinstance(k, (int, float)):
        return None
    scaled = float(k) * 16.0
    rounded = round(scaled)
    if abs(scaled - rounded) > 1e-6 or rounded < 0 or rounded > 1024:
        return None
    n = int(rounded)
    return n if MIN_N <= n <= MAX_N and n % 2 == 0 else None


def window_from_config(v) -> Optional[int]:
    """windowFromConfig (root.zig:219): absent is 16; an integer 8..16; anything else None."""
    if v is None:
        return 16
    if isinstance(v, bool) or not isinstance(v, int):
        return None
    return v if v in WINDOWS else None


def resolve_table(block: dict, codebook, window: int) -> dict:
    """codebook_tables.resolve (codebook_tables.zig:266): the table the block names, by name."""
    if codebook not in TABLED:
        raise Exl3ConfigError("Exl3CodebookTableCodebookMismatch")
    name = block.get("codebook_table")
    tables = _tables()
    if not isinstance(name, str) or name not in tables:
        raise Exl3ConfigError("Exl3CodebookTableUnknown")
    table = tables[name]
    digest = block.get("codebook_digest")
    if not isinstance(digest, str):
        raise Exl3ConfigError("Exl3CodebookTableDigestMismatch")
    if digest in SUPERSEDED.get(name, ()):
        raise Exl3ConfigError("Exl3CodebookTableLegacyConfig")
    if digest != table["digest"]:
        raise Exl3ConfigError("Exl3CodebookTableDigestMismatch")
    if exl3.Codebook(table["codebook"]) != codebook:
        raise Exl3ConfigError("Exl3CodebookTableCodebookMismatch")
    if codebook not in HASH_MASK and table["window_bits"] != window:  # Table.admits
        raise Exl3ConfigError("Exl3CodebookTableWindowMismatch")
    return table


def parse_quant_block(block) -> Spec:
    """parseQuantBlock (root.zig:236): format, k, codebook, window and the STQ table."""
    if not isinstance(block, dict):
        raise Exl3ConfigError("ExpertLayoutUnsupported")
    fmt = block.get("format")
    if not isinstance(fmt, str) or fmt not in ("stq", "exl3"):
        raise Exl3ConfigError("ExpertLayoutUnsupported")
    stq = fmt == "stq"
    n = rate_from_config_k(block.get("k"))
    if "k" not in block or n is None:
        raise Exl3ConfigError("ExpertLayoutUnsupported")
    cb_name = block.get("codebook")
    if not isinstance(cb_name, str) or cb_name not in CODEBOOK_NAMES:
        raise Exl3ConfigError("ExpertLayoutUnsupported")
    codebook = CODEBOOK_NAMES[cb_name]
    if (codebook in TABLED) != stq:
        raise Exl3ConfigError("ExpertLayoutUnsupported")
    window = window_from_config(block.get("window"))
    if window is None:
        raise Exl3ConfigError("Exl3WindowUnsupported")
    if codebook not in TABLED:
        if "codebook_table" in block:
            raise Exl3ConfigError("Exl3CodebookTableCodebookMismatch")
        return Spec(n=n, codebook=codebook, window=window)
    table = resolve_table(block, codebook, window)
    if n not in table["rates"]:
        raise Exl3ConfigError("Exl3CodebookTableRateMissing")
    return Spec(n=n, codebook=codebook, window=window, rates=table["rates"], table=table["index"])


def parse_expert_quant(config: dict) -> Spec:
    """parseExpertQuant (root.zig:225): the config's `expert_quant` block, plus its tile order
    (`pair_major`; absent is the pack order; anything else refused by name)."""
    block = config.get("expert_quant") if isinstance(config, dict) else None
    if block is None:
        raise Exl3ConfigError("ExpertLayoutUnsupported")
    spec = parse_quant_block(block)
    if "tile_order" in block:
        if block["tile_order"] != "pair_major":
            raise Exl3ConfigError("Exl3TileOrderUnsupported")
        spec.tile_order = exl3.TileOrder.PAIR_MAJOR
    return spec


def decode_of(spec: Spec) -> "exl3.Decode":
    return exl3.Decode(spec.codebook, spec.window, spec.table)


def shard_tile_order_agrees(order, stamp: Optional[str]) -> None:
    """shardTileOrderAgrees (root.zig:258): a shard stamps `pair_major` or nothing (pack order)."""
    if stamp is None:
        stamped = exl3.TileOrder.PACK
    elif stamp == "pair_major":
        stamped = exl3.TileOrder.PAIR_MAJOR
    else:
        raise Exl3ConfigError("Exl3ShardStampMismatch")
    if stamped != exl3.TileOrder(order):
        raise Exl3ConfigError("Exl3ShardStampMismatch")


def shard_stamp_agrees(spec: Spec, k: Optional[str], codebook: Optional[str], window: Optional[str]) -> None:
    """shardStampAgrees (root.zig:263): a shard's k / codebook / window stamps against the spec; a
    narrower k is over-billed (admitted), a wider one refused."""
    if codebook is not None and CODEBOOK_NAMES.get(codebook) != spec.codebook:
        raise Exl3ConfigError("Exl3ShardStampMismatch")
    if window is not None:
        try:
            w = int(window, 10)
        except ValueError:
            raise Exl3ConfigError("Exl3ShardStampMismatch") from None
        if w not in WINDOWS or w != spec.window:
            raise Exl3ConfigError("Exl3ShardStampMismatch")
    if k is not None:
        try:
            rk = float(k)
        except ValueError:
            raise Exl3ConfigError("Exl3ShardStampMismatch") from None
        if not math.isfinite(rk):
            raise Exl3ConfigError("Exl3ShardStampMismatch")
        scaled = round(rk * 16.0)
        if abs(rk * 16.0 - scaled) > 1e-6 or scaled < MIN_N or scaled > MAX_N or scaled % 2:
            raise Exl3ConfigError("Exl3ShardStampMismatch")
        if scaled > spec.n:
            raise Exl3ConfigError("Exl3ShardStampMismatch")


def trellis_admitted(shape, experts: int, in_dim: int, out_dim: int, n: int) -> bool:
    """trellisAdmitted (root.zig:449): [experts, in/16, out/16, n_packed] with n_packed a rate at or
    below the billed one."""
    if len(shape) != 4 or any(d <= 0 for d in shape) or in_dim % 16 or out_dim % 16:
        return False
    if list(shape[:3]) != [experts, in_dim // 16, out_dim // 16]:
        return False
    packed = shape[3]
    return MIN_N <= packed <= MAX_N and packed % 2 == 0 and packed <= n


# ------------------------------------------------------------------ safetensors shards
_DTYPES = {"U16": np.uint16, "I16": np.int16, "F16": np.float16, "BF16": np.uint16, "F32": np.float32,
           "U32": np.uint32, "I32": np.int32, "U8": np.uint8, "I64": np.int64}


class SafeTensors:
    """A safetensors shard: an 8-byte little-endian header length, a JSON header (tensor name ->
    dtype, shape, data offsets; `__metadata__` for the shard's stamps) and the data, read through
    a memory map."""

    def __init__(self, path: str):
        self.path = path
        with open(path, "rb") as f:
            (hlen,) = struct.unpack("<Q", f.read(8))
            header = json.loads(f.read(hlen))
        self.metadata = header.pop("__metadata__", {}) or {}
        self.entries = header
        self._data = np.memmap(path, dtype=np.uint8, mode="r", offset=8 + hlen)

    def names(self):
        return list(self.entries)

    def shape(self, name):
        return tuple(self.entries[name]["shape"])

    def numpy(self, name) -> np.ndarray:
        e = self.entries[name]
        if e["dtype"] not in _DTYPES:
            raise Exl3ConfigError("BadExl3Dtype")
        a, b = e["data_offsets"]
        return np.frombuffer(self._data[a:b], dtype=_DTYPES[e["dtype"]]).reshape(e["shape"])

    def load(self, name, device="cuda"):
        """The tensor on the device; U16 trellis words arrive as int16 bit patterns."""
        import torch

        a = self.numpy(name)
        if a.dtype == np.uint16:
            a = a.view(np.int16)
        return torch.from_numpy(np.array(a)).to(device)  # a private copy of the mapped bytes

    def proj(self, prefix: str, spec: Spec, device="cuda") -> "exl3.Proj":
        """One projection `{prefix}.trellis` (or `.trellis_pm` under pair_major, converted to the pack
        order the kernels read), `{prefix}.suh`, `{prefix}.svh`."""
        shard_tile_order_agrees(spec.tile_order, self.metadata.get("tile_order"))
        if spec.tile_order == exl3.TileOrder.PAIR_MAJOR:
            pm = self.load(prefix + ".trellis_pm", device)
            tr = exl3.tile_order_convert(pm, exl3.TileOrder.PACK, exl3.TileOrder.PAIR_MAJOR)
        else:
            tr = self.load(prefix + ".trellis", device)
        if tr.dim() == 3:
            tr = tr.unsqueeze(0)
        su = self.load(prefix + ".suh", device)
        sv = self.load(prefix + ".svh", device)
        experts, it, ot, n = tr.shape
        if not trellis_admitted(tr.shape, experts, it * 16, ot * 16, spec.n):
            raise Exl3ConfigError("BadExl3Shape")
        return exl3.Proj(tr, su.reshape(experts, -1), sv.reshape(experts, -1))


def write_safetensors(path: str, tensors: dict, metadata: Optional[dict] = None) -> None:
    """Writes numpy arrays as a safetensors shard (U16 / F16 / F32 / I32 ...), for packs made here."""
    rev = {np.dtype(np.uint16): "U16", np.dtype(np.int16): "I16", np.dtype(np.float16): "F16",
           np.dtype(np.float32): "F32", np.dtype(np.uint32): "U32", np.dtype(np.int32): "I32", np.dtype(np.uint8): "U8"}
    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        b = a.tobytes()
        header[name] = {"dtype": rev[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    raw = json.dumps(header).encode()
    raw += b" " * ((8 - len(raw) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        for b in blobs:
            f.write(b)
