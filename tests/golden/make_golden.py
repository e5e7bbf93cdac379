"""Extract the reference's committed EXL3 fixtures into compact numpy archives.

The reference (beamivalice/sushi 1.7.2) pins its host decoder and CPU encoder with
safetensors fixtures written by the upstream converter:

  src/exl3/fixtures/exl3_{k2,k3,k4}_linear.safetensors          MUL1 packs, 128x128
  src/exl3/fixtures/exl3_{k2p5,k3}_mcg_linear.safetensors       MCG packs, 128x128
  src/exl3/fixtures/exl3_k2p5_mcg_w12_linear.safetensors        MCG at window 12
  src/exl3/fixtures/exl3_pair1_tiles.safetensors                PAIR1 tiles, every even n 24..64
  src/encoder/fixtures/exl3_encode_tiles.safetensors            per-tile Viterbi codes + costs
  src/encoder/fixtures/exl3_encode_tensor.safetensors           whole-tensor quantize results

Their tests are `src/exl3/expert_exl3.zig:797-997`, `src/encoder/encode.zig:464-485` and
`src/encoder/quantize.zig:683-800`.  This script is run once in a container where the
reference tree is mounted and writes `tests/golden/*.npz`; the tests read only those
archives, so nothing at test time needs the reference tree.  Each archive keeps every
tensor under its original name, with its dtype (u16 bit patterns for F16/U16 data).

Usage: python tests/golden/make_golden.py <reference-root>
"""

import json
import os
import struct
import sys

import numpy as np

_DT = {
    "F16": np.uint16,  # kept as raw bit patterns: the tests compare bits
    "U16": np.uint16,
    "F32": np.float32,
    "F64": np.float64,
    "U8": np.uint8,
    "U32": np.uint32,
    "I32": np.int32,
}

FIXTURES = [
    ("src/exl3/fixtures/exl3_k2_linear.safetensors", "exl3_k2_linear"),
    ("src/exl3/fixtures/exl3_k3_linear.safetensors", "exl3_k3_linear"),
    ("src/exl3/fixtures/exl3_k4_linear.safetensors", "exl3_k4_linear"),
    ("src/exl3/fixtures/exl3_k2p5_mcg_linear.safetensors", "exl3_k2p5_mcg_linear"),
    ("src/exl3/fixtures/exl3_k3_mcg_linear.safetensors", "exl3_k3_mcg_linear"),
    ("src/exl3/fixtures/exl3_k2p5_mcg_w12_linear.safetensors", "exl3_k2p5_mcg_w12_linear"),
    ("src/exl3/fixtures/exl3_pair1_tiles.safetensors", "exl3_pair1_tiles"),
    ("src/encoder/fixtures/exl3_encode_tiles.safetensors", "exl3_encode_tiles"),
    ("src/encoder/fixtures/exl3_encode_tensor.safetensors", "exl3_encode_tensor"),
]


def read_safetensors(path):
    raw = open(path, "rb").read()
    (hlen,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8 : 8 + hlen])
    data = raw[8 + hlen :]
    out = {}
    for name, spec in header.items():
        if name == "__metadata__":
            continue
        start, end = spec["data_offsets"]
        arr = np.frombuffer(data[start:end], dtype=_DT[spec["dtype"]]).reshape(spec["shape"])
        out[name] = arr.copy()
    return out


def main(ref_root):
    here = os.path.dirname(os.path.abspath(__file__))
    for rel, stem in FIXTURES:
        tensors = read_safetensors(os.path.join(ref_root, rel))
        dst = os.path.join(here, stem + ".npz")
        np.savez_compressed(dst, **tensors)
        print(f"{stem}: {len(tensors)} tensors -> {os.path.relpath(dst)}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference-root>")
    main(sys.argv[1])
