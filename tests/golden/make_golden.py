"""Writes tests/golden/reference_luts.json from the reference's own LUT source.

Usage: python tests/golden/make_golden.py <reference checkout root>
(a read-only checkout of atimics/nsrl).  The fixture records, for each of the three 8-bit tables of
crates/nsrl-core/src/rsqrt_lut_8bit.rs, its length, its FNV-1a-64 hash over
little-endian bytes and its first and last entries, so that tables derived
from their mathematical definitions can be pinned to the reference's values
without the reference being present at test time.
"""
import json
import os
import re
import struct
import sys

LUT_SOURCE = "crates/nsrl-core/src/rsqrt_lut_8bit.rs"
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_luts.json")


def fnv(data: bytes) -> int:
    h = 0xCBF29CE484222325
    for b in data:
        h = ((h ^ b) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def table(src, name):
    m = re.search(name + r": \[[^\]]+\] = \[(.*?)\];", src, re.S)
    return [int(x) for x in m.group(1).replace("\n", " ").split(",") if x.strip()]


def main(reference_root: str):
    src = open(os.path.join(reference_root, LUT_SOURCE)).read()
    out = {"source": "crates/nsrl-core/src/rsqrt_lut_8bit.rs"}
    for name, fmt in (("RSQRT_LUT_8BIT", "<h"), ("EXP2_NEG_FRAC_LUT_8BIT", "<h"), ("RECIP_LUT_8BIT_Q31", "<I")):
        vals = table(src, name)
        data = b"".join(struct.pack(fmt, v) for v in vals)
        out[name] = {"len": len(vals), "fnv1a64": "0x%016x" % fnv(data), "first": vals[0], "last": vals[-1]}
    with open(OUT, "w") as f:
        json.dump(out, f, indent=1)
        f.write("\n")
    print(OUT)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout root>")
    main(sys.argv[1])
