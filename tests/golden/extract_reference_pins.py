"""Generate ``ornith_pins.json`` from the reference's own unit-test source.

The reference pins its decode against four raw blocks of a real Q4_K_M GGUF
(two Q6_K, two Q4_K; crates/unltd-tensor/src/quants.rs:1094-1152) with
expected dot products and single weights computed by gguf-py
(quants.rs:1169-1198, deterministic x formulas at :1157-1166, tolerance 1e-4).
This script reads that Rust file as text and writes the bytes and expected
values as a JSON fixture, so the tests can pin the oracle without the
reference tree being present.

Usage: python tests/golden/extract_reference_pins.py path/to/quants.rs
   or: UNLTD_REFERENCE=<reference checkout> python tests/golden/extract_reference_pins.py
"""
from __future__ import annotations

import json
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
QUANTS_RS = "crates/unltd-tensor/src/quants.rs"


def extract(src_text: str) -> dict:
    blocks = {}
    for name, n in (("Q6K_B0", 210), ("Q6K_B15", 210), ("Q4K_B0", 144), ("Q4K_B15", 144)):
        m = re.search(r"const %s: \[u8; %d\] = \[(.*?)\];" % (name, n), src_text, re.S)
        if not m:
            raise SystemExit(f"block {name} not found")
        vals = [int(t, 16) for t in re.findall(r"0x[0-9a-fA-F]{2}", m.group(1))]
        assert len(vals) == n, (name, len(vals))
        blocks[name] = bytes(vals).hex()
    m = re.search(r"let cases: \[\(&\[u8\], f64, f64, f64, f64\); 4\] = \[(.*?)\];", src_text, re.S)
    if not m:
        raise SystemExit("cases table not found")
    cases = []
    for cm in re.finditer(r"\(\s*&(\w+),\s*([-0-9.e]+),\s*([-0-9.e]+),\s*([-0-9.e]+),\s*([-0-9.e]+),\s*\)", m.group(1)):
        cases.append(
            {
                "block": cm.group(1),
                "dot_x_pattern": float(cm.group(2)),
                "dot_x_alt": float(cm.group(3)),
                "w7": float(cm.group(4)),
                "w200": float(cm.group(5)),
            }
        )
    assert len(cases) == 4, cases
    return {
        "source": "crates/unltd-tensor/src/quants.rs:1094-1198 (ornith_decode_pin)",
        "tolerance": 1e-4,
        "x_pattern": "x[i] = ((i*7919) % 1009) / 1009 - 0.5 (f32)",
        "x_alt": "x[i] = ((i*31 + 17) % 257) / 257 - 0.5 (f32)",
        "blocks_hex": blocks,
        "cases": cases,
    }


def main() -> None:
    if len(sys.argv) > 1:
        src = sys.argv[1]
    elif os.environ.get("UNLTD_REFERENCE"):
        src = os.path.join(os.environ["UNLTD_REFERENCE"], QUANTS_RS)
    else:
        raise SystemExit("give the path of quants.rs, or set UNLTD_REFERENCE to the reference checkout")
    with open(src, encoding="utf-8") as f:
        data = extract(f.read())
    out = os.path.join(HERE, "ornith_pins.json")
    with open(out, "w") as f:
        json.dump(data, f, indent=1)
    print("wrote", out)


if __name__ == "__main__":
    main()
