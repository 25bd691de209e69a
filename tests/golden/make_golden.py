"""Generates tests/golden/iq2_tables.json from the reference tree.

Run in the build container (where the pulsar reference is mounted):
    python tests/golden/make_golden.py /path/to/pulsar
It parses the reference's CUDA tables crates/kernels/cuda/iq2_tables.inc
(cuda_iq2xxs_grid[256] u64, cuda_ksigns_iq2xs[128] u8) and stores only
their SHA-256 digests over the little-endian bytes, so the tests can pin
the grid this project derives from the packed 2-bit points without
carrying a copy of the table.
"""
import hashlib
import json
import os
import re
import sys


def parse(src: str, name: str):
    body = src.split(name, 1)[1].split("{", 1)[1].split("}", 1)[0]
    return [int(t, 0) for t in re.findall(r"0x[0-9a-fA-F]+|\d+", body)]


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PULSAR_REFERENCE")
    if not ref:  # BASELINE.json names the reference tree
        ref = json.load(open(os.path.join(os.path.dirname(__file__), "..", "..", "BASELINE.json")))["reference_path"]
    src = open(os.path.join(ref, "crates/kernels/cuda/iq2_tables.inc")).read()
    grid = parse(src, "cuda_iq2xxs_grid[256]")
    ks = parse(src, "cuda_ksigns_iq2xs[128]")
    assert len(grid) == 256 and len(ks) == 128
    out = {
        "source": "crates/kernels/cuda/iq2_tables.inc (cuda_iq2xxs_grid, cuda_ksigns_iq2xs)",
        "iq2xxs_grid_sha256": hashlib.sha256(b"".join(g.to_bytes(8, "little") for g in grid)).hexdigest(),
        "ksigns_iq2xs_sha256": hashlib.sha256(bytes(ks)).hexdigest(),
    }
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "iq2_tables.json")
    json.dump(out, open(path, "w"), indent=1)
    print(path, out)


if __name__ == "__main__":
    main()
