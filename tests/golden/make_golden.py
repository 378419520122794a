"""Regenerate the golden fixtures (golden.npz + manifest.json).

Compiles make_golden.cpp with the host C++ compiler, runs it, and packs its
arrays.  Expected outputs longer than STORE_LIMIT elements are kept only as a
SHA-256 digest of their little-endian bytes (the tests hash their own output
and compare); every input and every short output is stored in full.

Usage: python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import json
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
STORE_LIMIT = 4096
DTYPES = {"u32": np.uint32, "i32": np.int32, "f32": np.float32, "u64": np.uint64, "i64": np.int64, "u8": np.uint8}


def is_expected_output(name: str) -> bool:
    return any(tag in name for tag in ("_out", "inclusive", "exclusive", "_order", "minmax"))


def main() -> int:
    with tempfile.TemporaryDirectory(dir=HERE) as tmp:
        exe = Path(tmp) / "make_golden"
        subprocess.run(["g++", "-O2", "-std=c++17", str(HERE / "make_golden.cpp"), "-o", str(exe)],
                       check=True)
        out_dir = Path(tmp) / "arrays"
        out_dir.mkdir()
        subprocess.run([str(exe), str(out_dir)], check=True)
        arrays = {}
        manifest = {}
        for line in (out_dir / "arrays.txt").read_text().splitlines():
            name, dt, count = line.split()
            a = np.fromfile(out_dir / f"{name}.bin", dtype=DTYPES[dt])
            assert a.size == int(count), name
            store = not (is_expected_output(name) and a.size > STORE_LIMIT)
            manifest[name] = {
                "dtype": dt,
                "count": int(count),
                "sha256": hashlib.sha256(a.astype(a.dtype.newbyteorder("<")).tobytes()).hexdigest(),
                "stored": store,
            }
            if store:
                arrays[name] = a
    np.savez_compressed(HERE / "golden.npz", **arrays)
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(arrays)} stored arrays, {len(manifest)} manifest entries")
    return 0


if __name__ == "__main__":
    sys.exit(main())
