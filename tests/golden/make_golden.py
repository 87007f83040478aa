"""Generate ``packed_golden.json``: the reference's own golden vectors for the packed path.

The reference (tinygrad-dx12) cannot be imported in this container: tinygrad is not
installed and the package needs Python >= 3.14. Its tests are therefore read as text.

* The exhaustive FP4/FP6 payload tables are extracted from the ``GOLDEN`` dict literal of
  ``test/backend/test_packed.py:8-78`` with ``ast.literal_eval`` (no reference code runs).
* The known-answer tests are transcribed below, each with the file:line it comes from.

Run from the repository root with the reference checked out at ``--reference``::

    python tests/golden/make_golden.py --reference <path-to-tinygrad-dx12>

The output file is committed; tests only read it.
"""

from __future__ import annotations

import argparse
import ast
import json
import pathlib


def extract_golden(test_file: pathlib.Path) -> dict:
    tree = ast.parse(test_file.read_text())
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(isinstance(t, ast.Name) and t.id == "GOLDEN" for t in node.targets):
            table = ast.literal_eval(node.value)
            return {k: [float(v) for v in vals] for k, vals in table.items()}
    raise SystemExit("GOLDEN table not found")


def known_answers() -> dict:
    """Known-answer tests transcribed from the reference tests (inputs and expected outputs)."""
    return {
        # test_packed.py:104-108 -- same 8 bytes (codes 0..15, LSB first) decoded as int4 / uint4
        "integer_nibbles": {
            "codes": list(range(16)),
            "int4": list(range(8)) + list(range(-8, 0)),
            "uint4": list(range(16)),
        },
        # test_packed.py:111-115 -- K-block scales stay with their blocks
        "scales_stay_with_k_blocks": {
            "data": [0x22, 0x22], "format": "fp4_e2m1", "shape": [1, 4], "scales": [[2.0, 7.0]],
            "scale_dtype": "float32", "block_size": 2, "rhs": [[1.0], [2.0], [3.0], [4.0]], "expected": [[55.0]],
        },
        # test_packed.py:118-124 -- fp32 activations are never quantised to FP8
        "matrix_intermediate": {
            "fp6_e2m3_unscaled_with_float32": "float32",
            "fp6_e2m3_unscaled_pair": "fp8e4m3",
            "unpack_fp8e5m2_code0": [[0.0]],
        },
        # test_packed.py:127-144 -- FP64 scales keep their fraction bits
        "double_block_scales": {
            "data": [0x22], "format": "fp4_e2m1", "shape": [1, 2],
            "scales": [[1099511627776.25, -1099511627776.0]], "scale_dtype": "float64", "block_size": 1,
            "unpack": [[1099511627776.25, -1099511627776.0]], "unpack_dtype": "float64",
            "intermediate": "float64", "rhs": [[1.0], [1.0]], "matmul": [[0.25]],
        },
        # test_packed.py:147-174 -- decode across signed 32-bit bit/element offsets,
        # backing store = 17-byte pattern (i*37+13)%256 repeated; scales [2,7,11] cycled per 32
        "large_bit_positions": {
            "pattern": [(i * 37 + 13) % 256 for i in range(17)],
            "cases": [[fmt, kind, False] for fmt in ("uint4", "fp6_e2m3", "fp6_e3m2") for kind in ("bit", "element")]
            + [["uint4", "element", True]],
            "scale_cycle": [2.0, 7.0, 11.0],
            "window": [-3, 7],
        },
        # test_linalg.py:202-218 -- packed integer matmul keeps integer precision
        "packed_integer_matmul_precision": [
            {"format": "int4", "byte": 0xF1, "dtype": "int32", "values": [16777217, 16777219], "expected": -2},
            {"format": "int4", "byte": 0xF1, "dtype": "int64", "values": [1099511627777, 1099511627779], "expected": -2},
            {"format": "uint4", "byte": 0x31, "dtype": "uint64", "values": [1099511627777, 1099511627779],
             "expected": 4398046511114},
        ],
        # test_linalg.py:221-230 -- accumulator width for narrow integer matrices
        "accumulator_width": [
            {"dtype": "int8", "values": [100, 120], "acc": "int32", "expected": 24400},
            {"dtype": "uint8", "values": [200, 250], "acc": "uint32", "expected": 102500},
        ],
        # README.md:153-167 -- documented uint4 example
        "readme_uint4": {
            "data": [0x21, 0x43], "format": "uint4", "shape": [2, 2], "unpack": [[1, 2], [3, 4]],
            "column": [[1.0], [2.0]], "matmul": [[5.0], [11.0]], "vector": [1.0, 2.0], "matvec": [5.0, 11.0],
        },
        # scripts/benchmark_dtypes.py:70-74 -- {-1,0,1} payload maps used by the reference benchmark
        "benchmark_code_maps": {
            "fp6_e2m3": {"-1": 40, "0": 0, "1": 8},
            "fp6_e3m2": {"-1": 44, "0": 0, "1": 12},
            "fp4_e2m1": {"-1": 10, "0": 0, "1": 2},
            "int4": {"-1": 15, "0": 0, "1": 1},
        },
    }


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=pathlib.Path)
    ap.add_argument("--out", type=pathlib.Path, default=pathlib.Path(__file__).with_name("packed_golden.json"))
    args = ap.parse_args()
    golden = extract_golden(args.reference / "test" / "backend" / "test_packed.py")
    doc = {
        "source": "tinygrad-dx12 test/backend/test_packed.py, test/backend/test_linalg.py, README.md, "
                  "scripts/benchmark_dtypes.py (read as text)",
        "golden_payload_tables": golden,
        "known_answers": known_answers(),
    }
    args.out.write_text(json.dumps(doc, indent=1) + "\n")
    print(f"wrote {args.out}")


if __name__ == "__main__":
    main()
