"""Regenerates dequant_samples.json from the reference's dequant fixtures.

Source (read-only, only present where the reference is mounted):
crates/firepit/tests/modelopt_dequant_samples.txt and fp8_dequant_samples.txt
of almightychang/firepit.  Each line there is `<tensor> <row> <col> <f32 bits>`,
the f32 bit pattern that ModelOpt / Qwen's Python dequantizer produced for
one weight of a real checkpoint (the reference pins its loader against them,
crates/firepit/src/checkpoint.rs:349-429).  The checkpoints themselves are
not available, so the tests use these values for structural checks of the
decode tables (tests/test_oracle_pins.py).

Usage: python tests/golden/make_dequant_fixture.py <reference_root>
(reference_root: the root of an almightychang/firepit checkout)
"""
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def parse(path: Path):
    out = []
    for line in path.read_text().splitlines():
        parts = line.split()
        if len(parts) == 4:
            out.append({"tensor": parts[0], "row": int(parts[1]), "col": int(parts[2]), "bits": int(parts[3])})
    return out


def main(ref_root: str) -> None:
    tests = Path(ref_root) / "crates" / "firepit" / "tests"
    data = {
        "source": "almightychang/firepit crates/firepit/tests/{modelopt,fp8}_dequant_samples.txt",
        "nvfp4_or_fp8_modelopt": parse(tests / "modelopt_dequant_samples.txt"),
        "fp8_block": parse(tests / "fp8_dequant_samples.txt"),
    }
    (HERE / "dequant_samples.json").write_text(json.dumps(data, indent=1) + "\n")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_dequant_fixture.py <reference_root>")
    main(sys.argv[1])
