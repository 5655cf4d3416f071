"""Export the reference's SM83 opcode table to ``isa_sm83.json``.

TEST INFRASTRUCTURE. Run where the reference tree is available:

    python tests/golden/make_isa_fixture.py --reference <path-to-gbxcule>

It imports ``src/gbxcule/core/isa_sm83.py`` (standard library only) and writes,
per unprefixed and CB-prefixed opcode, the mnemonic, instruction length,
cycle counts (taken, not taken for conditionals), group and whether the
reference implements it. ``tests/isa_probe.py`` derives each probe's expected
next PC and cycles from this file.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    args = ap.parse_args()
    src = args.reference / "src" / "gbxcule" / "core" / "isa_sm83.py"
    spec = importlib.util.spec_from_file_location("isa_sm83", src)
    isa = importlib.util.module_from_spec(spec)
    sys.modules["isa_sm83"] = isa  # dataclasses look their module up while the class is built
    spec.loader.exec_module(isa)

    def rows(specs):
        return [{"opcode": s.opcode, "mnemonic": s.mnemonic, "length": s.length, "cycles": list(s.cycles),
                 "group": s.group, "implemented": s.implemented} for s in specs]

    out = {"about": "SM83 opcode table of the reference (src/gbxcule/core/isa_sm83.py iter_unprefixed / "
                    "iter_cb), exported by tests/golden/make_isa_fixture.py",
           "unprefixed": rows(isa.iter_unprefixed()), "cb": rows(isa.iter_cb())}
    (HERE / "isa_sm83.json").write_text(json.dumps(out, indent=0) + "\n")


if __name__ == "__main__":
    main()
