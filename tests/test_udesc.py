"""The uniform interpreter's descriptor table pinned to the reference's ISA table (CPU).

``gbxcule_b200/csrc/gbx_udesc.h`` builds one descriptor per opcode (and per
CB-prefixed opcode) at compile time; the step kernel takes each
instruction's length, its cycles taken / not taken and whether it traps from
it. Here the header is compiled for the host with g++ and every descriptor is
compared with ``src/gbxcule/core/isa_sm83.py``'s table (exported to
``golden/isa_sm83.json``): length, cycle counts (both for the conditional
jumps, calls and returns) and the unimplemented opcodes, which must be the
special (trapping) entries with zero cycles. The GPU runs the same decoder
on the every-opcode probe batch in ``test_gpu_isa.py``.
"""

from __future__ import annotations

import shutil
import subprocess

import pytest

from tests import isa_probe
from tests.conftest import REPO

PROGRAM = r"""
#define __host__
#define __device__
#include <stdio.h>
#include "gbx_udesc.h"
int main() {
  for (int k = 0; k < gbx::UDESC_KEYS; k++) {
    const gbx::UDesc d = gbx::make_udesc(k);
    const unsigned len = (d.q1x >> gbx::UV_LEN) & 3, nt = (d.q1x >> gbx::UV_CYC_NT) & 15;
    const unsigned t = (d.q1x >> gbx::UV_CYC_T) & 15;
    printf("%d %u %u %u %u %u\n", k, len, 4 * t, 4 * nt, (d.q0z & gbx::UF_SPECIAL) ? 1u : 0u,
           (d.q1y & 0xFF) ? 1u : 0u);
  }
  return 0;
}
"""


@pytest.fixture(scope="module")
def table(tmp_path_factory):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    d = tmp_path_factory.mktemp("udesc")
    (d / "dump.cpp").write_text(PROGRAM)
    exe = d / "dump"
    subprocess.run([gxx, "-std=c++17", "-O1", "-I", str(REPO / "gbxcule_b200" / "csrc"), str(d / "dump.cpp"),
                    "-o", str(exe)], check=True, capture_output=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    rows = {}
    for line in out:
        if line.strip():
            k, length, taken, not_taken, special, cond = map(int, line.split())
            rows[k] = dict(length=length, taken=taken, not_taken=not_taken, special=special, cond=cond)
    assert len(rows) == 512
    return rows


def test_unprefixed_descriptors_match_the_isa_table(table):
    bad = []
    for e in isa_probe.isa_table()["unprefixed"]:
        op = e["opcode"]
        if op == 0xCB:
            continue  # the prefix: its descriptors are keys 256..511
        d = table[op]
        if not e["implemented"]:
            if not (d["special"] and d["taken"] == 0 and d["not_taken"] == 0):
                bad.append(f"{op:#04x} {e['mnemonic']}: unimplemented but {d}")
            continue
        want = e["cycles"]
        got = [d["taken"], d["not_taken"]] if d["cond"] else [d["taken"]]
        if d["length"] != e["length"] or got != want or (not d["cond"] and d["taken"] != d["not_taken"]):
            bad.append(f"{op:#04x} {e['mnemonic']}: length {d['length']} cycles {got}, "
                       f"table {e['length']} {want}")
    assert not bad, "\n".join(bad)


def test_cb_descriptors_match_the_isa_table(table):
    bad = []
    for e in isa_probe.isa_table()["cb"]:
        d = table[256 + e["opcode"]]
        if (d["length"], [d["taken"]], d["cond"], d["special"]) != (e["length"], e["cycles"], 0, 0):
            bad.append(f"CB {e['opcode']:#04x} {e['mnemonic']}: {d}, table {e['length']} {e['cycles']}")
    assert not bad, "\n".join(bad)


def test_conditional_set_is_the_reference_set(table):
    cond = {k for k in range(256) if table[k]["cond"]}
    assert cond == isa_probe.CONDITIONAL
