"""The prefill GEMM's shared-memory plan (csrc/gemm_plan.h), compiled on the host with g++: for every
token tile the kernel accepts (16..256 in steps of 16) and every raw chunk size (Q8_0 8,704 B, Q4_0
4,608 B, Q5_1 6,144 B, the affine layout 12,288 B) the raw-chunk ring is even or at least NS + 2
slots deep, so the two decoder groups' parity waits on it are exact; the plan fits the dynamic
shared memory of one CTA, and every ring slot sits where its copies and descriptors need it."""
from __future__ import annotations

import subprocess

from conftest import REPO

CHUNKS = {"Q8_0": 8704, "Q4_0": 4608, "Q5_1": 6144, "QX": 12288}
MAX_DYNAMIC_SMEM = 232448  # 227 KB per CTA on sm_100a

PROGRAM = r"""
#include <cstdio>
#include "gemm_plan.h"
int main() {
    const int chunks[] = {%s};
    for (int cb : chunks)
        for (int bn = 16; bn <= 256; bn += 16) {
            jv::GemmRingPlan p;
            const bool ok = jv::gemm_ring_plan(bn, cb, &p);
            std::printf("%%d %%d %%d %%d %%d %%d %%d %%d %%zu\n", cb, bn, ok ? 1 : 0, p.ns, p.nr, p.b_off, p.raw_off,
                        p.bar_off, p.smem);
        }
    return 0;
}
"""


def plans(tmp_path):
    src = tmp_path / "plan.cpp"
    src.write_text(PROGRAM % ", ".join(str(c) for c in CHUNKS.values()))
    exe = tmp_path / "plan"
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Werror", "-I", str(REPO / "llm-shield_b200" / "csrc"), str(src), "-o",
                    str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    rows = []
    for line in out.splitlines():
        cb, bn, ok, ns, nr, b_off, raw_off, bar_off, smem = (int(v) for v in line.split())
        rows.append(dict(cb=cb, bn=bn, ok=ok, ns=ns, nr=nr, b_off=b_off, raw_off=raw_off, bar_off=bar_off, smem=smem))
    assert len(rows) == 16 * len(CHUNKS)
    return rows


def test_every_raw_ring_keeps_the_decoder_parity_waits_exact(tmp_path):
    for p in plans(tmp_path):
        assert p["ok"], p
        assert p["ns"] in (3, 4), p
        assert p["nr"] >= 2, p
        assert p["nr"] % 2 == 0 or p["nr"] >= p["ns"] + 2, p


def test_the_plan_fits_one_cta_and_aligns_every_slot(tmp_path):
    for p in plans(tmp_path):
        bn, cb, ns, nr = p["bn"], p["cb"], p["ns"], p["nr"]
        assert p["smem"] <= MAX_DYNAMIC_SMEM, p
        # decoded-weight stages from 0, activation stages after them, then the raw ring, then the barriers
        assert p["b_off"] == 16384 * ns, p
        assert p["raw_off"] == p["b_off"] + bn * 128 * ns, p
        assert p["bar_off"] >= p["raw_off"] + cb * nr and p["bar_off"] % 16 == 0, p
        # SWIZZLE_128B operand tiles start on 1024-byte boundaries; bulk copies on 16-byte ones
        assert p["b_off"] % 1024 == 0 and (bn * 128) % 1024 == 0, p
        assert p["raw_off"] % 16 == 0 and cb % 16 == 0, p


def test_the_plans_that_had_an_odd_short_ring(tmp_path):
    """Q8_0 at a 224-token tile had 5 raw slots beside 4 stages (the parity waits could pass on the
    other group's chunk in flight); it now has 4. At 256 (C5's tile) 9 beside 3 stays: 9 >= 3 + 2."""
    got = {(p["cb"], p["bn"]): (p["ns"], p["nr"]) for p in plans(tmp_path)}
    assert got[(8704, 224)] == (4, 4)
    assert got[(8704, 256)] == (3, 9)
    assert got[(8704, 112)] == (4, 12)
