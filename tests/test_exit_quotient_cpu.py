"""The grid kernel's exit quotient, restated in C with the C library's fmaf, against the
IEEE float division of the host (no GPU): RN(q0 + RN(a - q0 * d) * r) with r = RN(1 / d)
and q0 = RN(a * r) equals RN(a / d), on random pairs and on significands at the ends of
their binades (the reciprocal's and the quotient's worst rounding).  The device form is
tsdf::exit_quotient in navi_b200/csrc/exit_quotient.cuh; the GPU tests check it against
__fdiv_rn exhaustively over significand pairs."""

from __future__ import annotations

import shutil
import subprocess

import pytest

SRC = r"""
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
static uint64_t s = 0x9E3779B97F4A7C15ull;
static uint64_t next(void) { s ^= s << 13; s ^= s >> 7; s ^= s << 17; return s; }
static float f(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }
static uint32_t u(float x) { uint32_t v; memcpy(&v, &x, 4); return v; }
int main(int argc, char** argv) {
    long n = atol(argv[1]), bad = 0, tested = 0;
    for (long i = 0; i < n; ++i) {
        uint32_t ma = (uint32_t)next() & 0x7FFFFF, md = (uint32_t)next() & 0x7FFFFF;
        int mode = (int)(i % 4);
        if (mode == 1) { ma |= 0x7FF000; md |= 0x7FF000; }        /* both near 2 */
        if (mode == 2) { ma |= 0x7FF000; md &= 0xFFF; }           /* a near 2, d near 1 */
        if (mode == 3) { ma &= 0xFFF; md |= 0x7FF000; }           /* a near 1, d near 2 */
        uint32_t ea = 90 + (uint32_t)(next() % 70), ed = 114 + (uint32_t)(next() % 24);
        float a = f(ma | (ea << 23) | ((uint32_t)next() & 0x80000000u));
        float d = f(md | (ed << 23) | ((uint32_t)next() & 0x80000000u));
        if (!(fabsf(d) > 1e-4f)) continue;
        volatile float r = 1.0f / d;
        volatile float q0 = a * r;
        float t = fmaf(fmaf(-q0, d, a), r, q0);
        volatile float q = a / d;
        ++tested;
        if (u(t) != u(q)) { if (bad < 3) printf("a=%a d=%a q=%a t=%a\n", a, d, q, t); ++bad; }
    }
    printf("%ld %ld\n", tested, bad);
    return bad != 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_exit_quotient_identity_on_the_host(tmp_path):
    c = tmp_path / "q.c"
    c.write_text(SRC)
    exe = tmp_path / "q"
    subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", str(c), "-o", str(exe), "-lm"], check=True)
    proc = subprocess.run([str(exe), "4000000"], capture_output=True, text=True, timeout=300)
    tested, bad = map(int, proc.stdout.split()[-2:])
    assert tested > 3_000_000
    assert proc.returncode == 0 and bad == 0, proc.stdout
