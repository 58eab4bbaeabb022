"""The kernels' expf (sardyne_b200/csrc/expf_ref.h) is the reference host's: the same float as
libm's expf, which the reference's softmax and SiLU call (reference csrc/ops.c:353-371), for every
one of the 2^32 inputs. The header is compiled for the host with the same operation order the
device code uses (fused multiply-adds exactly where the device's __fma_rn stand) and compared with
the host's expf exhaustively (multi-threaded, about a minute of CPU time)."""
import os
import pathlib
import shutil
import subprocess

import pytest

REPO = pathlib.Path(__file__).resolve().parent.parent

CHECK = r"""
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>
#include "expf_ref.h"
int main(void) {
    long long bad = 0, n = 0;
    #pragma omp parallel for reduction(+:bad, n) schedule(static)
    for (long long u = 0; u < (1ll << 32); u++) {
        const uint32_t b = (uint32_t)u;
        float x;
        memcpy(&x, &b, 4);
        if (isnan(x)) continue;
        const float a = sdy::expf_ref(x), r = expf(x);
        uint32_t ua, ur;
        memcpy(&ua, &a, 4);
        memcpy(&ur, &r, 4);
        n++;
        if (ua != ur) bad++;
    }
    printf("%lld %lld\n", n, bad);
    return 0;
}
"""


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_expf_ref_equals_host_expf_on_every_input(tmp_path):
    src = tmp_path / "check.cpp"
    src.write_text(CHECK)
    exe = tmp_path / "check"
    subprocess.run(["g++", "-O2", "-fopenmp", "-ffp-contract=off", "-std=c++17",
                    "-I", str(REPO / "sardyne_b200" / "csrc"), str(src), "-o", str(exe), "-lm"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True,
                         env=dict(os.environ, OMP_NUM_THREADS=str(os.cpu_count() or 1)), timeout=900)
    n, bad = map(int, out.stdout.split())
    assert n == (1 << 32) - (1 << 24) + 2  # every non-NaN float
    assert bad == 0
