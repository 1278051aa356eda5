"""CPU proof for the detector normalisation's division (csrc/preprocess.cu,
normalize()): Markstein's correction step q' = fma(fma(-s, q, a), 1/s, q),
q = a * (1/s), equals the IEEE quotient a / s for each channel std s of the
detector (0.229, 0.224, 0.225) and EVERY float a with 2^-60 <= |a| <= 0.75 --
a superset of the numerators the kernel forms (0, or fma(v, 1/255, -mean)
with v in [0, 255], whose magnitude lies in [2^-49, 0.6]). Exhaustive over
~2.5e9 operands: a C program on all host cores."""

import os
import subprocess
import tempfile
from pathlib import Path

SRC = r"""
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>
int main(void) {
  const float ds[3] = {0.229f, 0.224f, 0.225f};
  long long bad = 0, n = 0;
  const uint32_t lo = (127u - 60u) << 23, hi = 0x3F400000u; /* 2^-60 .. 0.75 */
  for (int k = 0; k < 3; ++k) {
    volatile float dv = ds[k];
    const float d = dv, y = 1.0f / d;
#pragma omp parallel for reduction(+ : bad, n)
    for (long long u = lo; u <= hi; ++u) {
      for (int sgn = 0; sgn < 2; ++sgn) {
        uint32_t bits = (uint32_t)u | (sgn ? 0x80000000u : 0u);
        float a, q2, ref;
        memcpy(&a, &bits, 4);
        const float q = a * y;
        q2 = fmaf(fmaf(-d, q, a), y, q);
        ref = a / d;
        bad += memcmp(&q2, &ref, 4) != 0;
        ++n;
      }
    }
  }
  printf("%lld %lld\n", n, bad);
  return 0;
}
"""


def test_markstein_division_is_exact_for_detector_stds():
    with tempfile.TemporaryDirectory() as d:
        c, exe = Path(d) / "div.c", Path(d) / "div"
        c.write_text(SRC)
        subprocess.run(["gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-o", str(exe), str(c), "-lm"], check=True)
        out = subprocess.run([str(exe)], check=True, capture_output=True, text=True,
                             env={**os.environ, "OMP_NUM_THREADS": str(os.cpu_count() or 1)}).stdout.split()
    n, bad = int(out[0]), int(out[1])
    assert n == 3 * 2 * (0x3F400000 - ((127 - 60) << 23) + 1)
    assert bad == 0
