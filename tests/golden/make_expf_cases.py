"""Generates tests/golden/expf_cases.npy: float32 inputs x at which the host C library's expf(-x)
(what the reference's silu calls, ops.cpp:733-772) differs from the correctly rounded exp(-x) AND the
difference changes silu(x) = x / (1 + expf(-x)) in fp32, plus inputs where it changes the softmax
term expf(x) alone (x <= 0). A device exp that is not glibc's expf fails the parity test on these
inputs; one that is passes. The search runs over every float in [-88, 104] with a small C program
built here (gcc, the host's libm).

Usage: python tests/golden/make_expf_cases.py
"""
import os
import subprocess
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = r'''
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
int main(void) {
    FILE* f = fopen(getenv("OUT"), "wb");
    long n_silu = 0, n_exp = 0;
    for (uint64_t u = 0; u < (1ull << 32); u++) {
        float x; uint32_t b = (uint32_t)u; memcpy(&x, &b, 4);
        if (!(x >= -88.0f && x <= 104.0f)) continue;
        const float e = expf(-x), c = (float)exp(-(double)x);
        if (e == c) continue;
        const float d1 = 1.0f + e, d2 = 1.0f + c;
        const int silu_diff = x / d1 != x / d2;
        const int exp_term = x <= 0.0f;  /* softmax arguments x - max are <= 0 */
        if ((silu_diff && n_silu < 3000) || (exp_term && (u % 97) == 0 && n_exp < 1000)) {
            fwrite(&x, 4, 1, f);
            n_silu += silu_diff; n_exp += exp_term && !silu_diff;
        }
    }
    fclose(f);
    printf("%ld silu cases, %ld exp cases\n", n_silu, n_exp);
    return 0;
}
'''


def main():
    with tempfile.TemporaryDirectory() as d:
        c, exe, out = os.path.join(d, "s.c"), os.path.join(d, "s"), os.path.join(d, "x.bin")
        open(c, "w").write(SRC)
        subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-o", exe, c, "-lm"], check=True)
        subprocess.run([exe], check=True, env=dict(os.environ, OUT=out))
        x = np.fromfile(out, np.float32)
    np.save(os.path.join(HERE, "expf_cases.npy"), x)
    print(x.size, "inputs")


if __name__ == "__main__":
    main()
