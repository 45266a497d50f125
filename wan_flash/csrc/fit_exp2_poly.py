"""Fit the polynomial used by ``exp2_poly2`` in wf_common.cuh.

Method: Cody-Waite style range reduction x = j + f with j = rint(x) and
f in [-1/2, 1/2]; 2^x = 2^j * p(f), where p is the degree-4 polynomial that
minimises the maximum RELATIVE error of p(f) / 2^f - 1 on [-1/2, 1/2],
found with the Remez exchange algorithm in double precision.  The script
prints the coefficients (rounded to fp32, as compiled into the kernels) and
the max relative error of a float32 Horner evaluation.

    python wan_flash/csrc/fit_exp2_poly.py
"""

import numpy as np


def remez_exp2(deg, a=-0.5, b=0.5, iters=30):
    n = deg + 2
    k = np.arange(n)
    x = (a + b) / 2 + (b - a) / 2 * np.cos(np.pi * k[::-1] / (n - 1))
    xs = np.linspace(a, b, 200001)
    for _ in range(iters):
        A = np.zeros((n, n))
        for i in range(n):
            A[i, : deg + 1] = x[i] ** np.arange(deg + 1)
            A[i, deg + 1] = -((-1) ** i) * np.exp2(x[i])
        c = np.linalg.solve(A, np.exp2(x))[: deg + 1]
        err = np.polyval(c[::-1], xs) / np.exp2(xs) - 1.0
        sgn = np.sign(err)
        ext, start = [], 0
        for i in range(1, len(xs)):
            if sgn[i] != sgn[i - 1]:
                ext.append(start + int(np.argmax(np.abs(err[start:i]))))
                start = i
        ext.append(start + int(np.argmax(np.abs(err[start:]))))
        if len(ext) >= n:
            best = max(range(len(ext) - n + 1), key=lambda s: min(abs(err[ext[s : s + n]])))
            x = xs[ext[best : best + n]]
    return c


def horner_f32(c32, f):
    p = np.full_like(f, c32[-1])
    for cc in c32[-2::-1]:
        p = (p * f + cc).astype(np.float32)
    return p


if __name__ == "__main__":
    c32 = remez_exp2(4).astype(np.float32)
    f = np.linspace(-0.5, 0.5, 100001).astype(np.float32)
    err = np.max(np.abs(horner_f32(c32, f).astype(np.float64) / np.exp2(f.astype(np.float64)) - 1.0))
    print("coefficients c0..c4:", ", ".join("%.9ef" % v for v in c32))
    print("max relative error (fp32 Horner):", err)
