"""Coefficients of the cubic behind exp2_fma2 (common.cuh).

Minimax-relative-error fit of 2^f on [0, 1) by p(f) = 1 + f*(c1 + f*(c2 + f*c3)), found with
Lawson's iteratively reweighted least squares; prints the fp32 coefficients and the maximum
relative error of the fp32 evaluation. Run: python fit_exp2.py
"""
import numpy as np
f = np.linspace(0, 1, 20001)[1:]
y = np.exp2(f)
A = np.stack([f, f**2, f**3], 1) / y[:, None]
b = (y - 1) / y
w = np.ones_like(f)
for _ in range(2000):
    sw = np.sqrt(w)
    c, *_ = np.linalg.lstsq(A * sw[:, None], b * sw, rcond=None)
    e = np.abs(A @ c - b)
    w = w * e; w /= w.sum()
c32 = c.astype(np.float32)
def p(ff):
    ff = ff.astype(np.float32)
    return np.float32(1) + ff * (c32[0] + ff * (c32[1] + ff * c32[2]))
ff = np.linspace(0, 1, 200001, dtype=np.float32)
rel = np.abs(p(ff).astype(np.float64) / np.exp2(ff.astype(np.float64)) - 1)
print("coeffs", [float(x) for x in c32], [x.view(np.uint32) for x in c32]); print("max rel err", rel.max())
