"""Fit the cubic used by the attention softmax to compute 2^f on the FMA
pipe (f in [-0.5, 0.5], after rounding the exponent argument to the nearest
integer): minimax relative error by iteratively reweighted least squares on
a dense grid. Run: python wam-egale_b200/csrc/exp2_fit.py
The coefficients are pasted into attention.cuh (ATT_EXP2_C0..C3)."""
import numpy as np

f = np.linspace(-0.5, 0.5, 20001)
y = np.exp2(f)
w = np.ones_like(f)
A = np.vander(f, 4, increasing=True)
for _ in range(200):
    c, *_ = np.linalg.lstsq(A * (w / y)[:, None], w, rcond=None)
    err = np.abs(A @ c / y - 1)
    w = w * (1 + 4 * err / err.max())
    w /= w.mean()
c32 = c.astype(np.float32)
err32 = np.abs((A @ c32.astype(np.float64)) / y - 1)
print("coefficients c0..c3:", [float(v) for v in c32])
print("max relative error (fp32 coefficients): %.3e" % err32.max())
