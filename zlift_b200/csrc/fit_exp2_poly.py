"""Derives the coefficients of fmha.cu's ex2_poly: the degree-3 polynomial
of least maximum relative error to 2^f on [-1/2, 1/2], found with the
Remez exchange algorithm (equioscillation of the relative error at deg+2
points).  Run: python fit_exp2_poly.py  (prints the coefficients and the
error of the float32 Horner evaluation the kernel uses)."""
import numpy as np
deg = 3
a, b = -0.5, 0.5
f = lambda x: np.exp2(x)
# initial reference: Chebyshev extrema
n = deg + 2
x = 0.5 * (a + b) + 0.5 * (b - a) * np.cos(np.pi * np.arange(n)[::-1] / (n - 1))
for it in range(30):
    # solve p(x_i) - f(x_i) = (-1)^i E f(x_i)   (relative error equioscillation)
    A = np.zeros((n, n))
    for i in range(n):
        A[i, :deg + 1] = x[i] ** np.arange(deg + 1)
        A[i, deg + 1] = -((-1) ** i) * f(x[i])
    sol = np.linalg.solve(A, f(x))
    c, E = sol[:deg + 1], sol[deg + 1]
    grid = np.linspace(a, b, 200001)
    err = (np.polyval(c[::-1], grid) - f(grid)) / f(grid)
    # new reference: local extrema of err, one per sign run
    idx = [0]
    s = np.sign(err)
    for i in range(1, len(grid)):
        if s[i] != s[idx[-1]]:
            idx.append(i)
        elif abs(err[i]) > abs(err[idx[-1]]):
            idx[-1] = i
    if len(idx) < n:
        break
    # keep n extrema with largest |err| contiguous
    idx = np.array(idx)
    while len(idx) > n:
        if abs(err[idx[0]]) < abs(err[idx[-1]]):
            idx = idx[1:]
        else:
            idx = idx[:-1]
    x = grid[idx]
print("coeffs c0..c3:", [float(np.float32(v)) for v in c])
print("max rel err:", np.max(np.abs(err)))
# check in float32 arithmetic with Horner
g = np.linspace(-0.5, 0.5, 100001).astype(np.float32)
c32 = np.float32(c)
p = ((c32[3] * g + c32[2]) * g + c32[1]) * g + c32[0]
print("f32 Horner max rel err:", np.max(np.abs(p.astype(np.float64) / np.exp2(g.astype(np.float64)) - 1)))
for v in c32: print(float(v).hex(), repr(float(v)))
