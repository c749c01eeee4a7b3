"""Fits the degree-3 polynomial for 2^f on [-0.5, 0.5] used by ex2_poly2 in
prefill_tc.cu: weighted least squares in relative error on Chebyshev nodes,
with Lawson reweighting toward the minimax solution.  Prints the float32
coefficients (constant term first) and their max relative error measured
with float32 Horner evaluation on a dense grid.
"""
import numpy as np


def fit(deg: int = 3, nodes: int = 2000, iters: int = 200):
    f = 0.5 * np.cos(np.pi * (np.arange(nodes) + 0.5) / nodes)
    y = np.exp2(f)
    a = np.vander(f, deg + 1, increasing=True) / y[:, None]
    b = np.ones(nodes)
    w = np.full(nodes, 1.0 / nodes)
    for _ in range(iters):
        sw = np.sqrt(w)
        c, *_ = np.linalg.lstsq(a * sw[:, None], b * sw, rcond=None)
        w = w * np.abs(a @ c - b)
        w /= w.sum()
    return c.astype(np.float32)


def max_rel_error(c32: np.ndarray) -> float:
    fd = np.linspace(-0.5, 0.5, 200001).astype(np.float32)
    p = np.full_like(fd, c32[-1])
    for k in range(len(c32) - 2, -1, -1):
        p = p * fd + c32[k]
    return float(np.abs(p.astype(np.float64) / np.exp2(fd.astype(np.float64)) - 1).max())


if __name__ == "__main__":
    c = fit()
    print([float(x) for x in c], f"max rel error {max_rel_error(c):.3e}")
