"""Derives the integer constant the softcap kernel uses for its reciprocal seed on the FMA pipe
(fa_sm100.cuh, MFA_SOFTCAP_TANH = 0 with MFA_RCP_EMU > 0).

Method: the bit pattern of 1/d is approximated by M - bits(d) (a float's bits are close to a
scaled, offset log2 of its value, so subtracting them negates the exponent); the guess is
refined by Newton steps r += r(1 - d r), each of which squares the relative error. The seed M
is chosen to minimise the maximum relative error |guess * d - 1| over one binade of d (the error
pattern repeats every binade), by a coarse scan followed by an exhaustive local search. Run it
to print the constant and its error bound:

    python mtlflashattn_b200/csrc/fit_rcp_seed.py
"""
import numpy as np


def max_rel_err(M, d_bits):
    g = (np.uint32(M) - d_bits).view(np.float32).astype(np.float64)
    d = d_bits.view(np.float32).astype(np.float64)
    return np.max(np.abs(g * d - 1.0))


def fit():
    # every float in [1, 2) with the low 7 mantissa bits dropped (65536 points), plus the binade
    # end points
    d_bits = (np.uint32(0x3F800000) + (np.arange(1 << 16, dtype=np.uint32) << np.uint32(7)))
    best = None
    for M in range(0x7EE00000, 0x7F000000, 1 << 12):  # coarse
        e = max_rel_err(M, d_bits)
        if best is None or e < best[1]:
            best = (M, e)
    lo, hi = best[0] - (1 << 12), best[0] + (1 << 12)
    for step in (1 << 8, 1 << 4, 1):  # refine around the best point
        for M in range(lo, hi, step):
            e = max_rel_err(M, d_bits)
            if e < best[1]:
                best = (M, e)
        lo, hi = best[0] - step, best[0] + step
    return best


if __name__ == "__main__":
    M, e = fit()
    print(f"seed constant 0x{M:08X}: max relative error of the guess {e:.4f} "
          f"(after 3 Newton steps <= {e ** 8:.2e})")
