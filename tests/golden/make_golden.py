"""Regenerate the golden fixtures in tests/golden/.

Run in a container where the reference checkout is mounted; its path is the
first argument.  The fixtures it writes are committed; tests never read the
reference at run time.

1. ``prime_chain_n17_d44_s59_f60_dnum4.json`` — the 45 Q + 12 P primes that
   the reference recorded from OpenFHE v1.4.2 / FIDESlib for
   N=2^17, depth 44, scaling 59, first 60, FLEXIBLEAUTO, HYBRID dnum 4
   (reference: results/b300/2026-09-28/long-accuracy/oracle-p-r3-base/native.json:1,
   written by experiments/ntt_warp_tail/probe.cu:207-219).
2. ``ntt_kat_n1024.npz`` — known-answer forward NTT vectors computed by the
   O(N^2) definition out[i] = sum_j a[j] psi^{(2 brv(i) + 1) j} mod q with
   pure Python integers (independent of the C oracle and of the CUDA code).
   Inputs follow the reference probe's patterns (probe.cu:41-56): q-1,
   alternating 0/q-1, and splitmix64-mixed values.  Primes: q_0, q_44 and p_0
   of the recorded chain (all are 1 mod 2^18, hence valid for N = 1024).
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
MASK = (1 << 64) - 1


def mix(x: int) -> int:  # probe.cu:41-46 (splitmix64 finaliser)
    x = (x + 0x9E3779B97F4A7C15) & MASK
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & MASK
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & MASK
    return x ^ (x >> 31)


def values(n: int, q: int, pattern: int, salt: int) -> list[int]:  # probe.cu:47-56
    if pattern == 0:
        return [0] * n
    if pattern == 1:
        return [q - 1] * n
    if pattern == 2:
        return [q - 1 if i % 2 else 0 for i in range(n)]
    return [mix(salt * n + i) % q for i in range(n)]


def min_root(m: int, q: int) -> int:
    x = 2
    while True:
        g = pow(x, (q - 1) // m, q)
        if pow(g, m // 2, q) == q - 1:
            break
        x += 1
    return min(pow(g, k, q) for k in range(1, m, 2))


def brv(i: int, bits: int) -> int:
    return int(format(i, f"0{bits}b")[::-1], 2)


def ntt_definition(a: list[int], q: int, psi: int) -> list[int]:
    n = len(a)
    bits = n.bit_length() - 1
    out = []
    for i in range(n):
        e = 2 * brv(i, bits) + 1
        w = pow(psi, e, q)
        acc, p = 0, 1
        for j in range(n):
            acc += a[j] * p
            p = p * w % q
        out.append(acc % q)
    return out


def main(ref: str) -> None:
    src = os.path.join(ref, "results/b300/2026-09-28/long-accuracy/oracle-p-r3-base/native.json")
    d = json.load(open(src))
    primes = d["all_primes"]
    chain = {
        "source": "results/b300/2026-09-28/long-accuracy/oracle-p-r3-base/native.json:1",
        "ring_dim": d["ring"], "log_n": 17, "mult_depth": 44, "scaling_mod_size": 59,
        "first_mod_size": 60, "num_large_digits": d["digits"],
        "q": primes[:45], "p": primes[45:],
    }
    with open(os.path.join(HERE, "prime_chain_n17_d44_s59_f60_dnum4.json"), "w") as f:
        json.dump(chain, f, indent=1)

    n = 1024
    sel = [primes[0], primes[44], primes[45]]
    ins, outs, qs, psis, pats = [], [], [], [], []
    for qi, q in enumerate(sel):
        psi = min_root(2 * n, q)
        for pat in (1, 2, 3):
            a = values(n, q, pat, 10 + qi)
            ins.append(a)
            outs.append(ntt_definition(a, q, psi))
            qs.append(q)
            psis.append(psi)
            pats.append(pat)
    np.savez(os.path.join(HERE, "ntt_kat_n1024.npz"),
             inputs=np.array(ins, dtype=np.uint64), outputs=np.array(outs, dtype=np.uint64),
             primes=np.array(qs, dtype=np.uint64), psi=np.array(psis, dtype=np.uint64),
             patterns=np.array(pats, dtype=np.int64))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py REFERENCE_CHECKOUT")
    main(sys.argv[1])
