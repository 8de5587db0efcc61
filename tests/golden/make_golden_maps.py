"""Generate tests/golden/maps.npz -- fixtures for the per-blade maps
(reverse, grade involution, Clifford conjugation, grade projection, dual)
and norm_sq -- from the reference itself.

Run in a container that has the reference checked out (read-only is fine):

    python tests/golden/make_golden_maps.py /path/to/CliffordCUDA

It runs the reference's own CliffordAlgebra methods (src/cliffordcuda/
algebra.py:195-336) and its free function reverse (extensions/ga/
inverse.py:64-67) on the CPU, on seeded float32 inputs (numpy default_rng).
The reference is CUDA-only at its boundary, so the script builds the algebra
objects without their constructor (no rotor tables are needed here) and
turns off the device checks of its _validate module; the methods' own sign
construction is what runs.
"""
from __future__ import annotations

import os
import sys

import numpy as np

sys.dont_write_bytecode = True
OUT = os.path.dirname(os.path.abspath(__file__))

METRICS = [
    (1, 1, 1), (1, -1, 0), (1, 1, 1, 1, 1), (-1,) * 5, (1, 1, 1, -1, 0),
    (1,) * 6 + (-1,), (1, -1) * 4, (1,) * 7 + (0,), (1,) * 9 + (0,),
    (1,) * 5 + (-1,) * 5, (-1,) * 10,
]


def main(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "src"))
    import torch
    import cliffordcuda._validate as V
    from cliffordcuda.algebra import CliffordAlgebra
    from cliffordcuda.extensions.ga import inverse as inv

    V._check_mv = lambda *a, **k: None
    rec = {}
    for idx, metric in enumerate(METRICS):
        n = len(metric)
        cl = object.__new__(CliffordAlgebra)
        cl.metric, cl.n, cl.dim = tuple(metric), n, 1 << n
        cl.device, cl.dtype = torch.device("cpu"), torch.float32
        rng = np.random.default_rng(7000 + idx)
        x = rng.standard_normal((3, 1 << n)).astype(np.float32)
        xt = torch.tensor(x)
        key = ",".join(map(str, metric))
        rec[key + "|x"] = x
        rec[key + "|reverse"] = cl.reverse(xt).numpy()
        rec[key + "|involute"] = cl.grade_involution(xt).numpy()
        rec[key + "|conjugate"] = cl.clifford_conjugation(xt).numpy()
        rec[key + "|grade"] = np.stack([cl.grade_projection(xt, k).numpy()
                                        for k in range(n + 1)])
        rec[key + "|norm_sq"] = cl.norm_sq(xt).numpy()
        if 0 not in metric:
            rec[key + "|dual"] = cl.dual(xt).numpy()
        rec[key + "|free_reverse"] = inv.reverse(xt).numpy()
    np.savez_compressed(os.path.join(OUT, "maps.npz"), **rec)
    print("wrote maps.npz", len(rec))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "../CliffordCUDA")
