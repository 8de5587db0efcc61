"""Generate tests/golden/large_n.npz -- fixtures for the large-n regime
(n = 11..14) -- from the reference itself.

Run in a container that has the reference checked out (read-only is fine):

    python tests/golden/make_golden_large.py /path/to/CliffordCUDA

It imports the reference's CPU einsum oracle (``_shared/_einsum_refs.py``,
_einsum_refs.py:26-124, which builds its sign table with
``geom_prod._build_sign_value_table``, geom_prod.py:44-74) and records, for
seeded float32 inputs (numpy default_rng), the forward product and both
gradients (float64 autograd through the einsum, upstream gradient g).

The cases follow the reference's own large-n tests: the forced-tiling
signatures of tests/correctness/test_geom_prod_tiled.py:22-30 at n = 11, 12
and 13, the past-the-limit signatures at n = 14 (:47-51, :134-138), and the
other products at n = 11 (tests/correctness/test_products_tiled.py:40-60).
The einsum materialises (batch, 2^n, 2^n) arrays, so the batch is 2 up to
n = 12 and 1 above (n = 14 needs about 16 GB of host memory).
"""
from __future__ import annotations

import os
import sys

import numpy as np

sys.dont_write_bytecode = True
OUT = os.path.dirname(os.path.abspath(__file__))

CASES = [
    # (op, metric, batch)
    ("gp", (1,) * 11, 2),
    ("gp", (1,) * 6 + (-1,) * 5, 2),
    ("wedge", (1, -1, 1, -1) * 2 + (1, -1, 1), 2),
    ("inner", (1, 1, 1, -1, -1, 0) + (1, 1, 1, -1, -1), 2),
    ("lc", (1,) * 11, 2),
    ("rc", (1,) * 9 + (-1, 0), 2),
    ("reg", (1,) * 9 + (-1, -1), 2),
    ("gp", (1, 1, -1, -1, 1, -1, 0, 0, 1, 1, -1, 0), 2),
    ("lc", (1,) * 10 + (-1, 0), 2),
    ("gp", (1,) * 13, 1),
    ("gp", (1,) * 11 + (-1, -1, 0), 1),
]


def inputs(n, seed, batch):
    rng = np.random.default_rng(seed)
    D = 1 << n
    return [rng.standard_normal((batch, D)).astype(np.float32) for _ in range(3)]


def main(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "src"))
    sys.path.insert(0, os.path.join(ref_root, "_shared"))
    import torch
    from _einsum_refs import (EinsumGP, EinsumWedge, EinsumInner,
                              EinsumLeftContract, EinsumRightContract,
                              EinsumRegressive)

    classes = {"gp": EinsumGP, "wedge": EinsumWedge, "inner": EinsumInner,
               "lc": EinsumLeftContract, "rc": EinsumRightContract,
               "reg": EinsumRegressive}
    rec = {}
    for idx, (op, metric, batch) in enumerate(CASES):
        n = len(metric)
        seed = 5000 + idx
        a, b, g = inputs(n, seed, batch)
        f = classes[op](n, metric=list(metric), device="cpu", dtype=torch.float64)
        at = torch.tensor(a, dtype=torch.float64, requires_grad=True)
        bt = torch.tensor(b, dtype=torch.float64, requires_grad=True)
        c = f(at, bt)
        (c * torch.tensor(g, dtype=torch.float64)).sum().backward()
        key = f"{op}|{','.join(map(str, metric))}"
        rec[key + "|seed"] = np.array(seed)
        rec[key + "|a"], rec[key + "|b"], rec[key + "|g"] = a, b, g
        rec[key + "|c"] = c.detach().numpy()
        rec[key + "|ga"], rec[key + "|gb"] = at.grad.numpy(), bt.grad.numpy()
        del f, c, at, bt
        print("done", key, flush=True)
    np.savez_compressed(os.path.join(OUT, "large_n.npz"), **rec)
    print("wrote large_n.npz")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "../CliffordCUDA")
