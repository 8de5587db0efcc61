"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run in a container that has the reference checked out (read-only is fine):

    python tests/golden/make_golden.py /path/to/CliffordCUDA

It imports the reference's CPU code -- ``_shared/_einsum_refs.py`` (the
reference's own einsum oracle, _einsum_refs.py:26-124) and
``cliffordcuda.extensions.ga.geom_prod._build_sign_value_table``
(geom_prod.py:44-74) and ``regressive_prod._build_regressive_sigma``
(regressive_prod.py:77-121) -- and records, for seeded inputs:

* products.npz   forward and both gradients (autograd in float64 through the
                 reference einsum) for every product and the signature spread
                 of the reference's tests (tests/_gradcheck.py:9-19,
                 tests/correctness/test_pqr.py:149-170);
* config1.npz    BASELINE config 1 (Cl(5,0), batch 4096, upstream grad = ones):
                 the first 64 rows exactly plus per-array sums and norms;
* sigma.npz      sha256 of the reference's sign tables (and of the direct
                 regressive table) for every algebra used by the configs;
* rotor.npz      y = R~ x R with R = exp(sum beta_ij e_i e_j) computed by the
                 reference's EinsumGP with the Euclidean metric (the reference
                 test's own witness construction, test_rotor_apply.py:37-92).

Inputs are float32 draws from numpy's default_rng(seed) so the tests can
also regenerate them. Nothing on the GPU box reads the reference: only these
committed fixtures travel.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

sys.dont_write_bytecode = True
OUT = os.path.dirname(os.path.abspath(__file__))


def signatures():
    sigs = []
    for n in (5, 7):
        sigs += [tuple([1] * n), tuple([-1] * n), tuple([1] * (n - 1) + [-1]),
                 tuple([1] * (n // 2) + [-1] * (n - n // 2)),
                 tuple([1] * (n - 1) + [0]), tuple([1] * (n - 2) + [-1, 0])]
    sigs += [(1, 1, 1, 1, 1, 0), (1, 1, 1, -1, -1, 0),
             (1, 1, 1, 1, 1, 1, -1),
             (1, 1, 1, 1, 1, 1, 1, -1), (1, 1, 1, 1, -1, -1, -1, 0),
             (1,) * 8,
             (1, 1, 1, 1, 1, 1, 1, 1, -1), (1, 1, 1, 1, 1, -1, -1, -1, 0)]
    out = []
    for s in sigs:
        if s not in out:
            out.append(s)
    return out


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
    from cliffordcuda.extensions.ga.geom_prod import _build_sign_value_table
    from cliffordcuda.extensions.ga.regressive_prod import _build_regressive_sigma

    classes = {"gp": EinsumGP, "wedge": EinsumWedge, "inner": EinsumInner,
               "lc": EinsumLeftContract, "rc": EinsumRightContract,
               "reg": EinsumRegressive}

    def fwd_bwd(op, n, metric, a, b, g):
        f = classes[op](n, metric=list(metric), device="cpu", dtype=torch.float64)
        at = torch.tensor(a, dtype=torch.float64, requires_grad=True)
        bt = torch.tensor(b, dtype=torch.float64, requires_grad=True)
        c = f(at, bt)
        (c * torch.tensor(g, dtype=torch.float64)).sum().backward()
        return c.detach().numpy(), at.grad.numpy(), bt.grad.numpy()

    rec = {}
    case = 0
    for metric in signatures():
        n = len(metric)
        ops = ["gp", "wedge", "inner", "lc", "rc"]
        if 0 not in metric:
            ops.append("reg")
        if n == 9:
            ops = ["gp", "wedge", "lc"]
        for op in ops:
            seed = 1000 + case
            case += 1
            a, b, g = inputs(n, seed, 2)
            c, ga, gb = fwd_bwd(op, n, metric, a, b, g)
            key = f"{op}|{','.join(map(str, metric))}"
            rec[key + "|seed"] = np.array(seed)
            rec[key + "|a"], rec[key + "|b"], rec[key + "|g"] = a, b, g
            rec[key + "|c"], rec[key + "|ga"], rec[key + "|gb"] = c, ga, gb
    np.savez_compressed(os.path.join(OUT, "products.npz"), **rec)

    n, metric = 5, (1,) * 5
    a, b, _ = inputs(n, 0, 4096)
    g = np.ones_like(a)
    c, ga, gb = fwd_bwd("gp", n, metric, a, b, g)
    np.savez_compressed(
        os.path.join(OUT, "config1.npz"), seed=np.array(0),
        c_head=c[:64], ga_head=ga[:64], gb_head=gb[:64],
        sums=np.array([c.sum(), ga.sum(), gb.sum()]),
        norms=np.array([np.linalg.norm(c), np.linalg.norm(ga), np.linalg.norm(gb)]))

    sig = {}
    for metric in signatures() + [(1,) * 6 + (-1,), (1,) * 7 + (-1,),
                                  (1,) * 9 + (0,), (1,) * 10]:
        n = len(metric)
        key = ",".join(map(str, metric))
        t = _build_sign_value_table(n, metric).numpy().astype(np.int8)
        sig["gp|" + key] = np.frombuffer(hashlib.sha256(t.tobytes()).digest(), np.uint8)
        if 0 not in metric:
            r = _build_regressive_sigma(n, metric).numpy().astype(np.int8)
            sig["regsigma|" + key] = np.frombuffer(
                hashlib.sha256(r.tobytes()).digest(), np.uint8)
    np.savez_compressed(os.path.join(OUT, "sigma.npz"), **sig)

    rot = {}
    for n in (7, 8):
        rng = np.random.default_rng(77 + n)
        nb = n * (n - 1) // 2
        beta = (0.1 * rng.standard_normal(nb)).astype(np.float32)
        x = rng.standard_normal((2, 1 << n)).astype(np.float32)
        gp = EinsumGP(n, metric=[1] * n, device="cpu", dtype=torch.float64)
        D = 1 << n
        Bv = torch.zeros(1, D, dtype=torch.float64)
        idx = 0
        for p in range(n - 1):
            for q in range(p + 1, n):
                Bv[0, (1 << p) | (1 << q)] = float(beta[idx])
                idx += 1
        s = 6
        Bs = Bv / (2 ** s)
        R = torch.zeros(1, D, dtype=torch.float64)
        R[0, 0] = 1.0
        term = R.clone()
        for m in range(1, 30):
            term = gp(term, Bs) / m
            R = R + term
        for _ in range(s):
            R = gp(R, R)
        k = torch.tensor([bin(i).count("1") for i in range(D)])
        rev = torch.where(((k * (k - 1) // 2) % 2) == 1, -1.0, 1.0).double()
        xt = torch.tensor(x, dtype=torch.float64)
        y = gp(gp(R * rev, xt), R)
        rot[f"{n}|beta"], rot[f"{n}|x"], rot[f"{n}|y"] = beta, x, y.numpy()
    np.savez_compressed(os.path.join(OUT, "rotor.npz"), **rot)
    print("wrote", sorted(os.listdir(OUT)))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "../CliffordCUDA")
