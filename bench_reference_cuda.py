"""Side-by-side: the reference's own CUDA kernels on the same B200.

Runs vsingh-group/CliffordCUDA unmodified (installed with
`pip install --no-deps --target baseline/_ref <reference>`, its torch
extensions JIT-built for sm_100 into baseline/_ref_build) through its public
API at this repository's bench workloads, times it with the same CUDA-event
method as bench.py, and checks that its results agree with this library's on
a row subset (relative L2). One JSON line per workload. This is a
measurement aid beside bench.py, not part of the product.

    python bench_reference_cuda.py [--workload headline|products|layer|rotor|pga|all]
                                   [--out FILE]
"""
from __future__ import annotations

import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(ROOT, "baseline", "_ref")
BUILD = os.path.join(ROOT, "baseline", "_ref_build")
sys.dont_write_bytecode = True


def prepare_reference_env():
    """Point the reference's torch JIT at baseline/_ref_build for sm_100. When
    its extensions were built there already (they travel with the tree), mark
    the build outputs newer than their sources so that ninja reuses them
    instead of rebuilding them (a copied tree need not keep modification
    times in order)."""
    os.environ["XDG_CACHE_HOME"] = BUILD
    os.environ["TORCH_EXTENSIONS_DIR"] = os.path.join(BUILD, "cliffordcuda", "torch_extensions")
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    ext = os.environ["TORCH_EXTENSIONS_DIR"]
    if os.path.isdir(ext):
        import time
        now = time.time()
        for d, _, files in os.walk(ext):
            for f in files:
                if f == "lock":
                    os.remove(os.path.join(d, f))
                else:
                    os.utime(os.path.join(d, f), (now, now))


# The reference's own extension loaders (each wraps torch.utils.cpp_extension.load).
_LOADERS = [
    ("cliffordcuda.extensions.ga.geom_prod", "load_geom_prod_cuda"),
    ("cliffordcuda.extensions.ga.geom_prod_tiled", "load_geom_prod_tiled_cuda"),
    ("cliffordcuda.extensions.ga.wedge_prod.chunk", "load_wedge_prod_cuda"),
    ("cliffordcuda.extensions.ga.inner_prod.chunk", "load_inner_prod_cuda"),
    ("cliffordcuda.extensions.ga.left_contract", "load_contract_cuda"),
    ("cliffordcuda.extensions.rotor.eigh_exp", "load_eigh_exp_cuda"),
    ("cliffordcuda.extensions.rotor.givens_factor", "load_givens_factor_cuda"),
    ("cliffordcuda.extensions.rotor.givens_apply.mb_perm_packed",
     "load_givens_apply_mb_perm_packed_cuda"),
]


def build_reference_extensions():
    """JIT-build (or load) all of the reference's extensions at once, one
    thread per extension: the reference builds each on first use, one after
    the other, which takes about ten minutes on a fresh tree."""
    import importlib
    from concurrent.futures import ThreadPoolExecutor
    if REF not in sys.path:
        sys.path.insert(0, REF)

    def one(spec):
        mod, fn = spec
        getattr(importlib.import_module(mod), fn)()

    mods = [importlib.import_module(m) for m, _ in _LOADERS]  # imports stay serial
    del mods
    with ThreadPoolExecutor(len(_LOADERS)) as ex:
        list(ex.map(one, _LOADERS))


prepare_reference_env()
import torch  # noqa: E402


def _ref():
    if not os.path.isdir(os.path.join(REF, "cliffordcuda")):
        raise SystemExit(json.dumps({"impl": "reference-cuda",
                                     "unavailable": "baseline/_ref not installed"}))
    sys.path.insert(0, REF)
    import cliffordcuda
    build_reference_extensions()
    return cliffordcuda


def timed(step, K, W):
    for _ in range(W):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K):
        step()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / K


def rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm()).item()


def products_pair(ref, ours, op_ref, op_ours, n, metric, B, K, W):
    D = 1 << n
    g = torch.Generator(device="cuda").manual_seed(0)
    a, b, gr = (torch.randn(B, D, device="cuda", generator=g) for _ in range(3))
    ar, br = a.clone().requires_grad_(True), b.clone().requires_grad_(True)

    def step():
        ar.grad = br.grad = None
        c = op_ref(ar, br, metric=list(metric))
        c.backward(gr)
    ms = timed(step, K, W)
    S = min(B, 4096)
    a1, b1 = a[:S].clone().requires_grad_(True), b[:S].clone().requires_grad_(True)
    a2, b2 = a[:S].clone().requires_grad_(True), b[:S].clone().requires_grad_(True)
    c1 = op_ref(a1, b1, metric=list(metric))
    c1.backward(gr[:S])
    c2 = op_ours(a2, b2, metric=metric)
    c2.backward(gr[:S])
    agree = max(rel(c2, c1), rel(a2.grad, a1.grad), rel(b2.grad, b1.grad))
    return {"products_per_s": B / (ms / 1e3), "ms_per_step": ms,
            "rel_l2_vs_this_library": agree}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="all")
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--out", default=None, help="also append each JSON line to this file")
    args = ap.parse_args()
    ref = _ref()
    import cliffordcuda_b200 as ours
    K, W = args.steps, args.warmup
    todo = ["headline", "products", "layer", "rotor", "pga"] if args.workload == "all" \
        else [args.workload]
    fns = {"gp": "geom_prod", "wedge": "wedge_prod", "inner": "inner_prod",
           "lc": "left_contract", "rc": "right_contract"}
    for w in todo:
        out = {"impl": "reference-cuda", "workload": w, "device": torch.cuda.get_device_name()}
        if w == "headline":
            out["ops"] = {"gp": products_pair(ref, ours, ref.geom_prod, ours.geom_prod, 8,
                                              (1,) * 8, 524_288, K, W)}
        elif w == "products":
            out["ops"] = {op: products_pair(ref, ours, getattr(ref, f), getattr(ours, f), 7,
                                            (1,) * 6 + (-1,), 1_048_576, K, W)
                          for op, f in fns.items()}
        elif w == "pga":
            out["ops"] = {op: products_pair(ref, ours, getattr(ref, fns[op]),
                                            getattr(ours, fns[op]), 10, (1,) * 9 + (0,),
                                            131_072, K, W) for op in ("gp", "lc")}
        elif w == "layer":
            B, D = 524_288, 256
            cl = ref.CliffordAlgebra([1] * 8, device="cuda")
            lay = ref.GeometricProductLayer(cl)
            g = torch.Generator(device="cuda").manual_seed(1)
            x = torch.randn(B, D, device="cuda", generator=g).requires_grad_(True)
            dy = torch.randn(B, D, device="cuda", generator=g)

            def step():
                lay.weight.grad = None
                x.grad = None
                lay(x).backward(dy)
            ms = timed(step, K, W)
            ocl = ours.CliffordAlgebra([1] * 8, device="cuda")
            olay = ours.GeometricProductLayer(ocl)
            olay.load_state_dict(lay.state_dict())
            S = 4096
            x1, x2 = x[:S].detach().clone().requires_grad_(True), x[:S].detach().clone().requires_grad_(True)
            lay.weight.grad = None
            y1 = lay(x1)
            y1.backward(dy[:S])
            y2 = olay(x2)
            y2.backward(dy[:S])
            agree = max(rel(y2, y1), rel(x2.grad, x1.grad), rel(olay.weight.grad, lay.weight.grad))
            out.update({"rows_per_s": B / (ms / 1e3), "ms_per_step": ms, "per_gpu_batch": B,
                        "rel_l2_vs_this_library": agree})
        elif w == "rotor":
            B, D = 2_097_152, 256
            cl = ref.CliffordAlgebra([1] * 7 + [-1], device="cuda")
            lay = ref.RotorLayer(cl)
            g = torch.Generator(device="cuda").manual_seed(2)
            with torch.no_grad():
                lay.bivector.copy_(0.1 * torch.randn(1, 28, device="cuda", generator=g))
            x = torch.randn(B, D, device="cuda", generator=g).requires_grad_(True)
            gy = torch.randn(B, D, device="cuda", generator=g)

            def step():
                lay.bivector.grad = None
                lay(x).backward(gy)
            ms = timed(step, K, W)
            lay.eval()
            with torch.no_grad():
                ms_eval = timed(lambda: lay(x), K, W)
            ocl = ours.CliffordAlgebra([1] * 7 + [-1], device="cuda")
            olay = ours.RotorLayer(ocl)
            olay.load_state_dict(lay.state_dict())
            S = 4096
            lay.train()
            lay.bivector.grad = None
            xs = x[:S].detach()
            y1 = lay(xs)
            y1.backward(gy[:S])
            y2 = olay(xs)
            y2.backward(gy[:S])
            out.update({"train_rows_per_s": B / (ms / 1e3), "train_ms": ms,
                        "eval_rows_per_s": B / (ms_eval / 1e3), "eval_ms": ms_eval,
                        "per_gpu_batch": B,
                        "rel_l2_y_vs_this_library": rel(y2, y1),
                        "rel_l2_dbivector_vs_this_library": rel(olay.bivector.grad,
                                                               lay.bivector.grad)})
        print(json.dumps(out), flush=True)
        if args.out:
            with open(args.out, "a") as f:
                f.write(json.dumps(out) + "\n")


if __name__ == "__main__":
    main()
