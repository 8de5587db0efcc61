"""Agreement with the reference's own CUDA kernels on identical seeded inputs.

The unmodified reference is installed under baseline/_ref (pip --target, no
dependencies; its torch extensions JIT-build for sm_100 into
baseline/_ref_build on first use; the fixture builds them in parallel, about
a minute and a half on a fresh tree). These tests run it through its public API
beside this library and require relative L2 <= 1e-5 between the two fp32
results, the bar the reference's own kernels must meet against each other.
They skip when baseline/_ref is not installed.
"""
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "cliffordcuda")),
                                 reason="reference not installed under baseline/_ref")]
DEV = "cuda:0"
TOL = 1e-5


@pytest.fixture(scope="module")
def ref():
    from bench_reference_cuda import build_reference_extensions, prepare_reference_env
    prepare_reference_env()
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import cliffordcuda
    build_reference_extensions()
    return cliffordcuda


def rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm()).item()


def _pair(ref_fn, our_fn, n, metric, batch, seed):
    gen = torch.Generator(device=DEV).manual_seed(seed)
    a, b, g = (torch.randn(batch, 1 << n, device=DEV, generator=gen) for _ in range(3))
    out = []
    for fn, kw in ((ref_fn, {"metric": list(metric)}), (our_fn, {"metric": tuple(metric)})):
        at, bt = a.clone().requires_grad_(True), b.clone().requires_grad_(True)
        c = fn(at, bt, **kw)
        c.backward(g)
        out.append((c.detach(), at.grad, bt.grad))
    return [rel(o, r) for o, r in zip(out[1], out[0])]


CASES = [
    ("geom_prod", 8, (1,) * 8, 4096),
    ("geom_prod", 7, (1,) * 6 + (-1,), 4096),
    ("wedge_prod", 7, (1,) * 6 + (-1,), 4096),
    ("inner_prod", 7, (1,) * 6 + (-1,), 4096),
    ("left_contract", 7, (1,) * 6 + (-1,), 4096),
    ("right_contract", 7, (1,) * 6 + (-1,), 4096),
    ("regressive_prod", 7, (1,) * 6 + (-1,), 1024),
    ("geom_prod", 10, (1,) * 9 + (0,), 512),
    ("left_contract", 10, (1,) * 9 + (0,), 512),
    ("geom_prod", 8, (-1,) * 8, 1024),
    ("geom_prod", 5, (1, 1, 1, -1, 0), 4096),
    ("geom_prod", 14, (1,) * 11 + (-1, -1, 0), 1),    # the reference's tiled fused path
    ("left_contract", 12, (1,) * 11 + (-1,), 4),
]


@pytest.mark.parametrize("fn,n,metric,batch", CASES,
                         ids=[f"{c[0]}-n{c[1]}-{i}" for i, c in enumerate(CASES)])
def test_products_agree(ref, fn, n, metric, batch):
    import cliffordcuda_b200 as ours
    errs = _pair(getattr(ref, fn), getattr(ours, fn), n, metric, batch, seed=n)
    assert max(errs) <= TOL, f"{fn} n={n}: rel L2 (c, ga, gb) = {errs}"


def test_geometric_product_layer_agrees(ref):
    import cliffordcuda_b200 as ours
    gen = torch.Generator(device=DEV).manual_seed(1)
    x = torch.randn(4096, 256, device=DEV, generator=gen)
    dy = torch.randn(4096, 256, device=DEV, generator=gen)
    rl = ref.GeometricProductLayer(ref.CliffordAlgebra([1] * 8, device=DEV))
    ol = ours.GeometricProductLayer(ours.CliffordAlgebra([1] * 8, device=DEV))
    ol.load_state_dict(rl.state_dict())
    res = []
    for lay in (rl, ol):
        xt = x.clone().requires_grad_(True)
        y = lay(xt)
        y.backward(dy)
        res.append((y.detach(), xt.grad, lay.weight.grad))
    errs = [rel(o, r) for o, r in zip(res[1], res[0])]
    assert max(errs) <= TOL, errs


def test_rotor_layer_agrees(ref):
    """RotorLayer in Cl(7,1) (config 4's algebra): the sandwich and the
    bivector gradient (the reference returns no x gradient)."""
    import cliffordcuda_b200 as ours
    gen = torch.Generator(device=DEV).manual_seed(2)
    rl = ref.RotorLayer(ref.CliffordAlgebra([1] * 7 + [-1], device=DEV))
    with torch.no_grad():
        rl.bivector.copy_(0.1 * torch.randn(1, 28, device=DEV, generator=gen))
    ol = ours.RotorLayer(ours.CliffordAlgebra([1] * 7 + [-1], device=DEV))
    ol.load_state_dict(rl.state_dict())
    x = torch.randn(4096, 256, device=DEV, generator=gen)
    gy = torch.randn(4096, 256, device=DEV, generator=gen)
    res = []
    for lay in (rl, ol):
        lay.train()
        y = lay(x)
        y.backward(gy)
        res.append((y.detach(), lay.bivector.grad))
    assert rel(res[1][0], res[0][0]) <= TOL
    assert rel(res[1][1], res[0][1]) <= TOL


def test_blade_maps_agree(ref):
    import cliffordcuda_b200 as ours
    metric = [1] * 6 + [-1]
    rc, oc = ref.CliffordAlgebra(metric, device=DEV), ours.CliffordAlgebra(metric, device=DEV)
    x = torch.randn(1000, 128, device=DEV, generator=torch.Generator(device=DEV).manual_seed(3))
    for name in ("reverse", "grade_involution", "clifford_conjugation", "dual"):
        assert torch.equal(getattr(oc, name)(x), getattr(rc, name)(x)), name
    assert torch.equal(oc.grade_projection(x, 3), rc.grade_projection(x, 3))
    assert rel(oc.norm_sq(x), rc.norm_sq(x)) <= 1e-6
    assert torch.equal(ours.reverse(x), ref.reverse(x))
