"""Measurements of BASELINE configs 2-5 (bench.py --workload ...).

Each workload prints one JSON line with the same timing rules as bench.py's
headline: W warm-up steps, K timed steps bracketed by a barrier and a device
synchronisation, CUDA events on the launching stream, max over ranks, clocks
sampled during the timed region. Inputs are seeded synthetic data of the
config's shapes, all larger than L2.

  products  config 2: Cl(6,1), all five products fwd + both grads, batch
            1,048,576 split over the GPUs (strong scaling).
  layer     config 3: GeometricProductLayer (and Wedge/LeftContraction) in
            Cl(8,0), x (4,194,304 x 256) split over the GPUs, fwd + dX + dW,
            dW all-reduced (NCCL) every step.
  rotor     config 4: RotorLayer train step in Cl(7,1) on 2,097,152 rows split
            over the GPUs (compile, sandwich, backward to x and the bivector,
            all-reduce of the bivector gradient); eval (cached compile) apart.
  pga       config 5: Cl(9,0,1), batch 131,072 split over the GPUs, 10% of rows
            restricted to grades 0/2/4; geometric product and left contraction.
"""
from __future__ import annotations

import json
import math
import os
import statistics

import torch

from bench import ClockSampler, fp32_peak_tflops
from cliffordcuda_b200.distributed import allreduce_grads

PEAKS = {}
try:
    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")) as f:
        PEAKS = json.load(f)
except Exception:
    pass
HBM_GBS = float(PEAKS.get("hbm_gbs", 6650.0))
BF16_TFLOPS = float(PEAKS.get("bf16_tflops", 1590.0))
SM_MAX_MHZ = float(PEAKS.get("sm_max_mhz", 1965.0))
# Nominal tcgen05 kind::tf32 rate at the maximum SM clock: one 128x256x8 MMA
# per 128 cycles per SM = 4096 FLOP/clk/SM (the issue rate a stand-alone MMA
# loop measured on a B200, for single CTAs and CTA pairs alike). Higher, i.e.
# stricter, than measured bf16 / 2, which carries cuBLAS's efficiency and the
# power cap.
TF32_TFLOPS = 148 * 4096 * SM_MAX_MHZ * 1e6 / 1e12
X3TF32_TFLOPS = TF32_TFLOPS / 3     # three tf32 MMAs per fp32-accurate product


def nnz_table(op, n, metric):
    if op == "reg":  # dual o wedge o dual: the wedge's terms
        op = "wedge"
    D = 1 << n
    zero = sum(1 << t for t, m in enumerate(metric) if m == 0)
    i = torch.arange(D).view(-1, 1)
    j = torch.arange(D).view(1, -1)
    valid = (i & j & zero) == 0
    if op == "wedge":
        valid &= (i & j) == 0
    elif op == "inner":
        valid &= ((i & ~j) == 0) | ((j & ~i) == 0)
    elif op == "lc":
        valid &= (i & ~j) == 0
    elif op == "rc":
        valid &= (j & ~i) == 0
    return int(valid.sum())


class CollectiveClock:
    """CUDA events around the gradient all-reduce inside timed steps: its mean
    time per step, to state the collective's share of the step."""

    def __init__(self, stream):
        self.stream, self.pairs = stream, []

    def allreduce(self, module):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        allreduce_grads(module)
        e1.record(self.stream)
        self.pairs.append((e0, e1))

    def mean_ms(self, last):
        pairs = self.pairs[-last:] if last else []
        if not pairs:
            return None
        torch.cuda.synchronize()
        return statistics.mean(a.elapsed_time(b) for a, b in pairs)


class Timer:
    def __init__(self, dev, world):
        self.dev, self.world = dev, world
        self.stream = torch.cuda.current_stream(dev)

    def barrier(self):
        if self.world > 1:
            torch.distributed.barrier()

    def time(self, step, K, W):
        for _ in range(W):
            step()
        torch.cuda.synchronize(self.dev)
        self.barrier()
        torch.cuda.synchronize(self.dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(self.dev) as clk:
            e0.record(self.stream)
            for _ in range(K):
                step()
            e1.record(self.stream)
            torch.cuda.synchronize(self.dev)
        self.barrier()
        ms = e0.elapsed_time(e1)
        if self.world > 1:
            t = torch.tensor([ms], device=self.dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = t.item()
        return ms / K, clk.summary()


def _line(args, world, metric, value, unit, ms, clocks, config, extra, scaling="strong"):
    line = {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": "f32",
            "data": "synthetic, seeded", "config": config, "clocks": clocks}
    line.update(extra)
    return line


def products(args, world, rank, dev, T):
    from cliffordcuda_b200.products import bilinear_raw
    n, metric = 7, (1,) * 6 + (-1,)
    D = 1 << n
    B = args.batch or (1_048_576 // world)
    gen = torch.Generator(device=dev).manual_seed(2 + rank)
    a, b, g = (torch.randn(B, D, device=dev, generator=gen) for _ in range(3))
    outs = [torch.empty_like(a) for _ in range(3)]
    per_op = {}
    total_ms = 0.0
    for op in ("gp", "wedge", "inner", "lc", "rc", "reg"):
        def step():
            bilinear_raw(op, "fwd", a, b, n, metric, out=outs[0])
            bilinear_raw(op, "grad_a", b, g, n, metric, out=outs[1])
            bilinear_raw(op, "grad_b", a, g, n, metric, out=outs[2])
        ms, clk = T.time(step, args.steps, args.warmup)
        if op != "reg":  # the regressive product is not one of config 2's five
            total_ms += ms
        flops = 3 * 2 * nnz_table(op, n, metric) * B
        bytes_ = 3 * 3 * D * 4 * B
        # gp runs as two Cl(6,0) sums per row (half the blade-by-blade FMAs), so
        # its FP32 figure counts flops it does not execute: reported as an equivalent
        frac_key = "blade_flop_equivalent_pct" if op == "gp" else "pct_fp32_peak"
        per_op[op] = {"extra_not_in_config": op == "reg", "products_per_s": world * B / (ms / 1e3), "ms_per_step": ms,
                      "route": ("Cl(6,0) + Cl(6,0) through the central pseudoscalar (tiled kernel)"
                                if op == "gp" else "tiled blade-by-blade kernel"),
                      "fp32_tflops": flops / (ms / 1e3) / 1e12,
                      frac_key: 100 * flops / (ms / 1e3) / 1e12 / fp32_peak_tflops(dev),
                      "hbm_gbs": bytes_ / (ms / 1e3) / 1e9,
                      "pct_hbm": 100 * bytes_ / (ms / 1e3) / 1e9 / HBM_GBS}
    cfg = {"workload": "config 2: Cl(6,1) five products fwd+bwd", "per_gpu_batch": B,
           "global_batch": B * world, "dim": D, "metric": list(metric),
           "l2": "inputs 1.5 GB > L2"}
    return _line(args, world, "Cl(6,1) five products fwd+bwd, products/s (each product)",
                 world * B / (total_ms / 1e3), "products/s", total_ms, clk, cfg,
                 {"ops": per_op, "gpu_launches": 15 * args.steps})


def layer(args, world, rank, dev, T):
    import cliffordcuda_b200 as cc
    n = 8
    D = 1 << n
    B = args.batch or (4_194_304 // world)
    cl = cc.CliffordAlgebra([1] * n, device=dev)
    gen = torch.Generator(device=dev).manual_seed(3 + rank)
    x = torch.randn(B, D, device=dev, generator=gen).requires_grad_(True)
    dy = torch.randn(B, D, device=dev, generator=gen)
    res = {}
    main = None
    from cliffordcuda_b200 import layer_ops
    runs = (("gp", cc.GeometricProductLayer, None), ("wedge", cc.WedgeProductLayer, None),
            ("lc", cc.LeftContractionLayer, None), ("gp_tensor_route", None, "gp"))
    for name, cls, forced in runs:
        lay = cls(cl) if cls is not None else cc.GeometricProductLayer(cl)
        with torch.no_grad():
            lay.weight.copy_(torch.randn(1, D, device=dev, generator=gen) / math.sqrt(D))

        cc_clock = CollectiveClock(T.stream)

        def step():
            lay.weight.grad = None
            x.grad = None
            if forced:  # the dense 3xTF32 tcgen05 route for the GP layer
                y = layer_ops._LayerFn.apply(x, lay.weight, forced, n, tuple([1] * n))
            else:
                y = lay(x)
            y.backward(dy)
            cc_clock.allreduce(lay)
        ms, clk = T.time(step, args.steps, args.warmup)
        ar_ms = cc_clock.mean_ms(args.steps) if world > 1 else None
        useful = 3 * 2 * B * D * D
        matrix_route = name == "gp"
        res[name] = {"route": "16x16 matrix representation (cb_layer_gp8_*)" if matrix_route
                     else "3xTF32 tcgen05 GEMM (cb_layer_*)",
                     "rows_per_s": world * B / (ms / 1e3), "ms_per_step": ms,
                     "allreduce_ms_per_step": ar_ms,
                     "allreduce_share": None if ar_ms is None else ar_ms / ms,
                     "hbm_gbs": 6 * D * 4 * B / (ms / 1e3) / 1e9 if matrix_route
                     else 5 * D * 4 * B / (ms / 1e3) / 1e9}
        if not matrix_route:
            res[name]["useful_tflops"] = useful / (ms / 1e3) / 1e12
            res[name]["frac_3xtf32_peak"] = useful / (ms / 1e3) / 1e12 / X3TF32_TFLOPS
        if main is None:
            main = (ms, clk)
    ms, clk = main
    cfg = {"workload": "config 3: GeometricProductLayer fwd+bwd (dX, dW), dW all-reduced",
           "per_gpu_batch": B, "global_batch": B * world, "dim": D, "metric": [1] * n,
           "l2": "x, dy 512 MiB each > L2", "parallelism": f"dp{world}"}
    r = res["gp"]
    # The GP layer of Cl(8,0) runs through the 16 x 16 representation: HBM-bound,
    # algorithmic bytes per row and step = x, y (forward) + dy, dx (dx) + x, dy (dw).
    roof = {"bound": "hbm", "achieved": r["hbm_gbs"], "peak": HBM_GBS, "unit": "GB/s",
            "frac": r["hbm_gbs"] / HBM_GBS, "traffic": None,
            "peak_source": "MEASURED_PEAKS.json hbm_gbs",
            "algorithmic_bytes_per_row": 6 * D * 4}
    t = res["gp_tensor_route"]
    tensor_route = {"layer": "GeometricProductLayer through cb_layer_* (3xTF32 tcgen05 GEMM)",
                    "rows_per_s": t["rows_per_s"], "useful_tflops": t["useful_tflops"],
                    "peak": X3TF32_TFLOPS, "frac": t["frac_3xtf32_peak"],
                    "peak_source": "nominal tf32 tensor rate at max SM clock (148 SMs x 4096 "
                                   "FLOP/clk, the measured per-clock MMA rate) / 3 "
                                   "(3xTF32 MMAs per product)",
                    "frac_of_measured_bf16_over_6": t["useful_tflops"] / (BF16_TFLOPS / 6)}
    return _line(args, world, "Cl(8,0) GeometricProductLayer training rows/s",
                 r["rows_per_s"], "rows/s", ms, clk, cfg,
                 {"roofline": roof, "tensor_route": tensor_route, "layers": res},
                 scaling="strong")


def rotor(args, world, rank, dev, T):
    import cliffordcuda_b200 as cc
    n = 8
    D = 1 << n
    B = args.batch or (2_097_152 // world)
    cl = cc.CliffordAlgebra([1] * 7 + [-1], device=dev)
    gen = torch.Generator(device=dev).manual_seed(4 + rank)
    lay = cc.RotorLayer(cl)
    with torch.no_grad():
        lay.bivector.copy_(0.1 * torch.randn(1, 28, device=dev, generator=gen))
    x = torch.randn(B, D, device=dev, generator=gen).requires_grad_(True)
    g = torch.randn(B, D, device=dev, generator=gen)
    lay.train()

    cc_clock = CollectiveClock(T.stream)

    def step():
        lay.bivector.grad = None
        x.grad = None
        y = lay(x)
        y.backward(g)
        cc_clock.allreduce(lay)
    ms, clk = T.time(step, args.steps, args.warmup)
    ar_ms = cc_clock.mean_ms(args.steps) if world > 1 else None
    lay.eval()
    xe = x.detach()

    def eval_step():
        with torch.no_grad():
            lay(xe)
    ms_eval, _ = T.time(eval_step, args.steps, args.warmup)

    def compile_step():
        with torch.no_grad():
            cl.compile_bivector(lay.bivector)
    ms_compile, _ = T.time(compile_step, args.steps, args.warmup)
    train_bytes = 5 * D * 4 * B
    eval_bytes = 2 * D * 4 * B
    cfg = {"workload": "config 4: RotorLayer train step in Cl(7,1)", "per_gpu_batch": B,
           "global_batch": B * world, "dim": D, "metric": [1] * 7 + [-1],
           "l2": "x, g 2 GiB each > L2", "parallelism": f"dp{world}"}
    roof = {"bound": "hbm", "achieved": train_bytes / (ms / 1e3) / 1e9, "peak": HBM_GBS,
            "unit": "GB/s", "frac": train_bytes / (ms / 1e3) / 1e9 / HBM_GBS, "traffic": None,
            "peak_source": "MEASURED_PEAKS.json hbm_gbs"}
    return _line(args, world, "Cl(7,1) RotorLayer training rows/s", world * B / (ms / 1e3),
                 "rows/s", ms, clk, cfg,
                 {"roofline": roof,
                  "allreduce_ms_per_step": ar_ms,
                  "allreduce_share": None if ar_ms is None else ar_ms / ms,
                  "eval": {"rows_per_s": world * B / (ms_eval / 1e3), "ms": ms_eval,
                           "hbm_gbs": eval_bytes / (ms_eval / 1e3) / 1e9,
                           "frac_hbm": eval_bytes / (ms_eval / 1e3) / 1e9 / HBM_GBS},
                  "compile_ms": ms_compile})


def pga(args, world, rank, dev, T):
    from cliffordcuda_b200.products import bilinear_bwd_raw, bilinear_raw
    n, metric = 10, (1,) * 9 + (0,)
    D = 1 << n
    B = args.batch or (131_072 // world)
    gen = torch.Generator(device=dev).manual_seed(5 + rank)
    a, b, g = (torch.randn(B, D, device=dev, generator=gen) for _ in range(3))
    grades = torch.tensor([bin(i).count("1") for i in range(D)], device=dev)
    even = ((grades == 0) | (grades == 2) | (grades == 4)).float()
    rows = torch.randperm(B, generator=torch.Generator().manual_seed(9))[: B // 10].to(dev)
    a[rows] *= even
    b[rows] *= even
    outs = [torch.empty_like(a) for _ in range(3)]
    res = {}
    total = 0.0
    for op in ("gp", "lc"):
        def step():
            # the two native calls of the public API's autograd: the forward
            # and both backward sums (cb_bilinear_bwd*)
            bilinear_raw(op, "fwd", a, b, n, metric, out=outs[0])
            bilinear_bwd_raw(op, a, b, g, n, metric, outs[1], outs[2])
        ms, clk = T.time(step, args.steps, args.warmup)
        total += ms
        flops = 3 * 2 * nnz_table(op, n, metric) * B
        bytes_ = 8 * D * 4 * B  # forward: a, b, c; backward: a, b, g, grad_a, grad_b
        res[op] = {"route": "dual numbers over Cl(9,0) = Cl(8,0) + Cl(8,0): six 16x16 matrix "
                            "products per sum, one launch (pga10_kernel)" if op == "gp" else
                            "tiled blade-by-blade kernel",
                   "products_per_s": world * B / (ms / 1e3), "ms_per_step": ms,
                   "fp32_tflops": flops / (ms / 1e3) / 1e12,
                   ("blade_flop_equivalent_pct" if op == "gp" else "pct_fp32_peak"):
                       100 * flops / (ms / 1e3) / 1e12 / fp32_peak_tflops(dev),
                   "hbm_gbs": bytes_ / (ms / 1e3) / 1e9,
                   "pct_hbm": 100 * bytes_ / (ms / 1e3) / 1e9 / HBM_GBS}
    cfg = {"workload": "config 5: Cl(9,0,1) gp and lc fwd+bwd, 10% rows even-versor",
           "per_gpu_batch": B, "global_batch": B * world, "dim": D, "metric": list(metric),
           "l2": "inputs 1.5 GB > L2"}
    return _line(args, world, "Cl(9,0,1) gp + lc fwd+bwd products/s", world * B / (total / 1e3),
                 "products/s", total, clk, cfg, {"ops": res})


def large(args, world, rank, dev, T):
    """Large algebras (not a BASELINE config; the reference's own large-n tests
    use these signatures): the geometric product fwd + both grads at n = 12, 14
    and 16 on the wide kernel, against the FP32 peak (2 * 4^n flops per sum)."""
    from cliffordcuda_b200.products import bilinear_bwd_raw, bilinear_raw
    res = {}
    total = 0.0
    clk = None
    for n, metric, B0 in ((12, (1,) * 12, 2048), (14, (1,) * 12 + (-1, -1), 128),
                          (16, (1,) * 13 + (-1, -1, 0), 8)):
        D = 1 << n
        B = args.batch or max(1, B0 // world)
        gen = torch.Generator(device=dev).manual_seed(n + rank)
        a, b, g = (torch.randn(B, D, device=dev, generator=gen) for _ in range(3))
        outs = [torch.empty_like(a) for _ in range(3)]

        def step():
            bilinear_raw("gp", "fwd", a, b, n, metric, out=outs[0])
            bilinear_bwd_raw("gp", a, b, g, n, metric, outs[1], outs[2])
        ms, clk = T.time(step, args.steps, args.warmup)
        total += ms
        flops = 3 * 2 * (4 ** n) * B
        res[f"n{n}"] = {"metric": list(metric), "batch": B, "products_per_s": world * B / (ms / 1e3),
                        "ms_per_step": ms, "pct_fp32_peak":
                            100 * flops / (ms / 1e3) / 1e12 / fp32_peak_tflops(dev)}
        del a, b, g, outs
    cfg = {"workload": "geometric product fwd+bwd at n = 12, 14, 16 (wide kernel)",
           "l2": "n = 12: inputs 100 MB; n = 14, 16: compute-bound"}
    return _line(args, world, "large-n gp fwd+bwd, % of FP32 peak", res["n14"]["pct_fp32_peak"],
                 "% FP32 peak", total, clk, cfg, {"sizes": res})


WORKLOADS = {"products": products, "layer": layer, "rotor": rotor, "pga": pga, "large": large}


def collect(args, world, rank, dev):
    """Every config workload on an initialised device (and process group when
    world > 1); {workload: line, or {"error": ...}}. Used by bench.py's
    default run so that configs 2-5 are measured beside the headline."""
    T = Timer(dev, world)
    out = {}
    for name, fn in WORKLOADS.items():
        try:
            out[name] = fn(args, world, rank, dev, T)
        except Exception as e:  # reported in the line, the headline still prints
            out[name] = {"error": repr(e)[:300]}
        torch.cuda.empty_cache()
    return out


def run(args, world, rank, local):
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        torch.distributed.init_process_group("nccl", device_id=dev)
    T = Timer(dev, world)
    fn = WORKLOADS[args.workload]
    line = fn(args, world, rank, dev, T)
    from cliffordcuda_b200 import _lib
    _lib.device_status(dev)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()
