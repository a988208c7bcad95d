"""Benchmark of the CompactLogic logic-layer hot path on B200 (prints ONE JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference] [--workload c2|c4]

Default workload c2 (the config the metric is quoted on): one data-parallel
training step of 784 -> 6 x LogicLayer(64000, K=16) -> GroupSum(10, tau=10) with cross-entropy,
per-layer NCCL all-reduce of the gate-logit gradients, clip_grad_norm_(10) and Adam(lr=0.01) — the
reference training loop (experiments/experiment_script.py:280-293).  Batch 1024 per GPU (weak
scaling); synthetic per-feature Bernoulli(p ~ U(0.1, 0.9)) inputs and uniform labels; activations of
one layer (64000 x 1024 x 4 B = 262 MB) exceed the 126 MB L2, so no explicit flush is needed.

The same line carries the packed discrete inference (c4: 784 -> 8 x 256000 -> GroupSum 10 over 2^22
samples sharded by sample) under "packed", each with its roofline, CPU baseline and end-to-end value.

--impl reference: the reference's CPU implementation of the path does not exist (its kernels are
CUDA-only), so the reference arm times the CPU oracle — a plain-C restatement of the reference
kernels, row-partitioned over all host threads — on a bounded sample of the same workload.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

C2 = dict(in_dim=784, width=64000, layers=6, K=16, k=10, tau=10.0, batch=1024)

# DRAM bytes (read + write) per launch of the dominant c2 kernel from one ncu capture (the backward
# kernel summary under profiles/): 2.160 GB for a 64000->64000 layer with grad_x, 0.317 GB for the
# 784->64000 first layer; averaged over the 6 backward launches of a step.  Cold-cache (ncu flushes
# before each pass), so an upper bound of the steady state.
NCU_TRAFFIC = {"logic_backward_kernel": (5 * 2.160e9 + 0.317e9) / 6}
C4 = dict(in_dim=784, width=256000, layers=8, k=10, tau=1.0, samples=1 << 22)
C3 = dict(batch=512, K=16, dense=128000, k=10, tau=20.0)
C5 = dict(in_dim=3072, width=1_000_000, layers=4, K=4, k=100, tau=30.0, batch=512)


# ------------------------------------------------------------------------------------------------
def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [v.strip() for v in ln.split(",")]
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def timed(fn, steps, warmup, dev):
    """Run fn() warmup times, then time exactly `steps` calls with CUDA events (barrier + sync on both
    sides); returns ms per step as the max over ranks."""
    from compactlogic_b200.parallel import max_over_ranks
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize(dev)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    torch.cuda.synchronize(dev)
    if dist.is_initialized():
        dist.barrier()
    return max_over_ranks(s.elapsed_time(e) / steps, dev)


# ------------------------------------------------------------------------------------------------
# c2: dense training step
# ------------------------------------------------------------------------------------------------
def build_c2(dev):
    import compactlogic_b200 as cl
    torch.manual_seed(0)  # identical replicas on every rank
    widths = [C2["in_dim"]] + [C2["width"]] * C2["layers"]
    layers = [cl.LogicLayer(widths[i], widths[i + 1], num_gates=C2["K"]) for i in range(C2["layers"])]
    model = torch.nn.Sequential(torch.nn.Flatten(), *layers, cl.GroupSum(C2["k"], C2["tau"])).to(dev)
    cl.fuse_groupsum(model)
    return model


def c2_inputs(seed, batch):
    g = torch.Generator().manual_seed(seed)
    p = torch.rand(C2["in_dim"], generator=g) * 0.8 + 0.1
    x = (torch.rand(batch, C2["in_dim"], generator=g) < p).float()
    y = torch.randint(0, C2["k"], (batch,), generator=g)
    return x, y


def c2_bytes_per_step(B):
    """Compulsory HBM bytes of one step (fp32, GroupSum fused, Adam excluded): per soft layer
    e*B*(in + out) + n_out*K*13 forward and e*B*(2 in + out) + n_out*K*13 backward, without y for the
    fused last layer, without grad_x for the first."""
    e, K, W, I = 4, C2["K"], C2["width"], C2["in_dim"]
    par = W * K * 13
    fwd = e * B * (I + W) + par + (C2["layers"] - 2) * (e * B * 2 * W + par) + (e * B * W + par)
    bwd = (e * B * (I + W) + par) + (C2["layers"] - 2) * (e * B * 3 * W + par) + (e * B * 2 * W + par)
    return fwd + bwd


def clip_sharded(params, max_norm):
    """clip_grad_norm_ over parameters sharded across the ranks (one all-reduce of the squared norm)."""
    sq = torch.stack([p.grad.float().pow(2).sum() for p in params if p.grad is not None]).sum()
    if dist.is_initialized():
        dist.all_reduce(sq)
    coef = torch.clamp(max_norm / (sq.sqrt() + 1e-6), max=1.0)
    for p in params:
        if p.grad is not None:
            p.grad.mul_(coef)


def bench_c2(args, dev, rank, world):
    from compactlogic_b200 import _lib
    from compactlogic_b200.functional import TIMER
    from compactlogic_b200.parallel import GradAllReduce
    width = args.parallel == "width"
    model = build_c2(dev)
    if width:
        # neuron-parallel: every rank runs the whole batch on its share of each layer's neurons
        from compactlogic_b200.sharded import shard_width
        model = shard_width(model)
    params = [p for p in model.parameters() if p.requires_grad]
    opt = torch.optim.Adam(params, lr=0.01, fused=True)
    sync = None if width else GradAllReduce(params)
    strong = args.strong and not width
    B = C2["batch"] // world if strong else C2["batch"]
    x_host, y_host = c2_inputs(1000 + (0 if width else rank), B)
    x_dev, y_dev = x_host.to(dev), y_host.to(dev)

    def step(x, y):
        opt.zero_grad(set_to_none=True)
        loss = torch.nn.functional.cross_entropy(model(x), y)
        loss.backward()
        if sync is not None:
            sync.finish()
            torch.nn.utils.clip_grad_norm_(params, 10.0)
        else:
            clip_sharded(params, 10.0)
        opt.step()
        return loss

    # device-resident inputs: `value`
    n0 = _lib.launches()
    TIMER.reset()
    TIMER.enabled = True
    with Clocks(dev.index) as clk:
        ms = timed(lambda: step(x_dev, y_dev), args.steps, args.warmup, dev)
    TIMER.enabled = False
    launches = (_lib.launches() - n0) * args.steps // (args.steps + args.warmup)
    kern = TIMER.summary()
    TIMER.reset()

    # end to end through the public API from pinned host buffers
    xp, yp = x_host.pin_memory(), y_host.pin_memory()
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()

    def e2e_step():
        x = xp.to(dev, non_blocking=True)
        y = yp.to(dev, non_blocking=True)
        loss = step(x, y)
        loss_host.copy_(loss.detach(), non_blocking=True)

    ms_e2e = timed(e2e_step, args.steps, max(1, args.warmup // 2), dev)

    hbm, src = peaks()
    # dominant kernel by total time
    dom = max(kern, key=lambda k: kern[k][1]) if kern else None
    roof = None
    if dom:
        n, tot_ms, tot_b = kern[dom]
        achieved = tot_b / (tot_ms / 1e3) / 1e9
        roof = {"kernel": f"logic_{dom}_kernel", "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm,
                "peak_source": src, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                "traffic": NCU_TRAFFIC.get(f"logic_{dom}_kernel") if C2["layers"] == 6 and B == 1024 and not width else None,
                "traffic_note": "ncu dram__bytes_read+write per launch, cold cache (profiles/)",
                "algorithmic_bytes_per_launch": round(tot_b / n), "launches": n, "avg_ms": round(tot_ms / n, 4),
                "shares": {k: round(v[1] / sum(w[1] for w in kern.values()), 3) for k, v in kern.items()}}
    step_bytes = c2_bytes_per_step(B)
    gb = B if width else B * world  # strong DP: B = 1024 / world, so gb = 1024
    res = {
        "metric": "train_samples_per_s", "value": round(gb / (ms / 1e3), 1), "unit": "samples/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "strong" if (width or strong) else "weak", "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": f"c2: 784 -> {C2['layers']}x LogicLayer(64000, K=16) -> GroupSum(10, tau=10); CE, "
                               + ("width-sharded neurons, peer-fused gather / reduce-scatter" if width else
                                  "all-reduce") + ", clip 10, Adam",
                   "batch_per_gpu": B, "global_batch": gb,
                   "parallelism": f"width{world}" if width else f"dp{world}",
                   "l2": "per-layer activations 262 MB > L2 126 MB (no flush)"},
        "step_hbm_bytes_algorithmic": step_bytes,
        "step_hbm_frac": round(step_bytes / (ms / 1e3) / 1e9 / hbm, 4),
        "roofline": roof,
        "kernels": {k: {"launches": v[0], "ms_total": round(v[1], 3), "gb": round(v[2] / 1e9, 3)}
                    for k, v in kern.items()},
        "clocks": clk.summary(),
        "e2e": {"value": round(gb / (ms_e2e / 1e3), 1), "unit": "samples/s",
                "h2d_bytes_per_step": x_host.numel() * 4 + y_host.numel() * 8, "d2h_bytes_per_step": 4},
        "gpu_launches": int(launches),
    }
    return res, model


def bench_c2_reference_kernels(args, dev):
    """The same c2 step driven through the reference's own CUDA kernels (oracle/_ref, built unmodified
    for sm_100) with the reference's Python around them: softmax in torch (compactlogic.py:108), the
    three kernels through the autograd bridge (compactlogic.py:474-508), GroupSum in torch
    (compactlogic.py:460-465).  Reported beside the native step; not part of the product."""
    import importlib.util
    path = os.path.join(ROOT, "oracle", "_ref", "difflogic_cuda.so")
    if not os.path.exists(path):
        return {"unavailable": "oracle/_ref/difflogic_cuda.so not built (needs the reference tree at build time)"}
    spec = importlib.util.spec_from_file_location("difflogic_cuda", path)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)

    class RefFn(torch.autograd.Function):
        @staticmethod
        def forward(ctx, x, a, b, w, g, st, ys, codes):
            ctx.save_for_backward(x, a, b, w, g, st, ys, codes)
            return ref.forward(x, a, b, w, g)

        @staticmethod
        def backward(ctx, gy):
            x, a, b, w, g, st, ys, codes = ctx.saved_tensors
            gy = gy.contiguous()
            gx = ref.backward_x(x, a, b, w, g, gy, st, ys, codes) if ctx.needs_input_grad[0] else None
            gw = ref.backward_w(x, a, b, g, gy) if ctx.needs_input_grad[3] else None
            return gx, None, None, gw, None, None, None, None

    model = build_c2(dev)
    layers = [m for m in model if hasattr(m, "indices")]
    params = [m.weights for m in layers]
    opt = torch.optim.Adam(params, lr=0.01, fused=True)
    x_host, y_host = c2_inputs(1000, C2["batch"])
    x_dev, y_dev = x_host.to(dev), y_host.to(dev)

    def step():
        opt.zero_grad(set_to_none=True)
        h = x_dev
        for m in layers:
            xt = h.transpose(0, 1).contiguous()
            w = torch.nn.functional.softmax(m.weights, dim=-1).to(xt.dtype)
            h = RefFn.apply(xt, m.indices[0], m.indices[1], w, m.gate_sequence, m.given_x_indices_of_y_start,
                            m.given_x_indices_of_y, m.given_x_indices_of_gate).transpose(0, 1)
        logits = h.reshape(h.shape[0], C2["k"], -1).sum(-1) / C2["tau"]
        loss = torch.nn.functional.cross_entropy(logits, y_dev)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(params, 10.0)
        opt.step()

    steps = max(2, args.steps // 3)
    ms = timed(step, steps, 2, dev)
    return {"value": round(C2["batch"] / (ms / 1e3), 1), "unit": "samples/s", "ms_per_step": round(ms, 3),
            "steps": steps, "what": "same c2 step on the reference CUDA kernels compiled for sm_100"}


# ------------------------------------------------------------------------------------------------
# c3: conv model training step;  c5: wide compact-gate bf16 training step
# ------------------------------------------------------------------------------------------------
def build_c3(dev):
    import compactlogic_b200 as cl
    torch.manual_seed(1)
    conv1 = cl.ConvLayer((9, 32, 32), 1, 128, 3, 2, num_gates=C3["K"])
    conv2 = cl.ConvLayer((128, 16, 16), 1, 256, 3, 2, num_gates=C3["K"])
    dense = cl.LogicLayer(256 * 8 * 8, C3["dense"], num_gates=C3["K"])
    model = torch.nn.Sequential(conv1, conv2, torch.nn.Flatten(), dense, cl.GroupSum(C3["k"], C3["tau"])).to(dev)
    return cl.fuse_groupsum(model)


def c3_inputs(seed, batch):
    """3 channels of U(0,1) pixels thresholded at 1/4, 2/4, 3/4 (experiments/experiment_script.py:92)."""
    g = torch.Generator().manual_seed(seed)
    px = torch.rand(batch, 3, 32, 32, generator=g)
    x = torch.cat([(px > (i + 1) / 4).float() for i in range(3)], dim=1)  # threshold-major channels
    return x, torch.randint(0, C3["k"], (batch,), generator=g)


def build_c5(dev):
    import compactlogic_b200 as cl
    torch.manual_seed(5)
    widths = [C5["in_dim"]] + [C5["width"]] * C5["layers"]
    layers = []
    for i in range(C5["layers"]):
        layer = cl.LogicLayer(widths[i], widths[i + 1], num_gates=C5["K"])
        with torch.no_grad():  # candidate gate ids uniform in [0, 16) instead of the constructor's 0..K-1
            layer.gate_sequence.copy_(torch.randint(0, 16, layer.gate_sequence.shape, dtype=torch.uint8))
        layers.append(layer)
    model = torch.nn.Sequential(*layers, cl.GroupSum(C5["k"], C5["tau"])).to(dev)
    return cl.fuse_groupsum(model)


def c5_inputs(seed, batch):
    g = torch.Generator().manual_seed(seed)
    return ((torch.rand(batch, C5["in_dim"], generator=g) < 0.5).to(torch.bfloat16),
            torch.randint(0, C5["k"], (batch,), generator=g))


def bench_train(args, dev, rank, world, workload):
    """Training step of c3 / c5 (same loop and timing rules as c2)."""
    from compactlogic_b200.parallel import GradAllReduce
    if workload == "c3":
        model, (x_host, y_host), B, dtype = build_c3(dev), c3_inputs(1000 + rank, C3["batch"]), C3["batch"], "f32"
        desc = "c3: (9,32,32) -> Conv(128,ks3,s2,p1) -> Conv(256,ks3,s2,p1) -> LogicLayer(128000) -> GroupSum(10, 20)"
    else:
        model, (x_host, y_host), B, dtype = build_c5(dev), c5_inputs(1000 + rank, C5["batch"]), C5["batch"], "bf16"
        desc = "c5: 3072 -> 4x LogicLayer(1e6, K=4, gate ids U{0..15}) -> GroupSum(100, 30); bf16 activations"
    params = [p for p in model.parameters() if p.requires_grad]
    opt = torch.optim.Adam(params, lr=0.01, fused=True)
    sync = GradAllReduce(params)
    x_dev, y_dev = x_host.to(dev), y_host.to(dev)

    def step(x, y):
        opt.zero_grad(set_to_none=True)
        loss = torch.nn.functional.cross_entropy(model(x), y)
        loss.backward()
        sync.finish()
        torch.nn.utils.clip_grad_norm_(params, 10.0)
        opt.step()
        return loss

    with Clocks(dev.index) as clk:
        ms = timed(lambda: step(x_dev, y_dev), args.steps, args.warmup, dev)
    xp, yp = x_host.pin_memory(), y_host.pin_memory()
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()

    def e2e():
        loss = step(xp.to(dev, non_blocking=True), yp.to(dev, non_blocking=True))
        loss_host.copy_(loss.detach(), non_blocking=True)

    ms_e2e = timed(e2e, args.steps, 1, dev)
    return {"metric": "train_samples_per_s", "value": round(world * B / (ms / 1e3), 1), "unit": "samples/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype, "data": "synthetic",
            "config": {"workload": desc, "batch_per_gpu": B, "global_batch": B * world, "parallelism": f"dp{world}"},
            "clocks": clk.summary(),
            "e2e": {"value": round(world * B / (ms_e2e / 1e3), 1), "unit": "samples/s",
                    "h2d_bytes_per_step": x_host.numel() * x_host.element_size() + y_host.numel() * 8,
                    "d2h_bytes_per_step": 4}}


def cpu_baseline_c2(model, budget_s, steps=1):
    """The oracle (reference kernels restated in C, all host threads) on a bounded sub-batch of the
    c2 step: forward through the 6 layers, GroupSum + CE gradient, backward (grad_x and grad_w)."""
    from oracle import oracle as O
    layers = [m for m in model if hasattr(m, "indices")]
    tabs = [(m.indices.cpu().numpy(), m.gate_sequence.cpu().numpy(),
             O.softmax(m.weights.detach().cpu().numpy().astype(np.float64))) for m in layers]

    def run(b):
        x, y = c2_inputs(7, b)
        h = [x.numpy().T.astype(np.float64)]
        for idx, g, p in tabs:
            h.append(O.dense_forward(h[-1], idx[0], idx[1], p, g))
        logits = O.group_sum(h[-1].T, C2["k"], C2["tau"])
        gy = O.group_sum_backward(O.cross_entropy_grad(logits, y.numpy()), C2["width"], C2["k"], C2["tau"]).T
        for li in range(len(tabs) - 1, -1, -1):
            idx, g, p = tabs[li]
            O.dense_backward_w(h[li], idx[0], idx[1], g, gy)
            if li > 0:
                gy = O.dense_backward_x(h[li], idx[0], idx[1], p, g, gy)

    t = time.perf_counter()
    run(4)
    t4 = time.perf_counter() - t
    b = int(max(4, min(1024, 4 * budget_s / max(t4, 1e-3))))
    b = max(4, (b // 4) * 4)
    t = time.perf_counter()
    for _ in range(steps):
        run(b)
    dt = (time.perf_counter() - t) / steps
    return {"value": round(b / dt, 3), "unit": "samples/s", "cores": O.THREADS, "kind": "port",
            "sample": f"one c2 training step (fwd+bwd of 6 layers, no optimizer) on a sub-batch of {b} samples, "
                      f"{dt:.1f} s"}


# ------------------------------------------------------------------------------------------------
# c4: packed discrete inference
# ------------------------------------------------------------------------------------------------
def build_c4(dev):
    """Frozen 784 -> 8 x 256000 -> GroupSum(10): winning gate ids uniform in [0, 16), winning pairs
    random (realised through the reference's own connection sampler and argmax of random logits)."""
    import compactlogic_b200 as cl
    torch.manual_seed(4)
    widths = [C4["in_dim"]] + [C4["width"]] * C4["layers"]
    layers = []
    for i in range(C4["layers"]):
        layer = cl.LogicLayer(widths[i], widths[i + 1], num_gates=1)
        with torch.no_grad():
            layer.gate_sequence.copy_(torch.randint(0, 16, layer.gate_sequence.shape, dtype=torch.uint8))
        layer.freeze()
        layers.append(layer)
    model = torch.nn.Sequential(*layers, cl.GroupSum(C4["k"], C4["tau"])).to(dev)
    return model


def bench_c4(args, dev, rank, world, chunk_words):
    import compactlogic_b200 as cl
    from compactlogic_b200 import _lib
    from compactlogic_b200.parallel import shard_range
    model = build_c4(dev)
    net = cl.PackedLogicNet(model, chunk_words=chunk_words)
    lo, hi = shard_range(C4["samples"], rank, world)
    n = hi - lo
    W = -(-n // 64)
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    xw = torch.randint(-2**63, 2**63 - 1, (C4["in_dim"], W), dtype=torch.int64, device=dev, generator=g)
    counts = torch.zeros(n, C4["k"], dtype=torch.int32, device=dev)
    steps = max(1, args.steps // 2)
    with Clocks(dev.index) as clk:
        ms = timed(lambda: net.counts_packed(xw, n, counts), steps, max(1, args.warmup // 2), dev)
    launches = net.launches_per_pass * steps
    evals = C4["samples"] * C4["width"] * C4["layers"]
    # end to end: packed words from pinned host memory into a fixed device buffer, counts back to
    # pinned host memory
    xh = xw.cpu().pin_memory()
    ch = torch.empty_like(counts, device="cpu").pin_memory()
    x_in = torch.empty_like(xw)

    def e2e():
        x_in.copy_(xh, non_blocking=True)
        c = net.counts_packed(x_in, n, counts)
        ch.copy_(c, non_blocking=True)

    ms_e2e = timed(e2e, steps, 1, dev)
    pruned = None
    if not args.no_prune:
        # the same network after the compiler's stage-1 pruning: fewer gates, identical counts
        pnet = cl.PackedLogicNet(model, chunk_words=chunk_words, prune="exact")
        pcounts = torch.zeros_like(counts)
        ms_p = timed(lambda: pnet.counts_packed(xw, n, pcounts), steps, 1, dev)
        pruned = {"value": round(evals / (ms_p / 1e3), 1), "unit": "network gate-evals/s",
                  "ms_per_step": round(ms_p, 3), "gates": pnet.prune_stats["gates"],
                  "kept_gates": pnet.prune_stats["kept"], "counts_equal_unpruned": bool(torch.equal(pcounts, counts)),
                  "note": "value counts the unpruned network's gates; the kernels evaluate only the kept ones"}
        del pnet
    # roofline of the packed layer kernel: time one chunk's layer launches with events
    hbm, src = peaks()
    bytes_model = (8 * W * (C4["in_dim"] + C4["width"]) + C4["width"] * 9 +
                   (C4["layers"] - 2) * (8 * W * 2 * C4["width"] + C4["width"] * 9) +
                   (8 * W * C4["width"] + C4["width"] * 9 + 4 * C4["k"] * 64 * W))
    achieved = bytes_model / (ms / 1e3) / 1e9
    return {
        "metric": "packed_infer_gate_evals_per_s", "value": round(evals / (ms / 1e3), 1), "unit": "gate-evals/s",
        "ms_per_step": round(ms, 3), "steps": steps, "dtype": "u64",
        "config": {"workload": "c4: 784 -> 8x256000 frozen -> GroupSum(10), 2^22 samples sharded by sample",
                   "samples_per_gpu": n, "chunk_words": chunk_words},
        "roofline": {"kernel": "packed layer chain (all launches of one pass)", "bound": "hbm",
                     "achieved": round(achieved, 1), "peak": hbm, "peak_source": src, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": None,
                     "note": "byte model: every layer's activations make one HBM round trip (128-word chunks "
                             "stream through HBM); frac > 1 would mean a chunk stayed in L2"},
        "clocks": clk.summary(),
        "e2e": {"value": round(evals / (ms_e2e / 1e3), 1), "unit": "gate-evals/s",
                "h2d_bytes_per_step": xh.numel() * 8, "d2h_bytes_per_step": ch.numel() * 4},
        "gpu_launches": int(launches),
        "pruned": pruned,
    }, model


def cpu_baseline_c4(model, budget_s, steps=1):
    from oracle import oracle as O
    layers = [m for m in model if hasattr(m, "indices")]
    tabs = [O.frozen_tables(m.indices.cpu().numpy(), m.gate_sequence.cpu().numpy(), m.w.cpu().numpy())
            for m in layers]
    rng = np.random.default_rng(0)

    def run(words):
        h = rng.integers(0, 2**63, (C4["in_dim"], words), dtype=np.int64).astype(np.uint64)
        for ab, g in tabs:
            h = O.packed_layer(h, ab, g, fast=True)
        O.packed_count(h, C4["k"], 64 * words)

    t = time.perf_counter()
    run(1)
    t1 = time.perf_counter() - t
    words = int(max(1, min(4096, budget_s / max(t1, 1e-3))))
    t = time.perf_counter()
    for _ in range(steps):
        run(words)
    dt = (time.perf_counter() - t) / steps
    evals = 64 * words * C4["width"] * C4["layers"]
    return {"value": round(evals / dt, 1), "unit": "gate-evals/s", "cores": O.THREADS, "kind": "port",
            "sample": f"{64 * words} samples through all 8 layers + counts (uint64 word loop), {dt:.1f} s"}


# ------------------------------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--workload", default="c2", choices=["c2", "c3", "c4", "c5"])
    ap.add_argument("--no-packed", action="store_true", help="skip the packed-inference (c4) sub-measurement")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--no-refcuda", action="store_true", help="skip the reference-CUDA-kernel step timing")
    ap.add_argument("--chunk-words", type=int, default=128)
    ap.add_argument("--no-prune", action="store_true", help="skip the pruned packed-inference sub-measurement")
    ap.add_argument("--strong", action="store_true",
                    help="c2 data parallel with the global batch fixed at 1024 (1024/N per GPU)")
    ap.add_argument("--parallel", default="dp", choices=["dp", "width"],
                    help="c2 multi-GPU scheme: data parallel (default) or width-sharded neurons")
    ap.add_argument("--layers", type=int, default=None, help="override the c2 depth (profiling on a smaller case)")
    ap.add_argument("--samples", type=int, default=None, help="override the c4 sample count (profiling)")
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU work per baseline sample")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.layers:
        C2["layers"] = args.layers
    if args.samples:
        C4["samples"] = args.samples

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        # CPU arm: rank 0 only, the other ranks exit without work.
        if rank != 0:
            return
        torch.manual_seed(0)
        per_step = max(1.0, min(args.cpu_budget, 150.0 / max(1, args.steps)))  # whole arm within a few minutes
        if args.workload == "c4":
            res = cpu_baseline_c4(build_c4("cpu"), per_step, args.steps)
            metric = "packed_infer_gate_evals_per_s"
        else:
            res = cpu_baseline_c2(build_c2("cpu"), per_step, args.steps)
            metric = "train_samples_per_s"
        line = {"impl": "reference", "metric": metric, "value": res["value"], "unit": res["unit"], "n_gpus": world,
                "steps": args.steps, "warmup": 0, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f64" if metric.startswith("train") else "u64", "data": "synthetic",
                "config": {"workload": args.workload, "arm": "CPU oracle (reference kernels restated in C)"},
                "cpu_baseline": res,
                "e2e": {"value": res["value"], "unit": res["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    if args.workload in ("c3", "c5"):
        res = bench_train(args, dev, rank, world, args.workload)
    elif args.workload == "c4":
        res, model = bench_c4(args, dev, rank, world, args.chunk_words)
        if rank == 0 and world == 1 and not args.no_cpu:
            res["cpu_baseline"] = cpu_baseline_c4(model, args.cpu_budget)
        res.update({"n_gpus": world, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
                    "vs_baseline": None, "data": "synthetic"})
    else:
        res, model = bench_c2(args, dev, rank, world)
        del model
        torch.cuda.empty_cache()
        if not args.no_packed:
            packed, pmodel = bench_c4(args, dev, rank, world, args.chunk_words)
            if rank == 0 and world == 1 and not args.no_cpu:
                packed["cpu_baseline"] = cpu_baseline_c4(pmodel, args.cpu_budget / 2)
            res["packed"] = packed
            del pmodel
        if world == 1 and not args.no_refcuda:
            res["reference_cuda_kernels"] = bench_c2_reference_kernels(args, dev)
            torch.cuda.empty_cache()
        if rank == 0 and world == 1 and not args.no_cpu:
            res["cpu_baseline"] = cpu_baseline_c2(build_c2("cpu"), args.cpu_budget)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
