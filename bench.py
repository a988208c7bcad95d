"""Benchmark of the CompactLogic logic-layer hot path on B200 (prints ONE JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference] [--workload c1|c2|c3|c4|c5]

Default workload c2 (the config the metric is quoted on): one data-parallel
training step of 784 -> 6 x LogicLayer(64000, K=16) -> GroupSum(10, tau=10) with cross-entropy,
per-layer NCCL all-reduce of the gate-logit gradients, clip_grad_norm_(10) and Adam(lr=0.01) — the
reference training loop (experiments/experiment_script.py:280-293).  Batch 1024 per GPU (weak
scaling); synthetic per-feature Bernoulli(p ~ U(0.1, 0.9)) inputs and uniform labels; activations of
one layer (64000 x 1024 x 4 B = 262 MB) exceed the 126 MB L2, so no explicit flush is needed.

The same line carries the other BASELINE configurations as sub-blocks, each with its own roofline,
CPU baseline and end-to-end value:
  "c1"      one LogicLayer(784, 12000, K=16) forward + backward at batch 256 (1 GPU only), with the
            same pass on the reference's own CUDA kernels;
  "c3"      the conv model training step at batch 512 per GPU, with the reference's kernels beside it;
  "c5"      the 1M-wide K=4 bf16 training step at batch 512 per GPU;
  "packed"  c4, discrete bit-packed inference of 784 -> 8 x 256000 -> GroupSum 10 over 2^22 samples
            sharded by sample, the count all-gather inside the timed region;
  "strong"  (N > 1) c2 with the global batch fixed at 1024 (1024/N per GPU).
The soft kernels are bound by L2 gather / reduction throughput, not HBM: each roofline carries an
"l2" object, the kernel's L2 bytes against a probe of the same access pattern measured in this run.

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

C1 = dict(in_dim=784, out=12000, K=16, batch=256)
C2 = dict(in_dim=784, width=64000, layers=6, K=16, k=10, tau=10.0, batch=1024)
C3 = dict(batch=512, K=16, dense=128000, k=10, tau=20.0)
C4 = dict(in_dim=784, width=256000, layers=8, k=10, tau=1.0, samples=1 << 22)
C5 = dict(in_dim=3072, width=1_000_000, layers=4, K=4, k=100, tau=30.0, batch=512)

# DRAM bytes (read + write) per launch from ncu captures (the summaries under profiles/), cold cache
# (ncu flushes before each pass), so upper bounds of the steady state:
#  - logic_backward_kernel at the c2 shapes: 2.160 GB for a 64000->64000 layer with grad_x, 0.317 GB for
#    the 784->64000 first layer; averaged over the 6 backward launches of a step;
#  - the c4 pass (2^22 samples, 128-word chunks = 512 chunks): per chunk one first-layer launch
#    (~0.263 GB: its 0.8 MB input + 262 MB output), six inner-layer launches (0.583 GB each, measured)
#    and one fused count launch (0.343 GB, measured).
# Checksum of the gathered c4 class counts (sum over samples i and classes of count * (i % 1009 + 1)) for the
# fixed seeds of build_c4 / c4_words, measured on one B200: every N must reproduce it.
C4_COUNTS_CHECKSUM = 270315957402565
#  - logic_backward_gather2_kernel (the default fp32 backward of the 64000->64000 layers): 1.078 GB per launch
#    (0.797 GB read + 0.281 GB write, profiles/logic_backward_gather_c2.md); the first layer keeps the
#    scatter kernel without grad_x (0.317 GB);
NCU_TRAFFIC = {"logic_backward_kernel": (5 * 2.160e9 + 0.317e9) / 6,
               "logic_backward_gather2_kernel": 1.078e9,
               "packed_pass": 512 * (0.263e9 + 6 * 0.583e9 + 0.343e9)}


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


def timed_kernels(fn, steps, warmup, dev):
    """timed() with the layer kernels' CUDA-event timer on; returns (ms per step, kernel summary, launches
    of this library per timed step)."""
    from compactlogic_b200 import _lib
    from compactlogic_b200.functional import TIMER
    n0 = _lib.launches()
    TIMER.reset()
    TIMER.enabled = True
    try:
        ms = timed(fn, steps, warmup, dev)
    finally:
        TIMER.enabled = False
    torch.cuda.synchronize(dev)
    kern = TIMER.summary()
    TIMER.reset()
    launches = (_lib.launches() - n0) * steps // (steps + warmup)
    return ms, kern, int(launches)


# ------------------------------------------------------------------------------------------------
# L2 ceiling of the soft kernels' access pattern, measured in this run
# ------------------------------------------------------------------------------------------------
_L2 = {}


def l2_peaks(dev):
    """GB/s of 512-byte row gathers (mode 0) and gathers + vector reductions (mode 1) at hashed rows of
    two 33.5 MB slabs (65536 rows, about one 128-column chunk of a c2 layer's x and grad_x), best of 5."""
    if _L2:
        return _L2
    from compactlogic_b200 import _lib as L
    rows, ctas, iters = 65536, 148 * 8, 2000
    src = torch.rand(rows, 128, device=dev)
    dst = torch.zeros(rows, 128, device=dev)
    sink = torch.zeros(1, device=dev)
    for mode, per_step in ((0, 1024), (1, 2048)):
        best = 0.0
        for i in range(6):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            L.call("clb_l2_probe", mode, L.ptr(src), L.ptr(dst), rows, iters, ctas, L.ptr(sink), L.stream(dev))
            e.record()
            torch.cuda.synchronize(dev)
            if i:
                best = max(best, ctas * 8 * iters * per_step / (s.elapsed_time(e) / 1e3) / 1e9)
        _L2["gather" if mode == 0 else "gather_reduce"] = round(best, 1)
    del src, dst
    return _L2


def roofline(kern, hbm, src, traffic=None, dev=None, extra=None):
    """Dominant kernel (by live CUDA-event time) of a TIMER summary: algorithmic HBM bytes / event time
    against the measured copy bandwidth, and its L2 gather (+ reduction) bytes against the probe."""
    if not kern:
        return None
    dom = max(kern, key=lambda k: kern[k][1])
    n, tot_ms, tot_b, tot_l2 = kern[dom]
    if isinstance(traffic, dict):
        traffic = traffic.get(dom)
    achieved = tot_b / (tot_ms / 1e3) / 1e9
    total = sum(w[1] for w in kern.values())
    r = {"kernel": {"backward": "logic_backward_kernel", "forward": "logic_forward_kernel",
                    "backward_gather": "logic_backward_gather2_kernel (+ bake_kernel)",
                    "conv_backward": "conv_plane_backward_kernel", "conv_forward": "conv_plane_forward_kernel"
                    }.get(dom, dom),
         "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "peak_source": src, "unit": "GB/s",
         "frac": round(achieved / hbm, 4), "traffic": traffic,
         "algorithmic_bytes_per_launch": round(tot_b / n), "launches": n, "avg_ms": round(tot_ms / n, 4),
         "shares": {k: round(v[1] / total, 3) for k, v in kern.items()}}
    if tot_l2 and dev is not None:
        pk = l2_peaks(dev)
        key = "gather_reduce" if dom in ("backward", "conv_backward") else "gather"
        l2 = tot_l2 / (tot_ms / 1e3) / 1e9
        r["l2"] = {"achieved": round(l2, 1), "peak": pk[key], "unit": "GB/s", "frac": round(l2 / pk[key], 4),
                   "bytes_per_launch": round(tot_l2 / n),
                   "peak_source": f"clb_l2_probe mode {'1 (row gathers + row reductions)' if key == 'gather_reduce' else '0 (row gathers)'}, this run",
                   "note": ("one read of the other operand's row and one of grad_y's per occurrence (used operand) "
                            "and column; no reductions" if dom == "backward_gather" else
                            "one read per used operand and column (+ one reduction with grad_x)") +
                           "; slabs of one 128-column chunk stay in L2"}
    if extra:
        r.update(extra)
    return r


def kernels_json(kern):
    return {k: {"launches": v[0], "ms_total": round(v[1], 3), "gb": round(v[2] / 1e9, 3)} for k, v in kern.items()}


def train_loop(model, params, sync):
    """One step of the reference loop: CE, backward, gradient all-reduce, clip 10, Adam."""
    opt = torch.optim.Adam(params, lr=0.01, fused=True)

    def step(x, y):
        opt.zero_grad(set_to_none=True)
        loss = torch.nn.functional.cross_entropy(model(x), y)
        loss.backward()
        sync.finish()
        torch.nn.utils.clip_grad_norm_(params, 10.0)
        opt.step()
        return loss
    return step


def e2e_of(step, x_host, y_host, dev, steps, unit_count):
    """The same step fed from pinned host memory each time, loss read back to pinned host memory."""
    xp, yp = x_host.pin_memory(), y_host.pin_memory()
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()

    def e2e():
        if hasattr(step, "graph"):  # captured step: the pinned inputs land directly in its static buffers
            loss = step(xp, yp)
        else:
            loss = step(xp.to(dev, non_blocking=True), yp.to(dev, non_blocking=True))
        loss_host.copy_(loss.detach(), non_blocking=True)
    ms = timed(e2e, steps, 2, dev)
    return ms, {"value": round(unit_count / (ms / 1e3), 1), "unit": "samples/s",
                "h2d_bytes_per_step": x_host.numel() * x_host.element_size() + y_host.numel() * y_host.element_size(),
                "d2h_bytes_per_step": 4}


def replica_checksum(params, dev):
    """All ranks' parameters must stay bitwise identical under data parallelism: the max and min over
    ranks of a float64 checksum of every parameter's bytes."""
    s = torch.zeros(2, dtype=torch.float64, device=dev)
    for p in params:
        v = p.detach().reshape(-1).view(torch.int32).to(torch.float64)
        s[0] += (v * torch.arange(1, v.numel() + 1, device=dev, dtype=torch.float64).remainder(9973)).sum()
    s[1] = -s[0]
    if dist.is_initialized():
        dist.all_reduce(s, op=dist.ReduceOp.MAX)
    return bool(s[0].item() == -s[1].item())


def load_ref(name):
    """The reference's own extension module, built unmodified for sm_100 into oracle/_ref (test oracle and
    GPU comparison only, never on the product path)."""
    import importlib.util
    path = os.path.join(ROOT, "oracle", "_ref", name + ".so")
    if not os.path.exists(path):
        return None
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def ref_dense_fn(ref):
    class RefFn(torch.autograd.Function):
        """compactlogic.py:474-508 around the reference kernels."""

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
    return RefFn


def ref_dense_layer(RefFn, m, h):
    """LogicLayer.forward_cuda (compactlogic.py:83-118) on the reference kernels: h [batch, in]."""
    xt = h.transpose(0, 1).contiguous()
    w = torch.nn.functional.softmax(m.weights, dim=-1).to(xt.dtype)
    return RefFn.apply(xt, m.indices[0], m.indices[1], w, m.gate_sequence, m.given_x_indices_of_y_start,
                       m.given_x_indices_of_y, m.given_x_indices_of_gate).transpose(0, 1)


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


def bench_c2(args, dev, rank, world, strong=False):
    from compactlogic_b200.parallel import GradAllReduce
    width = args.parallel == "width"
    model = build_c2(dev)
    if width:
        # neuron-parallel: every rank runs the whole batch on its share of each layer's neurons
        from compactlogic_b200.sharded import shard_width
        model = shard_width(model)
    params = [p for p in model.parameters() if p.requires_grad]
    opt = torch.optim.Adam(params, lr=0.01, fused=True)
    strong = strong and not width
    # per-layer buckets overlap a long backward (1024 per GPU); one flat bucket after a short one (strong
    # scaling at 1024/N per GPU, see GradAllReduce)
    sync = None if width else GradAllReduce(params, bucket=os.environ.get("CLB_DP_BUCKET",
                                                                          "flat" if strong and world > 2 else "layer"))
    B = C2["batch"] // world if strong else C2["batch"]
    x_host, y_host = c2_inputs(1000 + (0 if width else rank), B)
    x_dev, y_dev = x_host.to(dev), y_host.to(dev)
    tail = {"n": 0, "ms": 0.0}

    def step(x, y):
        opt.zero_grad(set_to_none=True)
        loss = torch.nn.functional.cross_entropy(model(x), y)
        loss.backward()
        if sync is not None:
            if world > 1 and args.measure_tail:
                # time from the end of the last backward kernel to the last gradient bucket's arrival:
                # the part of the all-reduce that no backward work overlaps
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                sync.finish()
                e.record()
                tail.setdefault("ev", []).append((s, e))
            else:
                sync.finish()
            torch.nn.utils.clip_grad_norm_(params, 10.0)
        else:
            clip_sharded(params, 10.0)
        opt.step()
        return loss

    with Clocks(dev.index) as clk:
        ms, kern, launches = timed_kernels(lambda: step(x_dev, y_dev), args.steps, args.warmup, dev)
    evs = tail.pop("ev", [])
    ms_e2e, e2e = e2e_of(step, x_host, y_host, dev, args.steps, B if width else B * world)
    hbm, src = peaks()
    full = C2["layers"] == 6 and B == 1024 and not width
    roof = roofline(kern, hbm, src, {"backward": NCU_TRAFFIC["logic_backward_kernel"],
                                     "backward_gather": NCU_TRAFFIC["logic_backward_gather2_kernel"]} if full else None,
                    dev,
                    {"traffic_note": "ncu dram__bytes_read+write per launch at the c2 shapes, cold cache (profiles/)"})
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
        "kernels": kernels_json(kern),
        "clocks": clk.summary(),
        "e2e": e2e,
        "gpu_launches": launches,
    }
    if world == 1 and not width and full and not args.no_sub:
        res["with_resampler"] = bench_c2_resampler(args, dev, model, params, step, x_dev, y_dev, ms)
    if world > 1 and not width:
        res["replicas_identical"] = replica_checksum(params, dev)
        if evs:
            torch.cuda.synchronize(dev)
            t = statistics.median(s.elapsed_time(e) for s, e in evs)
            res["limiter"] = {"allreduce_tail_ms": round(t, 4), "share_of_step": round(t / ms, 4),
                              "bucket": sync.bucket,
                              "what": ("wait for the last per-layer gradient bucket after the last backward kernel "
                                       "(the first layer's bucket has no backward work left to overlap)")
                              if sync.bucket == "layer" else
                              "one all-reduce of all gate-logit gradients (24.6 MB) after the backward"}
    return res, model


def bench_c2_resampler(args, dev, model, params, step, x_dev, y_dev, ms_plain):
    """The c2 step followed by EntropyRowResampler.step (compactlogic.py:1113-1150) every iteration, in a
    stress setting where every row of every layer counts as converged after 2 steps (eps 1, patience 2):
    the device monitor, one host read per step, then per layer one resampling kernel and a device sort of
    the inverse index.  With the reference's default patience (200) nothing would be resampled inside a
    short timed window and only the monitor would run."""
    import compactlogic_b200 as cl
    opt_state = {}

    class _Opt:  # the resampler only reads optimizer.state; Adam moments live in the step's optimizer
        state = opt_state
    rs = cl.EntropyRowResampler([m for m in model if hasattr(m, "indices")], ema_decay=0.99, eps=1.0, patience=2,
                                threshold_high=0.95, threshold_low=0.2)
    it = [0]

    def stepr():
        step(x_dev, y_dev)
        rs.step(it[0], _Opt)
        it[0] += 1
    ms = timed(stepr, args.steps, args.warmup, dev)
    return {"ms_per_step": round(ms, 4), "value": round(C2["batch"] / (ms / 1e3), 1), "unit": "samples/s",
            "overhead_vs_plain": round(ms / ms_plain - 1, 4),
            "setting": "EntropyRowResampler(eps=1, patience=2, threshold_low=0.2, threshold_high=0.95): every row "
                       "is picked each step after the second; weak/strong rows rewritten on the device"}


def bench_c2_reference_kernels(args, dev):
    """The same c2 step driven through the reference's own CUDA kernels (oracle/_ref, built unmodified
    for sm_100) with the reference's Python around them: softmax in torch (compactlogic.py:108), the
    three kernels through the autograd bridge (compactlogic.py:474-508), GroupSum in torch
    (compactlogic.py:460-465).  Reported beside the native step; not part of the product."""
    ref = load_ref("difflogic_cuda")
    if ref is None:
        return {"unavailable": "oracle/_ref/difflogic_cuda.so not built (needs the reference tree at build time)"}
    RefFn = ref_dense_fn(ref)
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
            h = ref_dense_layer(RefFn, m, h)
        logits = h.reshape(h.shape[0], C2["k"], -1).sum(-1) / C2["tau"]
        loss = torch.nn.functional.cross_entropy(logits, y_dev)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(params, 10.0)
        opt.step()

    steps = max(2, args.steps // 3)
    ms = timed(step, steps, 2, dev)
    return {"value": round(C2["batch"] / (ms / 1e3), 1), "unit": "samples/s", "ms_per_step": round(ms, 3),
            "steps": steps, "what": "same c2 step on the reference CUDA kernels compiled for sm_100"}


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

    b, dt = _sized(run, budget_s, steps, 4, 1024)
    return {"value": round(b / dt, 3), "unit": "samples/s", "cores": O.THREADS, "kind": "port",
            "sample": f"one c2 training step (fwd+bwd of 6 layers, no optimizer) on a sub-batch of {b} samples, "
                      f"{dt:.1f} s"}


def _sized(run, budget_s, steps, b0, bmax):
    """Time run(b) on a sub-batch sized for about budget_s seconds (multiple of 4); returns (b, s/run)."""
    t = time.perf_counter()
    run(b0)
    t0 = time.perf_counter() - t
    b = int(max(b0, min(bmax, b0 * budget_s / max(t0, 1e-3))))
    b = max(4, (b // 4) * 4)
    t = time.perf_counter()
    for _ in range(steps):
        run(b)
    return b, (time.perf_counter() - t) / steps


# ------------------------------------------------------------------------------------------------
# c1: one LogicLayer forward + backward
# ------------------------------------------------------------------------------------------------
def build_c1(dev):
    import compactlogic_b200 as cl
    torch.manual_seed(0)
    return cl.LogicLayer(C1["in_dim"], C1["out"], num_gates=C1["K"]).to(dev)


def c1_inputs(batch):
    g = torch.Generator().manual_seed(0)
    p = torch.rand(C1["in_dim"], generator=g) * 0.8 + 0.1
    x = (torch.rand(batch, C1["in_dim"], generator=g) < p).float()
    gy = torch.randn(batch, C1["out"], generator=g)
    return x, gy


def bench_c1(args, dev):
    layer = build_c1(dev)
    B = C1["batch"]
    x_host, gy_host = c1_inputs(B)
    x_dev, gy_dev = x_host.to(dev), gy_host.to(dev)

    def step(x, gy):
        layer.weights.grad = None
        xr = x.requires_grad_(True)
        layer(xr).backward(gy)
        return xr.grad

    # per-kernel event times from an eager pass (the roofline), the value from the CUDA-graph replay
    ms_eager, kern, launches = timed_kernels(lambda: step(x_dev.detach(), gy_dev), args.steps * 5, args.warmup, dev)
    from compactlogic_b200.graph import GraphedLayerPass
    graphed = GraphedLayerPass(layer, x_dev, gy_dev)
    with Clocks(dev.index) as clk:
        ms = timed(graphed, args.steps * 20, args.warmup, dev)
    xp, gp = x_host.pin_memory(), gy_host.pin_memory()
    gw_host = torch.empty(C1["out"], C1["K"]).pin_memory()

    def e2e():
        gw_host.copy_(graphed(xp.to(dev, non_blocking=True), gp.to(dev, non_blocking=True))[1], non_blocking=True)
    ms_e2e = timed(e2e, args.steps * 20, 2, dev)
    hbm, src = peaks()
    e, K, I, O_ = 4, C1["K"], C1["in_dim"], C1["out"]
    step_bytes = e * B * (I + O_) + O_ * K * 13 + e * B * (2 * I + O_) + O_ * K * 13
    res = {"metric": "train_samples_per_s", "value": round(B / (ms / 1e3), 1), "unit": "samples/s",
           "ms_per_step": round(ms, 4), "steps": args.steps * 20, "dtype": "f32",
           "eager_ms_per_step": round(ms_eager, 4),
           "config": {"workload": "c1: LogicLayer(784, 12000, K=16) forward + backward (grad_x, grad_logits), "
                                  "batch 256, upstream grad N(0,1)", "l2": "working set < L2 (small layer)",
                      "cuda_graph": "forward + backward captured once and replayed (eager_ms_per_step: the same "
                                    "pass issued op by op; roofline from the eager pass's per-kernel events)"},
           "step_hbm_bytes_algorithmic": step_bytes,
           "step_hbm_frac": round(step_bytes / (ms / 1e3) / 1e9 / hbm, 4),
           "roofline": roofline(kern, hbm, src, None, dev), "kernels": kernels_json(kern), "clocks": clk.summary(),
           "e2e": {"value": round(B / (ms_e2e / 1e3), 1), "unit": "samples/s",
                   "h2d_bytes_per_step": (x_host.numel() + gy_host.numel()) * 4,
                   "d2h_bytes_per_step": gw_host.numel() * 4},
           "gpu_launches": launches}
    if not args.no_refcuda:
        res["reference_cuda_kernels"] = bench_c1_reference(args, dev, layer, x_dev, gy_dev)
    return res, layer


def bench_c1_reference(args, dev, layer, x_dev, gy_dev):
    """The same pass on the reference's kernels: softmax in torch, forward, backward_x over the inverse
    index, backward_w, softmax backward in torch (compactlogic.py:83-118, 474-508)."""
    ref = load_ref("difflogic_cuda")
    if ref is None:
        return {"unavailable": "oracle/_ref/difflogic_cuda.so not built"}
    RefFn = ref_dense_fn(ref)

    def step():
        layer.weights.grad = None
        xr = x_dev.detach().requires_grad_(True)
        ref_dense_layer(RefFn, layer, xr).backward(gy_dev)

    ms = timed(step, args.steps * 2, 2, dev)
    return {"value": round(C1["batch"] / (ms / 1e3), 1), "unit": "samples/s", "ms_per_step": round(ms, 4),
            "what": "same forward + backward on the reference CUDA kernels compiled for sm_100"}


def cpu_baseline_c1(layer, budget_s):
    from oracle import oracle as O
    idx, g = layer.indices.cpu().numpy(), layer.gate_sequence.cpu().numpy()
    p = O.softmax(layer.weights.detach().cpu().numpy().astype(np.float64))

    def run(b):
        x, gy = c1_inputs(b)
        xr, gyr = x.numpy().T.astype(np.float64), gy.numpy().T.astype(np.float64)
        O.dense_forward(xr, idx[0], idx[1], p, g)
        O.dense_backward_w(xr, idx[0], idx[1], g, gyr)
        O.dense_backward_x(xr, idx[0], idx[1], p, g, gyr)

    b, dt = _sized(run, budget_s, 1, 8, 256)
    return {"value": round(b / dt, 3), "unit": "samples/s", "cores": O.THREADS, "kind": "port",
            "sample": f"c1 forward + backward_w + backward_x on {b} samples, {dt:.2f} s"}


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
        l2note = "conv activations 18.9 / 33.6 MB (L2-resident), dense layer output 262 MB > L2 (no flush)"
    else:
        model, (x_host, y_host), B, dtype = build_c5(dev), c5_inputs(1000 + rank, C5["batch"]), C5["batch"], "bf16"
        desc = "c5: 3072 -> 4x LogicLayer(1e6, K=4, gate ids U{0..15}) -> GroupSum(100, 30); bf16 activations"
        l2note = "per-layer activations 1.02 GB > L2 126 MB (no flush)"
    params = [p for p in model.parameters() if p.requires_grad]
    sync = GradAllReduce(params)
    x_dev, y_dev = x_host.to(dev), y_host.to(dev)
    steps = args.steps if workload == "c3" else max(3, args.steps // 2)
    graph = workload == "c3" and world == 1 and not args.no_graph
    extra = {}
    if graph:
        # c3 is host-bound op by op (~20 short kernels): per-kernel event times from an eager pass for the
        # roofline, the value from the step captured in a CUDA graph
        from compactlogic_b200.graph import GraphedTrainStep
        ms_eager, kern, launches = timed_kernels(lambda: train_loop(model, params, sync)(x_dev, y_dev), 1, 1, dev)
        opt = torch.optim.Adam(params, lr=0.01, fused=True, capturable=True)
        gstep = GraphedTrainStep(model, opt, torch.nn.functional.cross_entropy, x_dev, y_dev, clip=10.0, params=params)
        step = gstep
        eager = train_loop(model, params, sync)
        ms_eager = timed(lambda: eager(x_dev, y_dev), steps, args.warmup, dev)
        with Clocks(dev.index) as clk:
            ms = timed(lambda: gstep(), steps * 3, args.warmup, dev)
        extra = {"eager_ms_per_step": round(ms_eager, 4),
                 "cuda_graph": "the whole step (forward, CE, backward, clip, Adam) captured once and replayed; "
                               "eager_ms_per_step: the same step issued op by op"}
    else:
        step = train_loop(model, params, sync)
        with Clocks(dev.index) as clk:
            ms, kern, launches = timed_kernels(lambda: step(x_dev, y_dev), steps, args.warmup, dev)
    _, e2e = e2e_of(step, x_host, y_host, dev, steps, world * B)
    hbm, src = peaks()
    res = {"metric": "train_samples_per_s", "value": round(world * B / (ms / 1e3), 1), "unit": "samples/s",
           "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype, "data": "synthetic",
           "config": {"workload": desc, "batch_per_gpu": B, "global_batch": B * world, "parallelism": f"dp{world}",
                      "l2": l2note, **({"cuda_graph": extra.pop("cuda_graph")} if "cuda_graph" in extra else {})},
           **extra,
           "roofline": roofline(kern, hbm, src, None, dev), "kernels": kernels_json(kern),
           "clocks": clk.summary(), "e2e": e2e, "gpu_launches": launches}
    if world > 1:
        res["replicas_identical"] = replica_checksum(params, dev)
    return res, model


def bench_c3_reference(args, dev):
    """The c3 step on the reference's own conv and dense kernels through its autograd bridges
    (compactlogic.py:598-626, 838-867, 83-118, 474-508), GroupSum in torch."""
    dl, cv = load_ref("difflogic_cuda"), load_ref("convlogic_cuda")
    if dl is None or cv is None:
        return {"unavailable": "oracle/_ref reference extensions not built"}
    RefFn = ref_dense_fn(dl)

    class RefConv(torch.autograd.Function):
        @staticmethod
        def forward(ctx, x, och, oh, ow, w, g, stride, pad, ks):
            ctx.save_for_backward(x, och, oh, ow, w, g)
            ctx.stride, ctx.pad = stride, pad
            return cv.forward(x, och, oh, ow, w, g, stride, pad, ks)

        @staticmethod
        def backward(ctx, gy):
            x, och, oh, ow, w, g = ctx.saved_tensors
            gy = gy.contiguous()
            gx = cv.backward_x(x, och, oh, ow, w, g, gy, ctx.stride, ctx.pad) if ctx.needs_input_grad[0] else None
            gw = cv.backward_w(x, och, oh, ow, g, gy, ctx.stride) if ctx.needs_input_grad[4] else None
            return gx, None, None, None, gw, None, None, None, None

    model = build_c3(dev)
    conv1, conv2, _, dense = list(model)[:4]
    params = [conv1.weights, conv2.weights, dense.weights]
    opt = torch.optim.Adam(params, lr=0.01, fused=True)
    x_host, y_host = c3_inputs(1000, C3["batch"])
    x_dev, y_dev = x_host.to(dev), y_host.to(dev)

    def conv(m, x):
        w = torch.nn.functional.softmax(m.weights, dim=-1).to(x.dtype)
        return RefConv.apply(x.contiguous(), m.offsets_ch, m.offsets_h, m.offsets_w, w, m.gate_sequence, m.stride,
                             m.padding, m.ks)

    def step():
        opt.zero_grad(set_to_none=True)
        h = conv(conv2, conv(conv1, x_dev)).reshape(C3["batch"], -1)
        h = ref_dense_layer(RefFn, dense, h)
        logits = h.reshape(h.shape[0], C3["k"], -1).sum(-1) / C3["tau"]
        torch.nn.functional.cross_entropy(logits, y_dev).backward()
        torch.nn.utils.clip_grad_norm_(params, 10.0)
        opt.step()

    steps = max(2, args.steps // 3)
    ms = timed(step, steps, 2, dev)
    return {"value": round(C3["batch"] / (ms / 1e3), 1), "unit": "samples/s", "ms_per_step": round(ms, 3),
            "steps": steps, "what": "same c3 step on the reference CUDA kernels compiled for sm_100"}


def cpu_baseline_c3(model, budget_s):
    """The oracle on a sub-batch of the c3 step: both conv layers, the dense layer, GroupSum + CE gradient
    and the full backward (no optimizer)."""
    from oracle import oracle as O
    conv1, conv2, _, dense = list(model)[:4]
    tc = [(m.offsets_ch.cpu().numpy(), m.offsets_h.cpu().numpy(), m.offsets_w.cpu().numpy(),
           m.gate_sequence.cpu().numpy(), O.softmax(m.weights.detach().cpu().numpy().astype(np.float64)))
          for m in (conv1, conv2)]
    di, dg = dense.indices.cpu().numpy(), dense.gate_sequence.cpu().numpy()
    dp = O.softmax(dense.weights.detach().cpu().numpy().astype(np.float64))

    def run(b):
        x, y = c3_inputs(7, b)
        xn = x.numpy().astype(np.float64)
        (o1, h1_, w1_, g1, p1), (o2, h2_, w2_, g2, p2) = tc
        a1 = O.conv_forward(xn, o1, h1_, w1_, p1, g1, 2, 1, 3)
        a2 = O.conv_forward(a1, o2, h2_, w2_, p2, g2, 2, 1, 3)
        hf = a2.reshape(b, -1).T
        y3 = O.dense_forward(hf, di[0], di[1], dp, dg)
        lg = O.group_sum(y3.T, C3["k"], C3["tau"])
        gy = O.group_sum_backward(O.cross_entropy_grad(lg, y.numpy()), C3["dense"], C3["k"], C3["tau"]).T
        O.dense_backward_w(hf, di[0], di[1], dg, gy)
        g2x = O.dense_backward_x(hf, di[0], di[1], dp, dg, gy).T.reshape(a2.shape)
        O.conv_backward_w(a1, o2, h2_, w2_, g2, g2x, 2)
        g1x = O.conv_backward_x(a1, o2, h2_, w2_, p2, g2, g2x, 2)
        O.conv_backward_w(xn, o1, h1_, w1_, g1, g1x, 2)

    b, dt = _sized(run, budget_s, 1, 4, 512)
    return {"value": round(b / dt, 3), "unit": "samples/s", "cores": O.THREADS, "kind": "port",
            "sample": f"one c3 training step (no optimizer) on a sub-batch of {b} samples, {dt:.1f} s"}


def cpu_baseline_c5(model, budget_s):
    from oracle import oracle as O
    layers = [m for m in model if hasattr(m, "indices")]
    tabs = [(m.indices.cpu().numpy(), m.gate_sequence.cpu().numpy(),
             O.softmax(m.weights.detach().cpu().numpy().astype(np.float64))) for m in layers]

    def run(b):
        x, y = c5_inputs(7, b)
        h = [x.float().numpy().T.astype(np.float64)]
        for idx, g, p in tabs:
            h.append(O.dense_forward(h[-1], idx[0], idx[1], p, g))
        lg = O.group_sum(h[-1].T, C5["k"], C5["tau"])
        gy = O.group_sum_backward(O.cross_entropy_grad(lg, y.numpy()), C5["width"], C5["k"], C5["tau"]).T
        for li in range(len(tabs) - 1, -1, -1):
            idx, g, p = tabs[li]
            O.dense_backward_w(h[li], idx[0], idx[1], g, gy)
            if li > 0:
                gy = O.dense_backward_x(h[li], idx[0], idx[1], p, g, gy)

    b, dt = _sized(run, budget_s, 1, 4, 512)
    return {"value": round(b / dt, 3), "unit": "samples/s", "cores": O.THREADS, "kind": "port",
            "sample": f"one c5 training step (f64, no optimizer) on a sub-batch of {b} samples, {dt:.1f} s"}


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


def c4_words(dev, rank, W):
    """The rank's packed input words: a fixed function of the global word index (seeded per word block), so
    the union over ranks is the same 2^22-sample input whatever N."""
    lo, _ = _c4_shard(rank)
    g = torch.Generator(device=dev).manual_seed(77)
    total = -(-C4["samples"] // 64)
    full = torch.randint(-2**63, 2**63 - 1, (C4["in_dim"], total), dtype=torch.int64, device=dev, generator=g)
    return full[:, lo // 64:lo // 64 + W].contiguous()


def _c4_shard(rank):
    from compactlogic_b200.parallel import shard_range
    world = dist.get_world_size() if dist.is_initialized() else 1
    return shard_range(C4["samples"], rank, world)


def bench_c4(args, dev, rank, world, chunk_words):
    import compactlogic_b200 as cl
    from compactlogic_b200.parallel import gather_counts
    model = build_c4(dev)
    net = cl.PackedLogicNet(model, chunk_words=chunk_words)
    lo, hi = _c4_shard(rank)
    n = hi - lo
    W = -(-n // 64)
    xw = c4_words(dev, rank, W)
    counts = torch.zeros(n, C4["k"], dtype=torch.int32, device=dev)
    out = {}

    def step():  # one pass over the rank's shard, then the all-gather of every rank's counts
        out["all"] = gather_counts(net.counts_packed(xw, n, counts), C4["samples"])
    steps = max(1, args.steps // 2)
    with Clocks(dev.index) as clk:
        ms = timed(step, steps, max(1, args.warmup // 2), dev)
    launches = net.launches_per_pass * steps
    allc = out["all"]
    checksum = int((allc.to(torch.int64) * (torch.arange(allc.shape[0], device=dev).unsqueeze(1) % 1009 + 1)).sum())
    evals = C4["samples"] * C4["width"] * C4["layers"]
    # end to end: packed words from pinned host memory into a fixed device buffer, the gathered counts
    # back to pinned host memory
    xh = xw.cpu().pin_memory()
    ch = torch.empty(allc.shape, dtype=torch.int32).pin_memory()
    x_in = torch.empty_like(xw)

    def e2e():
        x_in.copy_(xh, non_blocking=True)
        ch.copy_(gather_counts(net.counts_packed(x_in, n, counts), C4["samples"]), non_blocking=True)

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
    # roofline of the whole pass (graph-replayed launches) on the byte model
    hbm, src = peaks()
    Wt = -(-C4["samples"] // 64)
    bytes_model = (8 * Wt * (C4["in_dim"] + C4["width"]) + C4["width"] * 9 +
                   (C4["layers"] - 2) * (8 * Wt * 2 * C4["width"] + C4["width"] * 9) +
                   (8 * Wt * C4["width"] + C4["width"] * 9 + 4 * C4["k"] * 64 * Wt))
    per_rank = bytes_model * n / C4["samples"]
    achieved = per_rank / (ms / 1e3) / 1e9
    full = C4["samples"] == 1 << 22 and chunk_words == 128
    return {
        "metric": "packed_infer_gate_evals_per_s", "value": round(evals / (ms / 1e3), 1), "unit": "gate-evals/s",
        "ms_per_step": round(ms, 3), "steps": steps, "dtype": "u64",
        "config": {"workload": "c4: 784 -> 8x256000 frozen -> GroupSum(10), 2^22 samples sharded by sample, "
                               "counts all-gathered inside the timed region",
                   "samples_per_gpu": n, "chunk_words": chunk_words,
                   "l2": "each layer's 128-word chunk output (262 MB) > L2 (no flush)"},
        "roofline": {"kernel": "packed pass (packed_layer_pipe_kernel + count_kernel, graph-replayed)", "bound": "hbm",
                     "achieved": round(achieved, 1), "peak": hbm, "peak_source": src, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4),
                     "traffic": NCU_TRAFFIC["packed_pass"] * n / C4["samples"] if full else None,
                     "algorithmic_bytes_per_pass": round(per_rank),
                     "note": "byte model: every layer's activations make one HBM round trip; traffic = per-launch "
                             "ncu DRAM bytes (profiles/packed_inference_c4.md) summed over the pass's launches"},
        "counts_checksum": checksum,
        "counts_match_single_gpu": (checksum == C4_COUNTS_CHECKSUM) if C4["samples"] == 1 << 22 else None,
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
def free(dev):
    import gc
    gc.collect()
    torch.cuda.empty_cache()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--workload", default="c2", choices=["c1", "c2", "c3", "c4", "c5"])
    ap.add_argument("--no-packed", action="store_true", help="skip the packed-inference (c4) sub-block")
    ap.add_argument("--no-sub", action="store_true", help="skip the c1 / c3 / c5 sub-blocks")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baselines")
    ap.add_argument("--no-refcuda", action="store_true", help="skip the reference-CUDA-kernel timings")
    ap.add_argument("--no-tail", dest="measure_tail", action="store_false",
                    help="do not time the un-overlapped all-reduce tail at N > 1")
    ap.add_argument("--no-graph", action="store_true", help="time c1 / c3 op by op instead of as CUDA graphs")
    ap.add_argument("--chunk-words", type=int, default=128)
    ap.add_argument("--no-prune", action="store_true", help="skip the pruned packed-inference sub-measurement")
    ap.add_argument("--strong", action="store_true",
                    help="headline c2 with the global batch fixed at 1024 (1024/N per GPU)")
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
                "config": {"workload": args.workload, "arm": "CPU oracle (reference kernels restated in C)",
                           "sub_batch": res["sample"], "optimizer": "none",
                           "same_config": False},
                "cpu_baseline": res,
                "e2e": {"value": res["value"], "unit": res["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    cpu = rank == 0 and world == 1 and not args.no_cpu
    cpu_sub = args.cpu_budget / 2

    if args.workload in ("c3", "c5"):
        res, model = bench_train(args, dev, rank, world, args.workload)
        if cpu:
            res["cpu_baseline"] = (cpu_baseline_c3 if args.workload == "c3" else cpu_baseline_c5)(model, cpu_sub)
    elif args.workload == "c1":
        res, layer = bench_c1(args, dev)
        res.update({"n_gpus": 1, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
                    "vs_baseline": None, "data": "synthetic"})
        if cpu:
            res["cpu_baseline"] = cpu_baseline_c1(layer, cpu_sub)
    elif args.workload == "c4":
        res, model = bench_c4(args, dev, rank, world, args.chunk_words)
        if cpu:
            res["cpu_baseline"] = cpu_baseline_c4(model, args.cpu_budget)
        res.update({"n_gpus": world, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
                    "vs_baseline": None, "data": "synthetic"})
    else:
        res, model = bench_c2(args, dev, rank, world, strong=args.strong)
        del model
        free(dev)
        if world > 1 and not args.strong and args.parallel == "dp":
            strong, m = bench_c2(args, dev, rank, world, strong=True)
            for k in ("kernels", "step_hbm_bytes_algorithmic", "gpu_launches"):
                strong.pop(k, None)
            res["strong"] = strong
            del m
            free(dev)
        if not args.no_packed:
            packed, pmodel = bench_c4(args, dev, rank, world, args.chunk_words)
            if cpu:
                packed["cpu_baseline"] = cpu_baseline_c4(pmodel, cpu_sub)
            res["packed"] = packed
            del pmodel
            free(dev)
        if not args.no_sub:
            if world == 1:
                c1, layer = bench_c1(args, dev)
                if cpu:
                    c1["cpu_baseline"] = cpu_baseline_c1(layer, cpu_sub)
                res["c1"] = c1
                del layer
                free(dev)
            for wl in ("c3", "c5"):
                sub, m = bench_train(args, dev, rank, world, wl)
                if cpu:
                    sub["cpu_baseline"] = (cpu_baseline_c3 if wl == "c3" else cpu_baseline_c5)(m, cpu_sub)
                del m
                free(dev)
                if wl == "c3" and world == 1 and not args.no_refcuda:
                    sub["reference_cuda_kernels"] = bench_c3_reference(args, dev)
                    free(dev)
                for k in ("n_gpus", "warmup", "higher_is_better", "vs_baseline", "data"):
                    sub.pop(k, None)
                res[wl] = sub
        if world == 1 and not args.no_refcuda:
            res["reference_cuda_kernels"] = bench_c2_reference_kernels(args, dev)
            free(dev)
        if cpu:
            res["cpu_baseline"] = cpu_baseline_c2(build_c2("cpu"), args.cpu_budget)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
