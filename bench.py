#!/usr/bin/env python
"""Throughput of the b200q quantized DiT-linear hot path on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c5] [--impl b200q|reference]

Prints ONE JSON line (rank 0).  A "step" is one pass of the hot path over one
batch of synthetic input with the shapes of a BASELINE.json config:

  c5 (default)  Wan-14B block, FP8 W8A8: per-tensor e4m3 activation quant + four
                linears (qkv 5120->15360, out 5120->5120, up 5120->13824 + GELU,
                down 13824->5120) over M = 2 x 32760 = 65520 tokens, rows split
                across ranks (no collective; weights replicated).
  c1            INT8 W8A8 single linear 4096x3072 -> 3072 (per-token quant + GEMM).
  c2            FP8 W8A16 linear 3072 -> 12288 + GELU, --m (default 4096).
  c3            FP8 W8A8 scaled_mm 8192x12288 -> 3072.
  c4            Flux double-stream block, INT8 W8A8, M = 9216 (qkv, out, up+GELU, down).

`value` is device time (CUDA events on the launching stream, per step, L2
flushed between steps outside the timed events), max over ranks, whole-job ops/s.
`e2e` is the same metric through the public torch ops with the step's inputs
copied from pinned host memory and its outputs copied back inside the timed
region.  `--impl reference` times the reference's CPU path (the oracle port of
its fallback semantics) on a bounded row sample on rank 0.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024


# ----------------------------------------------------------------------------- setup
def _dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _load_pack():
    import importlib.util
    os.environ.setdefault("B200Q_NO_BOOTSTRAP", "1")
    if "b200q" in sys.modules:
        return sys.modules["b200q"]
    pack = os.path.join(ROOT, "comfyui-applesilicon-optimized_b200")
    spec = importlib.util.spec_from_file_location("b200q", os.path.join(pack, "__init__.py"),
                                                  submodule_search_locations=[pack])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["b200q"] = mod
    spec.loader.exec_module(mod)
    return mod


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16": d["bf16_tflops"],
                "bf16_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


def _split_rows(M, world, rank):
    base, rem = divmod(M, world)
    start = rank * base + min(rank, rem)
    return start, base + (1 if rank < rem else 0)


# ----------------------------------------------------------------------------- workloads
class Layer:
    """One quantized linear: weight codes + scale + bias + epilogue activation."""

    def __init__(self, name, K, N, act=None):
        self.name, self.K, self.N, self.act = name, K, N, act


def _workload_spec(name, m_override=None):
    spec = _base_spec(name)
    if m_override:
        spec["M"] = m_override
    return spec


def _base_spec(name):
    if name == "c5":
        return dict(route="fp8", M=65520, seed=4, hidden=5120, layers=[
            Layer("qkv", 5120, 15360), Layer("out", 5120, 5120),
            Layer("up", 5120, 13824, "gelu_tanh"), Layer("down", 13824, 5120)],
            inputs=["x", "attn", "x"], desc="Wan-14B block FP8 W8A8 (BASELINE config 5)")
    if name == "c4":
        return dict(route="int8", M=9216, seed=3, hidden=3072, layers=[
            Layer("qkv", 3072, 9216), Layer("out", 3072, 3072),
            Layer("up", 3072, 12288, "gelu_tanh"), Layer("down", 12288, 3072)],
            inputs=["x", "attn", "x"], desc="Flux double-stream block INT8 W8A8 (BASELINE config 4)")
    if name == "c1":
        return dict(route="int8", M=4096, seed=0, hidden=3072, outliers=8, recipe="cpu",
                    layers=[Layer("linear", 3072, 3072)],
                    inputs=["x"], desc="INT8 W8A8 single linear (BASELINE config 1)")
    if name == "c3":
        return dict(route="fp8", M=8192, seed=2, hidden=12288, layers=[Layer("down", 12288, 3072)],
                    inputs=["x"], w_std=0.01, x_gelu=True,
                    desc="FP8 W8A8 scaled_mm (BASELINE config 3)")
    if name == "c2":
        return dict(route="w8a16", M=4096, seed=1, hidden=3072,
                    layers=[Layer("up", 3072, 12288, "gelu_tanh")], inputs=["x"],
                    desc="FP8 W8A16 linear (BASELINE config 2)")
    if name == "h3mlp":
        return dict(route="mlp", M=5378, seed=5, hidden=5376, layers=[
            Layer("fc1", 5376, 28672, "swiglu"), Layer("fc2", 14336, 5376)], inputs=["x"],
            desc="MiniMax H3 MLP, INT8: FC1 with SwiGLU in the epilogue -> convrot quant -> FC2 "
                 "(the reference's fc2 SwiGLU fast-path shape [5378,28672]->[5378,5376])")
    raise SystemExit(f"unknown workload {name}")


def _unit(spec):
    return "TOP/s" if spec["route"] in ("int8", "mlp") else "TFLOP/s"


def _flops(spec, M):
    return sum(2.0 * M * l.K * l.N for l in spec["layers"])


class B200Block:
    """Device-resident weights + the step, through the public torch.ops.b200q API.

    Inputs follow BASELINE.json.  Config 1 uses its recipe draw for draw on one
    CPU generator seeded 0: X bf16 [4096, 3072] ~ N(0,1), 8 outlier channels
    torch.randperm(3072)[:8] scaled x20, W = bf16(N(0, 0.02)) quantized per
    output channel (s_w = absmax/127, round-half-even), bias bf16 ~ N(0, 0.01);
    a rank takes its rows [start, start + M) of that X.  The other configs draw
    on a device generator seeded with the config's seed (their sizes make CPU
    generation slow): weights N(0, 0.02) (per-channel int8 or per-tensor e4m3),
    biases N(0, 0.01), activations N(0, 1) per rank shard, 1% outlier channels
    x20 for the INT8 configs.  Config 3 follows its own recipe: weights
    N(0, 0.01) and the activation GELU(N(0,1))."""

    def __init__(self, spec, M, dev, rank, fused=False, start=0):
        self.spec, self.M, self.dev = spec, M, dev
        self.fused = fused  # activation quant inside the GEMM launch (8-bit routes)
        self.amax_epilogue = True  # FP8: amax of a chained layer's input from the GEMM before it
        self.weights = []
        self.inputs = {}
        self.gemm_events = []
        if spec.get("recipe") == "cpu":
            self._init_cpu_recipe(spec, M, dev, start)
            return
        ops = torch.ops.b200q
        g = torch.Generator(device=dev)
        g.manual_seed(spec["seed"])
        for l in spec["layers"]:
            w = torch.randn((l.N, l.K), generator=g, device=dev, dtype=torch.float32) * spec.get("w_std", 0.02)
            b = (torch.randn((l.N,), generator=g, device=dev) * 0.01).to(torch.bfloat16)
            if spec["route"] in ("int8", "mlp"):
                s = (w.abs().amax(dim=1) / 127.0).clamp_min(1e-30)
                q = torch.clamp(torch.round(w / s[:, None]), -128, 127).to(torch.int8)
                self.weights.append((q, s.float().contiguous(), b))
            else:
                q, s = ops.fp8_quant_tensorwise(w.to(torch.bfloat16))
                self.weights.append((q, s.reshape(1), b))
            del w
        # Activations: N(0,1) bf16 per rank shard; 1% outlier channels x20 for INT8 configs.
        gx = torch.Generator(device=dev)
        gx.manual_seed(spec["seed"] * 1000 + 17 + rank)
        for key in sorted(set(spec["inputs"])):
            K0 = spec["layers"][0].K
            x = torch.randn((M, K0), generator=gx, device=dev, dtype=torch.bfloat16)
            if spec.get("x_gelu"):  # config 3: the down-projection's input is GELU(N(0,1))
                x = torch.nn.functional.gelu(x.float()).to(torch.bfloat16)
            if spec["route"] in ("int8", "mlp"):
                n_out = spec.get("outliers", max(1, round(K0 / 100)))
                idx = torch.randperm(K0, generator=gx, device=dev)[:n_out]
                x[:, idx] *= 20
            self.inputs[key] = x

    def _init_cpu_recipe(self, spec, M, dev, start):
        (l,) = spec["layers"]
        g = torch.Generator().manual_seed(spec["seed"])
        x = torch.randn(spec["M"], l.K, generator=g).to(torch.bfloat16)
        idx = torch.randperm(l.K, generator=g)[: spec["outliers"]]
        x[:, idx] *= 20
        w = (torch.randn(l.N, l.K, generator=g) * 0.02).to(torch.bfloat16).float()
        b = (torch.randn(l.N, generator=g) * 0.01).to(torch.bfloat16)
        s = (w.abs().amax(dim=1) / 127.0).clamp_min(1e-30)
        q = torch.clamp(torch.round(w / s[:, None]), -128, 127).to(torch.int8)
        self.weights.append((q.to(dev), s.float().to(dev), b.to(dev)))
        self.inputs["x"] = x[start:start + M].contiguous().to(dev)
        self.outlier_channels = idx

    def step(self, inputs, record=False):
        """Runs the block; returns its outputs.  With record=True, CUDA events
        bracket every GEMM launch (for the per-kernel roofline)."""
        ops = torch.ops.b200q
        spec = self.spec
        outs = []
        h = amax = None
        if spec["route"] == "mlp":
            return self._mlp_step(inputs, record)
        for i, (l, (w, s, b)) in enumerate(zip(spec["layers"], self.weights)):
            x = inputs[spec["inputs"][i]] if i < len(spec["inputs"]) else h
            if spec["route"] == "fp8" and self.fused:
                ev = self._ev(record)
                y = ops.fp8_linear(x, w, s, b, torch.bfloat16, l.act or "none")
                self._ev_end(ev, record, l)
            elif spec["route"] == "fp8":
                xq, xs = (ops.fp8_quant_from_amax(x, amax) if amax is not None
                          else ops.fp8_quant_tensorwise(x))
                ev = self._ev(record)
                if self._feeds_next(i):  # the epilogue takes the next quant's amax
                    y, amax = ops.fp8_scaled_mm_amax(xq, w, xs.reshape(1), s, None, b,
                                                     torch.bfloat16, l.act or "none")
                else:
                    y, amax = ops.fp8_scaled_mm(xq, w, xs.reshape(1), s, None, b, torch.bfloat16,
                                                l.act or "none"), None
                self._ev_end(ev, record, l)
            elif spec["route"] == "int8" and self.fused:
                ev = self._ev(record)
                y = ops.i8_linear(x, w, s, b, torch.bfloat16, l.act or "none")
                self._ev_end(ev, record, l)
            elif spec["route"] == "int8":
                xq, xs = ops.quant_rowwise_i8(x)
                ev = self._ev(record)
                y = ops.i8_matmul_nt_fused_cs(xq, w, xs, s, b, torch.bfloat16, l.act or "none")
                self._ev_end(ev, record, l)
            else:
                ev = self._ev(record)
                y = ops.w8a16_linear(x, w, s, b, l.act or "none")
                self._ev_end(ev, record, l)
            outs.append(y)
            h = y
        return outs

    def _mlp_step(self, inputs, record):
        """FC1 -> SwiGLU -> convrot -> FC2 (the i8_mlp_bridge_prequant route: its two
        launches, FC1 with the SwiGLU epilogue and the convrot quant of act, are
        issued as their ops here so that each GEMM is timed on its own)."""
        ops = torch.ops.b200q
        (l1, l2), ((w1, s1, b1), (w2, s2, b2)) = self.spec["layers"], self.weights
        xq, xs = ops.quant_rowwise_i8(inputs["x"])
        ev = self._ev(record)
        act = ops.i8_matmul_nt_fused_cs_swiglu(xq, w1, xs, s1, b1)
        self._ev_end(ev, record, l1)
        q2, s2a = ops.quant_rowwise_i8_convrot(act, 256)
        ev = self._ev(record)
        y = ops.i8_matmul_nt_fused_cs(q2, w2, s2a, s2, b2, torch.bfloat16)
        self._ev_end(ev, record, l2)
        return [y]

    def _feeds_next(self, i):
        """Separate-quant FP8 route: layer i's output is the next layer's input, so
        its GEMM epilogue also takes that input's amax (the quant skips its amax
        pass; same codes)."""
        spec = self.spec
        return (spec["route"] == "fp8" and not self.fused and self.amax_epilogue
                and i + 1 < len(spec["layers"]) and i + 1 >= len(spec["inputs"]))

    def build_graphs(self, inputs):
        """Captures every op of one step as its own CUDA graph over static buffers.
        Returns [(graph, gemm_flops)] in execution order (flops 0 for quant ops) and
        the number of b200q kernel launches one step makes."""
        from b200q._patches import _native
        ops = torch.ops.b200q
        spec = self.spec
        pool = torch.cuda.graph_pool_handle()
        seq, h, self.graph_outs = [], None, []
        amax = None
        n0 = _native.launch_count()

        def capture(fn):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=pool):
                out = fn()
            return g, out

        if spec["route"] == "mlp":
            (l1, l2), ((w1, s1, b1), (w2, s2, b2)) = spec["layers"], self.weights
            x = inputs["x"]
            g, (xq, xs) = capture(lambda: ops.quant_rowwise_i8(x))
            seq.append((g, 0.0))
            g, act = capture(lambda: ops.i8_matmul_nt_fused_cs_swiglu(xq, w1, xs, s1, b1))
            seq.append((g, 2.0 * self.M * l1.K * l1.N))
            g, (q2, s2a) = capture(lambda: ops.quant_rowwise_i8_convrot(act, 256))
            seq.append((g, 0.0))
            g, y = capture(lambda: ops.i8_matmul_nt_fused_cs(q2, w2, s2a, s2, b2, torch.bfloat16))
            seq.append((g, 2.0 * self.M * l2.K * l2.N))
            self.graph_outs.append(y)
            return seq, _native.launch_count() - n0
        for i, (l, (w, s, b)) in enumerate(zip(spec["layers"], self.weights)):
            x = inputs[spec["inputs"][i]] if i < len(spec["inputs"]) else h
            flops = 2.0 * self.M * l.K * l.N
            act = l.act or "none"
            if spec["route"] == "fp8" and self.fused:
                g, y = capture(lambda: ops.fp8_linear(x, w, s, b, torch.bfloat16, act))
            elif spec["route"] == "int8" and self.fused:
                g, y = capture(lambda: ops.i8_linear(x, w, s, b, torch.bfloat16, act))
            elif spec["route"] == "fp8":
                if amax is not None:
                    g, (xq, xs) = capture(lambda: ops.fp8_quant_from_amax(x, amax))
                else:
                    g, (xq, xs) = capture(lambda: ops.fp8_quant_tensorwise(x))
                seq.append((g, 0.0))
                if self._feeds_next(i):
                    g, (y, amax) = capture(lambda: ops.fp8_scaled_mm_amax(
                        xq, w, xs.reshape(1), s, None, b, torch.bfloat16, act))
                else:
                    g, y = capture(lambda: ops.fp8_scaled_mm(xq, w, xs.reshape(1), s, None, b,
                                                             torch.bfloat16, act))
                    amax = None
            elif spec["route"] == "int8":
                g, (xq, xs) = capture(lambda: ops.quant_rowwise_i8(x))
                seq.append((g, 0.0))
                g, y = capture(lambda: ops.i8_matmul_nt_fused_cs(xq, w, xs, s, b, torch.bfloat16, act))
            else:
                g, y = capture(lambda: ops.w8a16_linear(x, w, s, b, act))
            seq.append((g, flops))
            self.graph_outs.append(y)
            h = y
        return seq, _native.launch_count() - n0

    def build_step_graph(self, inputs):
        """The whole step (every op, in order) captured as one CUDA graph."""
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step_graph_outs = self.step(inputs)
        return g

    def _ev(self, record):
        if not record:
            return None
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def _ev_end(self, ev, record, layer):
        if not record:
            return
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self.gemm_events.append((ev, e, 2.0 * self.M * layer.K * layer.N))


def w8a16_back_to_back_ms(blk, reps=16, copies=4, iters=10):
    """Average launch time of the small-M W8A16 linear (the HBM-bound case):
    `reps` launches captured back to back in one CUDA graph, cycling through
    `copies` copies of the layer-0 weight (together larger than L2, so every
    launch streams its weight from HBM), one event pair per replay.  A single
    launch between two events would also time the ~6 us event/launch overhead of
    a graph replay, which is larger than the kernel itself at M <= 32."""
    ops = torch.ops.b200q
    l = blk.spec["layers"][0]
    w, s, b = blk.weights[0]
    x = blk.inputs[blk.spec["inputs"][0]]
    act = l.act or "none"
    ws = [w] + [w.clone() for _ in range(copies - 1)]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        ops.w8a16_linear(x, w, s, b, act)
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(reps):
            ops.w8a16_linear(x, ws[i % copies], s, b, act)
    g.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) / reps)
    del g, ws
    return statistics.median(ts)


# ----------------------------------------------------------------------------- vendor
def _time_iso(fn, flush, reps=5):
    """Median of `reps` launches, L2 flushed before each, CUDA events."""
    ts = []
    for _ in range(reps):
        flush.zero_()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    return statistics.median(ts)


def _time_b2b(fn, dev, seconds=0.4):
    """Average launch time of `fn` replayed back to back for about `seconds`
    (10 launches per CUDA graph), with the SM clock sampled meanwhile: the
    power-capped steady state a long step runs in."""
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(10):
            fn()
    g.replay()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    g.replay()
    torch.cuda.synchronize()
    reps = max(3, int(seconds / max(time.perf_counter() - t0, 1e-6)))
    with ClockSampler([dev]) as clk:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
    del g
    c = clk.summary() or {}
    return e0.elapsed_time(e1) / (reps * 10), c.get("sm_mhz")


def vendor_baseline(blk, flush):
    """Each GEMM of the workload, b200q against stock torch on the same device,
    shapes and operands, timed the same two ways (isolated launches with L2
    flushed; back to back for ~0.4 s under the power cap, SM clock sampled):
    torch._scaled_mm (cuBLASLt FP8, per-tensor scales, bf16 bias, bf16 out) for
    the FP8 routes, torch._int_mm (cuBLASLt int8, int32 out, no dequant) for the
    INT8 routes, and for W8A16 the stock route of an e4m3 weight (decode to bf16,
    then F.linear on cuBLAS).  Epilogue activations are left out of both arms;
    the b200q arm runs its GEMM op with the workload's own epilogue otherwise."""
    spec, M, dev = blk.spec, blk.M, blk.dev
    route = spec["route"]
    if route == "mlp":
        return None
    ops = torch.ops.b200q
    per, tot = [], {"ours": [0.0, 0.0], "vendor": [0.0, 0.0]}
    g = torch.Generator(device=dev)
    g.manual_seed(99)
    what = None
    for l, (w, s, b) in zip(spec["layers"], blk.weights):
        x = torch.randn((M, l.K), generator=g, device=dev, dtype=torch.bfloat16)
        try:
            if route == "fp8":
                q, sa = ops.fp8_quant_tensorwise(x)
                sa1 = sa.reshape(1)
                ours = lambda q=q, w=w, sa1=sa1, s=s, b=b: ops.fp8_scaled_mm(
                    q, w, sa1, s, None, b, torch.bfloat16, "none")
                vend = lambda q=q, w=w, sa=sa, sb=s.reshape(()), b=b: torch._scaled_mm(
                    q, w.t(), scale_a=sa, scale_b=sb, bias=b, out_dtype=torch.bfloat16)
                what = "torch._scaled_mm (cuBLASLt FP8)"
            elif route == "int8":
                q, xs = ops.quant_rowwise_i8(x)
                ours = lambda q=q, w=w, xs=xs, s=s, b=b: ops.i8_matmul_nt_fused_cs(
                    q, w, xs, s, b, torch.bfloat16, "none")
                vend = lambda q=q, w=w: torch._int_mm(q, w.t())
                what = "torch._int_mm (cuBLASLt int8, int32 out, no dequant)"
            else:
                ours = lambda x=x, w=w, s=s, b=b: ops.w8a16_linear(x, w, s, b, "none")
                vend = lambda x=x, w=w, b=b: torch.nn.functional.linear(x, w.to(torch.bfloat16), b)
                what = "e4m3 -> bf16 weight decode + F.linear (cuBLAS), per call"
            fl = 2.0 * M * l.K * l.N
            row = {"layer": l.name}
            for name, fn in (("ours", ours), ("vendor", vend)):
                fn()
                torch.cuda.synchronize()
                iso = _time_iso(fn, flush)
                b2b, mhz = _time_b2b(fn, dev)
                row[name] = {"iso_tflops": round(fl / iso / 1e9, 1),
                             "b2b_tflops": round(fl / b2b / 1e9, 1), "b2b_sm_mhz": mhz,
                             "b2b_tflops_per_ghz": round(fl / b2b / 1e9 / (mhz / 1e3), 1)
                             if mhz else None}
                tot[name][0] += fl
                tot[name][1] += b2b
            per.append(row)
        except Exception as e:  # a stock kernel missing for this shape/type
            per.append({"layer": l.name, "error": repr(e)[:200]})
        del x
    torch.cuda.synchronize()
    out = {"what": what, "unit": _unit(spec), "per_layer": per,
           "timing": "per layer, both arms alike: iso = median of 5 launches, L2 flushed before "
                     "each; b2b = 10-launch CUDA graph replayed ~0.4 s, NVML SM clock median"}
    if tot["vendor"][1]:
        out["value"] = round(tot["vendor"][0] / tot["vendor"][1] / 1e9, 1)
        out["ours_same_timing"] = round(tot["ours"][0] / tot["ours"][1] / 1e9, 1)
    return out


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock, power and clock-event reasons of the given CUDA devices, sampled
    every 5 ms by a thread through NVML (read-only queries) while the context is
    open; nvidia-smi polling (50 ms) when NVML is unavailable.  Devices are
    matched to NVML handles by UUID, so CUDA_VISIBLE_DEVICES remapping is
    honoured."""
    REASONS = (("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20),
               ("hw_thermal_slowdown", 0x40), ("hw_power_brake_slowdown", 0x80),
               ("sw_power_cap", 0x4))
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, cuda_devices, period_s=0.005):
        self.devices, self.period = list(cuda_devices), period_s
        self.samples, self.proc, self.thread, self.out = [], None, None, ""

    def _nvml_handles(self):
        import pynvml
        pynvml.nvmlInit()
        hs = []
        for d in self.devices:
            uuid = str(torch.cuda.get_device_properties(d).uuid)
            uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            hs.append(pynvml.nvmlDeviceGetHandleByUUID(uuid))
        return pynvml, hs

    def __enter__(self):
        if not self.devices:
            return self
        try:
            nv, hs = self._nvml_handles()
            import threading
            self._stop = threading.Event()

            def run():
                while not self._stop.is_set():
                    for h in hs:
                        try:
                            self.samples.append((
                                nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM),
                                nv.nvmlDeviceGetCurrentClocksEventReasons(h),
                                nv.nvmlDeviceGetPowerUsage(h) / 1000.0))
                        except Exception:
                            pass
                    self._stop.wait(self.period)

            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
        except Exception:
            self.thread = None
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                     "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except Exception:
                self.proc = None
        return self

    def __exit__(self, *a):
        if self.thread is not None:
            self._stop.set()
            self.thread.join(timeout=5)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons, power = [], None, set(), []
        for clk, cmax, bits, watts in self.samples:
            sm.append(float(clk))
            mx = float(cmax)
            power.append(watts)
            for name, bit in self.REASONS:
                if bits & bit:
                    reasons.add(name)
        for line in (self.out or "").splitlines():  # nvidia-smi fallback
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                             "sw_power_cap"], f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        out = {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
               "samples": len(sm), "source": "nvml 5 ms" if self.samples else "nvidia-smi 50 ms"}
        if power:
            out["power_w_max"] = round(max(power), 1)
        return out


# ----------------------------------------------------------------------------- b200q arm
def e2e_pipelined(blk, host_in, host_out, steps, dev):
    """End-to-end steps through the public ops with the PCIe copies overlapped
    the way a serving loop would: step i+1's inputs go host -> device on one
    stream while step i computes and step i-1's outputs go device -> host on a
    third (PCIe is full duplex).  Every step still copies all its inputs in and
    all its outputs out; returns the elapsed ms of all steps (CUDA events on the
    compute stream, which waits for the last copy-out)."""
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    s_in.wait_stream(comp)
    s_out.wait_stream(comp)
    def stage():
        with torch.cuda.stream(s_in):
            dev_in = {k: v.to(dev, non_blocking=True) for k, v in host_in.items()}
            ready = torch.cuda.Event()
            ready.record(s_in)
        return dev_in, ready

    staged = [stage() for _ in range(min(2, steps))]  # inputs at most two steps ahead
    done_out = None
    for i in range(steps):
        dev_in, ready = staged.pop(0)
        if i + 2 < steps:
            staged.append(stage())
        comp.wait_event(ready)
        for t in dev_in.values():
            t.record_stream(comp)
        outs = blk.step(dev_in)
        fin = torch.cuda.Event()
        fin.record(comp)
        s_out.wait_event(fin)
        with torch.cuda.stream(s_out):
            for ho, o in zip(host_out, outs):
                o.record_stream(s_out)
                ho.copy_(o, non_blocking=True)
            done_out = torch.cuda.Event()
            done_out.record(s_out)
        del outs, dev_in
    comp.wait_event(done_out)
    e1.record(comp)
    e1.synchronize()
    return e0.elapsed_time(e1)


def run_b200q(args):
    world, rank, local = _dist_env()
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    _load_pack()
    from b200q._patches import _native
    if not _native.available():
        raise SystemExit("b200q library not built or device is not a B200")

    spec = _workload_spec(args.workload, args.m)
    start, M = _split_rows(spec["M"], world, rank)
    blk = B200Block(spec, M, dev, rank, fused=args.prologue == "fused", start=start)
    blk.amax_epilogue = args.amax_epilogue
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()

    for _ in range(args.warmup):
        blk.step(blk.inputs)
    barrier()
    graphs = step_graph = None
    if args.launch == "graph":
        graphs, launches_per_step = blk.build_graphs(blk.inputs)
        for g, _ in graphs:  # one untimed replay after capture
            g.replay()
        step_graph = blk.build_step_graph(blk.inputs)
        step_graph.replay()
        barrier()

    # ---- device-resident timing, L2 flushed between steps (outside the events).
    # value: one event pair per step around the whole step (with graphs: the step
    # replayed as one CUDA graph).  roofline: event pairs around each GEMM launch
    # (with graphs: each op replayed as its own graph), in a second timed loop.
    launches0 = _native.launch_count()
    step_ms = []
    blk.gemm_events = []
    with ClockSampler([dev]) as clk:
        barrier()
        for _ in range(args.steps):
            flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            if step_graph is None:
                blk.step(blk.inputs, record=True)
            else:
                step_graph.replay()
            e1.record()
            step_ms.append((e0, e1))
        barrier()
        if graphs is not None:
            for _ in range(args.steps):
                flush.zero_()
                for g, fl in graphs:
                    if fl:
                        ea = torch.cuda.Event(enable_timing=True)
                        eb = torch.cuda.Event(enable_timing=True)
                        ea.record()
                        g.replay()
                        eb.record()
                        blk.gemm_events.append((ea, eb, fl))
                    else:
                        g.replay()
            barrier()
        launches = (_native.launch_count() - launches0 if graphs is None
                    else launches_per_step * args.steps)
        b2b_ms = (w8a16_back_to_back_ms(blk) if spec["route"] == "w8a16" and M <= 256
                  and graphs is not None else None)
    t_dev = sum(a.elapsed_time(b) for a, b in step_ms)
    gemm_ms = sum(a.elapsed_time(b) for a, b, _ in blk.gemm_events)
    # stock torch on the same shapes (outside every timed region above)
    vendor = vendor_baseline(blk, flush) if args.vendor and world == 1 else None
    gemm_flops = sum(f for _, _, f in blk.gemm_events)
    n_gemm = len(blk.gemm_events)

    # ---- end-to-end through the public ops: pinned host inputs in, outputs back
    host_in = {k: v.cpu().pin_memory() for k, v in blk.inputs.items()}
    outs_dev = blk.step(blk.inputs)
    host_out = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs_dev]
    del outs_dev
    h2d = sum(t.numel() * t.element_size() for t in host_in.values())
    d2h = sum(t.numel() * t.element_size() for t in host_out)
    e2e_steps = max(1, min(args.steps, 6))
    barrier()
    e2e_pipelined(blk, host_in, host_out, 2, dev)  # untimed: streams, events, first copies
    barrier()
    t_e2e = e2e_pipelined(blk, host_in, host_out, e2e_steps, dev)
    barrier()

    vals = torch.tensor([t_dev, t_e2e, gemm_ms, float(launches)], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
    t_dev, t_e2e, gemm_ms_max, launches_max = vals.tolist()

    total_flops = _flops(spec, spec["M"])  # all ranks together, one step
    value = total_flops * args.steps / (t_dev / 1e3) / 1e12
    e2e = total_flops * e2e_steps / (t_e2e / 1e3) / 1e12
    peaks = _peaks()
    eight_bit = spec["route"] in ("fp8", "int8", "mlp")
    # Each GEMM is timed as its own launch (a few ms), so the burst rate is the
    # denominator; the sustained one is reported beside it.
    peak = (2.0 if eight_bit else 1.0) * peaks["bf16"]
    peak_sus = (2.0 if eight_bit else 1.0) * peaks["bf16_sustained"]
    achieved = gemm_flops / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else None
    # W8A16 with <= 256 tokens is bound by the FP8 weight stream (an HBM
    # roofline), so its roofline is bytes moved per launch / launch time.
    hbm_bound = spec["route"] == "w8a16" and M <= 256
    achieved_gbs, bytes_per_launch = None, 0
    per_launch_event_gbs = None
    if hbm_bound and n_gemm:
        l0 = spec["layers"][0]
        bytes_per_launch = (l0.N * l0.K + M * l0.K * 2 + M * l0.N * 2 + l0.N * 2) * len(spec["layers"])
        per_launch_event_gbs = bytes_per_launch * n_gemm / (gemm_ms / 1e3) / 1e9 / len(spec["layers"]) \
            if gemm_ms > 0 else None
        achieved_gbs = (bytes_per_launch / len(spec["layers"]) / (b2b_ms / 1e3) / 1e9
                        if b2b_ms else per_launch_event_gbs)
    # W8A16 at M <= 256: the roofline is the slower of the weight stream at the
    # HBM rate and the product at the dense bf16 tensor rate (at 3072 x 12288
    # the tensor side takes over above M ~ 140).
    small_bound, small_tflops = "hbm", None
    if hbm_bound and n_gemm:
        l0 = spec["layers"][0]
        t_hbm = bytes_per_launch / len(spec["layers"]) / (peaks["hbm_gbs"] * 1e9)
        t_ten = 2.0 * M * l0.K * l0.N / (peaks["bf16"] * 1e12)
        if t_ten > t_hbm:
            small_bound = "tensor"
            t_call = (b2b_ms / 1e3) if b2b_ms else (gemm_ms / 1e3 / n_gemm)
            small_tflops = 2.0 * M * l0.K * l0.N / t_call / 1e12
    traffic, traffic_src = _committed_traffic(args.workload) if args.m is None else (None, None)

    if rank == 0:
        clocks = clk.summary()
        line = {
            "metric": "INT8/FP8 linear TOPS and % of tensor-core peak at 1/2/4/8 B200",
            "value": round(value, 2), "unit": _unit(spec),
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_dev / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": {"fp8": "e4m3", "int8": "int8", "mlp": "int8", "w8a16": "e4m3xbf16"}[spec["route"]],
            "data": (f"synthetic (seeded {'GELU(N(0,1))' if spec.get('x_gelu') else 'N(0,1)'} "
                     f"activations, N(0,{spec.get('w_std', 0.02)}) weights; BASELINE shapes)"),
            "config": {"workload": f"{args.workload}: {spec['desc']}", "M_total": spec["M"],
                       "M_per_rank": M, "layers": [(l.name, l.K, l.N, l.act) for l in spec["layers"]],
                       "parallelism": f"token-rows split over {world} rank(s), weights replicated, no collective",
                       "l2": "flushed (256 MB write) between timed steps, outside the events",
                       "activation_quant": (
                           "FC1 input: own launch; FC2 input: SwiGLU in FC1's epilogue, then one "
                           "convrot + per-token quant launch" if spec["route"] == "mlp" else
                           {"fused": "inside each GEMM launch (quant prologue; fp8: "
                                     "+1 amax-reduction launch per linear)",
                            "separate": ("own launch(es) before each GEMM" + (
                                "; fp8: a layer fed by the previous layer's output takes that "
                                "output's amax from the previous GEMM's epilogue"
                                if args.amax_epilogue else ""))}[args.prologue]
                           if spec["route"] != "w8a16" else "none (weight-only)"),
                       "launch": ("the step captured once as one CUDA graph, replayed per step (value); "
                                  "each op also captured as its own graph for the per-GEMM events "
                                  "(roofline), timed in a second loop"
                                  if args.launch == "graph" else "eager torch.ops calls")},
            "roofline": ({"bound": small_bound,
                          "achieved": (round(small_tflops, 1) if small_bound == "tensor" else
                                       round(achieved_gbs, 1) if achieved_gbs else None),
                          "peak": peaks["bf16"] if small_bound == "tensor" else peaks["hbm_gbs"],
                          "unit": "TFLOP/s" if small_bound == "tensor" else "GB/s",
                          "frac": (round(small_tflops / peaks["bf16"], 4) if small_bound == "tensor"
                                   else round(achieved_gbs / peaks["hbm_gbs"], 4)
                                   if achieved_gbs else None),
                          "frac_of_hbm": (round(achieved_gbs / peaks["hbm_gbs"], 4)
                                          if achieved_gbs else None),
                          "bound_rule": ("slower of the FP8 weight stream at hbm_gbs and 2*M*K*N "
                                         "at bf16_tflops (burst)"),
                          "traffic": None, "traffic_source": None,
                          "algorithmic_bytes_per_launch": bytes_per_launch // len(spec["layers"]),
                          "kernel": ("x_planes_kernel + w8a16_pgemv_kernel (activation planes on "
                                     "warp-level e4m3 MMAs, one call = both launches)"
                                     if 2 * M <= 8 and os.environ.get("B200Q_W8A16_PGEMV", "1") != "0"
                                     else "w8a16_gemv_kernel" if M <= 16 and spec["layers"][0].K <= 4096 else
                                     "x_planes_kernel + w8a16_planes_kernel (activation planes on "
                                     "kind::f8f6f4, one call = both launches)"),
                          "peak_source": (f"{'bf16_tflops (burst)' if small_bound == 'tensor' else 'hbm_gbs'}"
                                          f" of {peaks['source']} MEASURED_PEAKS.json"),
                          "timing": ("16 calls back to back in one CUDA graph over 4 weight copies "
                                     "(151 MB > L2), events around the replay, median of 10; per call"
                                     if b2b_ms else "CUDA events around each launch"),
                          "us_per_call": round(b2b_ms * 1e3, 2) if b2b_ms else None,
                          "per_launch_event_gbs": (round(per_launch_event_gbs, 1)
                                                   if per_launch_event_gbs else None),
                          "gemm_launches_timed": n_gemm} if hbm_bound else
                         {"bound": "tensor", "achieved": round(achieved, 1) if achieved else None,
                         "peak": round(peak, 1), "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4) if achieved else None,
                         "frac_vs_sustained": round(achieved / peak_sus, 4) if achieved else None,
                         "traffic": traffic, "traffic_source": traffic_src,
                         "algorithmic_flops_per_launch": (round(gemm_flops / n_gemm) if n_gemm else None),
                         "kernel": _gemm_kernel_label(spec, M),
                         "peak_source": (f"{'2 x ' if eight_bit else ''}bf16_tflops (burst) of "
                                         f"{peaks['source']} MEASURED_PEAKS.json"
                                         + (" (dense FP8/INT8 rate = 2 x BF16 on B200)" if eight_bit else "")),
                         "gemm_launches_timed": n_gemm}),
            "e2e": {"value": round(e2e, 3), "unit": _unit(spec),
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                    "steps": e2e_steps},
            "gpu_launches": int(launches_max),
            "clocks": clocks,
        }
        if vendor is not None:
            line["vendor_baseline"] = vendor
        if args.cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(spec, args)
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


NVLINK_GBS = 770.0  # measured peer copy per direction per GPU on this pool's B200s


def run_nsplit(args):
    """--split n: the Wan-shaped block column-parallel.  Every rank holds 1/g of
    each layer's weight rows (its output columns), computes them for all tokens,
    and the GEMM epilogue writes each output block into every rank's full-width
    output (peer mappings over NVLink), so each layer's output is all-gathered
    inside the GEMM.  A one-element NCCL all-reduce orders the ranks where a
    layer reads another's gathered output (down after up) and at the end of the
    step.  The activation quant of each layer input runs on every rank (the
    inputs are replicated)."""
    world, rank, local = _dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import datetime
    pg_kw = dict(timeout=datetime.timedelta(seconds=120), device_id=dev)
    if world == 1:  # not under torchrun: a one-rank group on an in-process store
        pg_kw.update(store=torch.distributed.HashStore(), rank=0, world_size=1)
    torch.distributed.init_process_group("nccl", **pg_kw)
    _load_pack()
    from b200q import nsplit
    from b200q._patches import _native
    if not _native.available():
        raise SystemExit("b200q library not built or device is not a B200")
    if args.workload != "c5":
        raise SystemExit("--split n is the Wan-shaped block's option (--workload c5)")
    spec = _workload_spec(args.workload, args.m)
    M = spec["M"]
    ops = torch.ops.b200q
    blk = B200Block(spec, M, dev, 0)   # full weights and inputs, identical on every rank
    layers = [nsplit.ColumnParallelFP8Linear(w, s, b, l.act)
              for l, (w, s, b) in zip(spec["layers"], blk.weights)]
    blk.weights = []                   # keep only this rank's column blocks
    torch.cuda.empty_cache()
    outs = [nsplit.PeerOutput(M, l.N, torch.bfloat16, dev) for l in spec["layers"]]
    n_in = len(spec["inputs"])
    gemm_events = []

    def step(inputs, record=False):
        h = None
        for i, (l, lay, out) in enumerate(zip(spec["layers"], layers, outs)):
            x = inputs[spec["inputs"][i]] if i < n_in else h
            xq, xs = ops.fp8_quant_tensorwise(x)
            if record:
                ea = torch.cuda.Event(enable_timing=True)
                ea.record()
            lay(xq, xs, out)
            if record:
                eb = torch.cuda.Event(enable_timing=True)
                eb.record()
                gemm_events.append((ea, eb, l, lay.n))
            if i + 1 < len(layers) and i + 1 >= n_in:
                nsplit.stream_barrier(device=dev)   # the next layer reads this gathered output
            h = out.buf
        nsplit.stream_barrier(device=dev)           # next step rewrites every rank's buffers
        return [o.buf for o in outs]

    def barrier():
        torch.cuda.synchronize()
        torch.distributed.barrier()

    for _ in range(args.warmup):
        step(blk.inputs)
    barrier()
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)
    launches0 = _native.launch_count()
    step_ev = []
    with ClockSampler([dev]) as clk:
        barrier()
        for _ in range(args.steps):
            flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            step(blk.inputs, record=True)
            e1.record()
            step_ev.append((e0, e1))
        barrier()
    launches = _native.launch_count() - launches0
    t_dev = sum(a.elapsed_time(b) for a, b in step_ev)
    gemm_ms = sum(a.elapsed_time(b) for a, b, _, _ in gemm_events)
    peaks = _peaks()
    peak = 2.0 * peaks["bf16"]
    # Fused compute + all-gather roofline: per launch the slower of the local
    # GEMM at the tensor peak and the bytes this rank sends over NVLink.
    t_target = 0.0
    nvl_bytes = 0.0
    flops_local = 0.0
    for _, _, l, n in gemm_events:
        f = 2.0 * M * l.K * n
        b = float(M) * n * 2 * (world - 1)
        flops_local += f
        nvl_bytes += b
        t_target += max(f / (peak * 1e12), b / (NVLINK_GBS * 1e9))
    bound = ("nvlink" if nvl_bytes / (NVLINK_GBS * 1e9) > flops_local / (peak * 1e12)
             else "tensor")

    # end to end: inputs from pinned host memory, each rank copies its own
    # column blocks of every output back
    host_in = {k: v.cpu().pin_memory() for k, v in blk.inputs.items()}
    host_out = [torch.empty((M, lay.n), dtype=torch.bfloat16).pin_memory() for lay in layers]
    h2d = sum(t.numel() * t.element_size() for t in host_in.values())
    d2h = sum(t.numel() * t.element_size() for t in host_out)
    e2e_steps = max(1, min(args.steps, 3))
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        dev_in = {k: v.to(dev, non_blocking=True) for k, v in host_in.items()}
        res = step(dev_in)
        for ho, o, lay in zip(host_out, res, layers):
            ho.copy_(o[:, lay.c0:lay.c0 + lay.n], non_blocking=True)
        del dev_in
    e1.record()
    barrier()
    t_e2e = e0.elapsed_time(e1)
    vals = torch.tensor([t_dev, t_e2e, gemm_ms, float(launches), t_target * 1e3], dtype=torch.float64,
                        device=dev)
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
    t_dev, t_e2e, gemm_ms, launches, t_target_ms = vals.tolist()
    total_flops = _flops(spec, M)
    value = total_flops * args.steps / (t_dev / 1e3) / 1e12
    e2e = total_flops * e2e_steps / (t_e2e / 1e3) / 1e12
    # per GPU (this rank's column blocks; the slowest rank's GEMM time)
    achieved = flops_local / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else None
    if rank == 0:
        line = {
            "metric": "INT8/FP8 linear TOPS and % of tensor-core peak at 1/2/4/8 B200",
            "value": round(value, 2), "unit": _unit(spec), "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t_dev / args.steps, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "e4m3",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights; BASELINE shapes)",
            "config": {"workload": f"c5: {spec['desc']}", "M_total": M, "M_per_rank": M,
                       "layers": [(l.name, l.K, l.N, l.act) for l in spec["layers"]],
                       "parallelism": (f"column-parallel N-split over {world} rank(s): weight rows "
                                       "sharded, every layer's output all-gathered inside its "
                                       "GEMM epilogue over NVLink peer mappings"),
                       "l2": "flushed (256 MB write) between timed steps, outside the events",
                       "activation_quant": "own launches before each GEMM, on every rank",
                       "launch": "eager torch.ops calls; NCCL one-element all-reduce as the "
                                 "inter-rank barrier (after up, end of step)"},
            "roofline": {"bound": bound,
                         "achieved": round(achieved, 1) if achieved else None,
                         "peak": round(peak, 1), "unit": "TFLOP/s",
                         "frac": round(t_target_ms / gemm_ms, 4) if gemm_ms > 0 else None,
                         "frac_definition": ("sum over GEMM launches of max(local FLOPs / "
                                             "2 x bf16_tflops, NVLink bytes sent / 770 GB/s) "
                                             "divided by their event-timed duration (max over "
                                             "ranks)"),
                         "nvlink_bytes_per_rank_per_step": nvl_bytes / args.steps,
                         "kernel": "gemm8_tc2_kernel (FP8, TMA-store epilogue to every rank's copy)",
                         "traffic": None, "gemm_launches_timed": len(gemm_events)},
            "e2e": {"value": round(e2e, 3), "unit": _unit(spec),
                    "h2d_bytes_per_step": int(h2d) * world, "d2h_bytes_per_step": int(d2h) * world,
                    "steps": e2e_steps},
            "gpu_launches": int(launches),
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    for o in outs:
        o.close()
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


def _gemm_kernel_label(spec, M):
    """Name of the tile kernel the workload's GEMM launches run (the dispatch of
    csrc/capi.cu gemm8/gemm16: CTA pair for M >= 256 and N > 128)."""
    names = set()
    for l in spec["layers"]:
        if spec["route"] == "w8a16" and M < 128:
            names.add("w8a16_tc_kernel")
            continue
        k = "gemm8_tc2_kernel" if (l.N > 128 and M >= 256) else "gemm8_tc_kernel"
        names.add(k)
    label = " + ".join(sorted(names))
    if spec["route"] == "w8a16":
        label = "e4m3_rows_to16_kernel + " + label + "<kind::f16> (weight decoded once per call)"
    elif spec["route"] == "mlp":
        label += " (FC1: SwiGLU epilogue; FC2: channelwise dequant)"
    elif "gemm8_tc2_kernel" in names:
        label += (" (CTA pair, tcgen05.mma.cta_group::2, kind::f8f6f4)" if spec["route"] == "fp8"
                  else " (CTA pair, tcgen05.mma.cta_group::2, kind::i8)")
    return label


def _committed_traffic(workload):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary
    (profiles/ncu_traffic.json), and where that number comes from."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        t = json.load(open(p)).get(workload)
        return (t["bytes_per_launch"], t["source"]) if t else (None, None)
    except Exception:
        return None, None


# ----------------------------------------------------------------------------- CPU arm
_CPU_CACHE = {}


def _cpu_layers(spec):
    """CPU weights of every layer (made once per process, untimed): int8 codes +
    per-channel scales for the INT8 routes, e4m3 codes + a per-tensor scale for
    the FP8 routes, bf16 bias; same distributions as the GPU arm."""
    key = spec["desc"]
    if key in _CPU_CACHE:
        return _CPU_CACHE[key]
    from oracle import torch_cpu_path as tp
    g = torch.Generator().manual_seed(spec["seed"])
    layers = []
    for l in spec["layers"]:
        w = torch.randn(l.N, l.K, generator=g) * spec.get("w_std", 0.02)
        b = (torch.randn(l.N, generator=g) * 0.01).to(torch.bfloat16)
        if spec["route"] in ("int8", "mlp"):
            s = (w.abs().amax(dim=1) / 127.0).clamp_min(1e-30)
            q = torch.clamp(torch.round(w / s[:, None]), -128, 127).to(torch.int8)
            layers.append((q, s, b))
        else:
            q, s = tp.quantize_fp8_tensorwise(w.to(torch.bfloat16))
            layers.append((q, s, b))
    _CPU_CACHE[key] = layers
    return layers


def _cpu_step(spec, rows, seed=0):
    """One pass of the reference's CPU route over `rows` token rows of every
    layer (torch CPU kernels, oracle/torch_cpu_path.py).  Returns (ops, seconds);
    input generation is outside the timed region, weight decode (part of the
    reference's per-call route) inside it."""
    from oracle import torch_cpu_path as tp
    layers = _cpu_layers(spec)
    g = torch.Generator().manual_seed(1000 + seed)
    x0 = None
    ops = elapsed = 0.0
    h = None
    if spec["route"] == "mlp":
        (l1, l2), ((w1, s1, b1), (w2, s2, b2)) = spec["layers"], layers
        x = torch.randn(rows, l1.K, generator=g).to(torch.bfloat16)
        t = time.perf_counter()
        wide = tp.int8_linear(x, w1, s1, b1)
        gate, up = wide[:, : l1.N // 2], wide[:, l1.N // 2:]
        act = (torch.nn.functional.silu(gate.float()).to(torch.bfloat16) * up)
        grp = act.reshape(rows, -1, 256).float()
        from oracle import oracle
        hmat = torch.from_numpy(oracle.hadamard_convrot(256)).float()
        act = (grp @ hmat).reshape(rows, -1).to(torch.bfloat16)
        tp.int8_linear(act, w2, s2, b2)
        elapsed = time.perf_counter() - t
        return 2.0 * rows * (l1.K * l1.N + l2.K * l2.N), elapsed
    for i, (l, (w, s, b)) in enumerate(zip(spec["layers"], layers)):
        if i < len(spec["inputs"]):
            if x0 is None or spec["inputs"][i] != spec["inputs"][0]:
                x = torch.randn(rows, l.K, generator=g).to(torch.bfloat16)
                if spec.get("x_gelu"):
                    x = torch.nn.functional.gelu(x.float()).to(torch.bfloat16)
                if spec["route"] == "int8":
                    n_out = spec.get("outliers", max(1, round(l.K / 100)))
                    x[:, torch.randperm(l.K, generator=g)[:n_out]] *= 20
                x0 = x0 if x0 is not None else x
            else:
                x = x0
        else:
            x = h
        t = time.perf_counter()
        if spec["route"] == "fp8":
            y = tp.fp8_linear(x, w, s, b, torch.bfloat16, l.act)
        elif spec["route"] == "int8":
            y = tp.int8_linear(x, w, s, b, torch.bfloat16, l.act)
        else:
            y = tp.w8a16_linear(x, w, s, b, l.act)
        elapsed += time.perf_counter() - t
        ops += 2.0 * rows * l.K * l.N
        h = y
    return ops, elapsed


def _cpu_rows(spec, M, target_s, forced=None):
    """Token rows for a bounded CPU sample of about `target_s` seconds (multiple
    of 64, at most the workload's M).  A step costs a fixed part (the per-call
    weight decode) plus a part per row: both are fitted from a 64-row and a
    256-row pass."""
    if forced:
        return min(int(forced), M)
    r0, r1 = min(64, M), min(256, M)
    _cpu_step(spec, r0)  # warm the weights and torch's CPU kernels
    _, t0 = _cpu_step(spec, r0)
    if r1 == r0:
        return r0
    _, t1 = _cpu_step(spec, r1)
    per_row = max((t1 - t0) / (r1 - r0), 1e-7)
    fixed = max(t0 - r0 * per_row, 0.0)
    rows = int((target_s - fixed) / per_row) // 64 * 64
    return max(64, min(rows, M))


def _cpu_sample_text(spec, rows, args):
    what = {"int8": "per-token quant -> torch._int_mm -> chunked fp32 rescale + bias (+ GELU)",
            "fp8": "per-tensor e4m3 quant -> e4m3->bf16 decode of both operands -> bf16 matmul "
                   "-> fp32 scales -> fp32 bias (+ GELU)",
            "w8a16": "e4m3->bf16 weight decode -> F.linear -> scale + bias (+ GELU)",
            "mlp": "INT8 FC1 -> SwiGLU -> convrot -> INT8 FC2 (eager torch)"}[spec["route"]]
    return (f"{rows} of {spec['M']} token rows per step through every layer of {args.workload}; "
            f"the reference's CPU fallback route on torch CPU kernels ({what}; "
            f"oracle/torch_cpu_path.py); weight prep untimed, weight decode timed")


def cpu_baseline(spec, args):
    """The reference's CPU route on a bounded row sample (about 10 s of work)."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rows = _cpu_rows(spec, spec["M"], 5.0, args.cpu_rows)
    ops = t = 0.0
    for rep in range(2):
        o, e = _cpu_step(spec, rows, seed=rep)
        ops, t = ops + o, t + e
    return {"value": round(ops / t / 1e12, 5), "unit": _unit(spec), "cores": threads,
            "kind": "port", "sample": _cpu_sample_text(spec, rows, args) + "; 2 passes"}


def run_reference(args):
    """The reference arm: the reference's CPU route (its kernels are Metal and do
    not build here) on the host cores, rank 0 only; every step is a bounded row
    sample of the workload."""
    world, rank, _ = _dist_env()
    spec = _workload_spec(args.workload, args.m)
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rows = _cpu_rows(spec, spec["M"], args.cpu_step_s, args.cpu_rows)
    for w in range(args.warmup):
        _cpu_step(spec, rows, seed=w)
    ops = t = 0.0
    t0 = time.perf_counter()
    for k in range(args.steps):
        o, e = _cpu_step(spec, rows, seed=100 + k)
        ops, t = ops + o, t + e
    wall = time.perf_counter() - t0
    value = ops / t / 1e12
    line = {
        "metric": "INT8/FP8 linear TOPS and % of tensor-core peak at 1/2/4/8 B200",
        "value": round(value, 5), "unit": _unit(spec),
        "impl": "reference", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t / max(1, args.steps) * 1e3, 2), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": {"fp8": "e4m3", "int8": "int8", "mlp": "int8", "w8a16": "e4m3xbf16"}[spec["route"]],
        "data": "synthetic (seeded; BASELINE shapes, bounded row sample per step)",
        "config": {"workload": f"{args.workload}: {spec['desc']}", "M_total": spec["M"],
                   "sample_rows": rows, "wall_s": round(wall, 2)},
        "cpu_baseline": {"value": round(value, 5), "unit": _unit(spec), "cores": threads,
                         "kind": "port", "sample": _cpu_sample_text(spec, rows, args)},
        "e2e": {"value": round(value, 5), "unit": _unit(spec),
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="c5", choices=["c1", "c2", "c3", "c4", "c5", "h3mlp"])
    ap.add_argument("--m", type=int, default=None, help="override the workload's total token count M")
    ap.add_argument("--launch", default="graph", choices=["graph", "eager"],
                    help="replay per-op CUDA graphs (default) or call the torch ops eagerly")
    ap.add_argument("--prologue", default=None, choices=["fused", "separate"],
                    help="8-bit routes: activation quant in its own launch before each GEMM, or "
                         "inside the GEMM launch (default: fused for c4, which BASELINE defines "
                         "with the quant in each GEMM's prologue and where the two measure level; "
                         "separate elsewhere)")
    ap.add_argument("--split", default="m", choices=["m", "n"],
                    help="multi-GPU layout: token rows (default, no communication) or the "
                         "column-parallel N-split with the all-gather fused into each GEMM "
                         "(config 5 only)")
    ap.add_argument("--no-amax-epilogue", dest="amax_epilogue", action="store_false",
                    help="fp8 separate-quant route: take every layer input's amax with its own "
                         "pass, also where the previous GEMM's epilogue could provide it")
    ap.add_argument("--impl", default="b200q", choices=["b200q", "reference"])
    ap.add_argument("--cpu-rows", type=int, default=None,
                    help="token rows of the CPU sample (default: sized to --cpu-step-s)")
    ap.add_argument("--cpu-step-s", type=float, default=4.0,
                    help="target seconds of CPU work per reference-arm step")
    ap.add_argument("--no-vendor", dest="vendor", action="store_false",
                    help="skip the stock-torch (cuBLASLt) comparison of every layer")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.prologue is None:
        args.prologue = "fused" if args.workload == "c4" else "separate"
    if args.impl == "reference":
        run_reference(args)
    elif args.split == "n":
        run_nsplit(args)
    else:
        run_b200q(args)


if __name__ == "__main__":
    main()
