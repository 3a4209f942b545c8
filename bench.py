#!/usr/bin/env python
"""Benchmark of the int8 quantised-linear path on B200 (one JSON line on rank 0).

Workload: the synthetic 36-layer projection stack, hidden 4096,
intermediate 12288, int8 weight-only, seeded N(0, 0.02) weights quantised by the reference's
per-channel recipe.  One step = one decode step at batch 1 through all 36 layers (every weight of
the stack streamed once, 9.06 GB).  With N GPUs the projections are output-channel sharded; by
default each grouped GEMV stores its output slice into every rank's buffer over NVLink and signals
per-launch arrival counters (peer exchange), --exchange nccl uses NCCL all-gathers instead
(strong scaling: the total work is fixed).

value      weight GB/s of the whole job (stack bytes / max-over-ranks step time), inputs resident,
           one CUDA graph replay per step, CUDA events on the launching stream.
e2e        the same metric through the public API with host buffers: pinned input copied in, the
           captured stack run, the output copied back, every step; beside it (module_api) the same
           step through the drop-in's module calls on host and on device tensors.
roofline   the grouped decode GEMV, which is every launch of the timed step: bytes per launch over
           the average launch time, against the measured HBM copy bandwidth; the fused gate/up
           launch timed alone is reported beside it.
cpu_baseline / --impl reference
           the reference's CPU algorithm (oracle/cpu_port.py) on a bounded sample of the same
           workload on this host's cores (and at the reference's own 4-thread setting).

Flags: --gpus N --steps K --warmup W [--impl reference] [--layers L] [--extra].
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "int8 decode GEMV HBM GB/s and prefill GEMM TFLOPS, % of B200 roofline"
FALLBACK_HBM_GBS = 6650.0


SPEC_HBM_GBS = 8000.0       # B200 HBM3e, nominal
SPEC_F16_TFLOPS = 2250.0    # dense fp16/bf16 tensor, nominal
SPEC_I8_TOPS = 4500.0       # dense int8 tensor, nominal


def peaks() -> dict:
    """Roofline denominators: HBM copy GB/s, and bf16 TFLOPS as a burst (a kernel timed alone) and
    sustained under the power cap (a kernel timed inside a long step)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        burst = float(d["bf16_tflops"])
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": burst,
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", burst)), "source": "measured"}
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled while the timed region runs.

    Every GPU of the host is queried (with its UUID) and only the samples of the GPUs this job
    runs on are kept."""

    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: list[str]):
        self.gpus = {g.strip().lower() for g in gpus}
        self.proc = None

    def __enter__(self):
        if not self.gpus:
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits", "-lms", "10"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            # the timed region starts once nvidia-smi is producing samples (it takes a moment to
            # start; a short timed region would otherwise end before the first sample)
            self.first = self.proc.stdout.readline()
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict:
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9 or f[0].lower() not in self.gpus:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def traffic_per_launch(launches: int, layers: int):
    """DRAM bytes per launch of the grouped decode GEMV, from the committed ncu summary (or None):
    the step's traffic (per layer x layers) over the step's ``launches``.

    profiles/gemv_w8_stack_decode_traffic.md records dram__bytes_read.sum + dram__bytes_write.sum
    summed over every launch of a captured decode step of the stack, per layer.
    """
    p = ROOT / "profiles" / "gemv_w8_stack_decode_traffic.md"
    if not p.exists():
        return None
    vals = {}
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_step_layer:") or line.startswith("launches_per_layer:"):
            k, v = line.split(":", 1)
            vals[k] = float(v)
    if len(vals) < 2:
        return None
    return int(vals["traffic_bytes_per_step_layer:"[:-1]] * layers / launches)


def dist_setup(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit("--gpus %d but WORLD_SIZE=%d" % (args.gpus, world))
    if world > 1:
        import datetime

        # keep stdout to the one JSON line (NCCL prints its version banner there at VERSION level)
        os.environ.setdefault("NCCL_DEBUG", "WARN")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def timed_graph(graph, steps: int, stream) -> float:
    """ms per replay of ``graph`` over ``steps`` replays, CUDA events on ``stream``."""
    import torch

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(steps):
            graph.replay()
        end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / steps


def capture(fn, stream):
    """Capture ``fn`` into a CUDA graph on ``stream``; returns (graph, fn's output)."""
    import torch

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        out = fn()
    return g, out


def reference_arm(args) -> None:
    """--impl reference: the reference algorithm on the host cores (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import cpu_port

    layers = 1
    r = cpu_port.time_stack_decode(layers=layers, warmup=args.warmup, max_steps=args.steps, max_seconds=120.0)
    line = {"metric": METRIC, "impl": "reference", "value": round(r["gbs"], 3), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": r["steps"], "warmup": args.warmup,
            "ms_per_step": round(r["s_per_step"] * 1e3, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8*fp32->fp32", "data": "synthetic",
            "config": {"workload": "cfg4-stack36-decode-b1", "layers_sampled": layers, "batch": 1},
            "cpu_baseline": {"value": round(r["gbs"], 3), "unit": "GB/s", "cores": r["cores"], "kind": "port",
                             "sample": "%d of 36 stack layers per step, batch 1, %d weight bytes per step, "
                                       "%d steps (capped at 120 s)" % (layers, r["bytes"], r["steps"])},
            "e2e": {"value": round(r["gbs"], 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _graph_time(fn, stream, reps: int, warmup: int, per: int = 1) -> float:
    """ms per call of ``fn``: ``per`` calls captured back to back into one CUDA graph, replayed
    ``reps`` times.  A graph replay costs about 2 us of launch overhead on its own, so short calls
    are also timed with several per replay, as they run inside a model's step."""
    import torch

    with torch.cuda.stream(stream):
        fn()
    stream.synchronize()

    def calls():
        for _ in range(per):
            fn()

    g, _ = capture(calls, stream)
    with torch.cuda.stream(stream):  # warm-up replays on the timed stream, finished before timing
        for _ in range(warmup):
            g.replay()
    stream.synchronize()
    ms = timed_graph(g, reps, stream) / per
    del g
    return ms


def kernel_cases(sbq, dev, stream, steps: int, warmup: int,
                 which=("gemv", "mlp", "gemm", "gemm_f32", "gemm_small", "dyn", "lora", "groups")) -> dict:
    """Configurations 0-3 at their own shapes, each kernel timed alone (CUDA graph, CUDA events).

    HBM-bound cases rotate over enough distinct weight copies that every launch reads its weight
    from HBM (the copies together exceed twice the 126 MB L2).
    """
    import torch
    from ctypes import c_void_p as vp

    L = sbq._lib
    W = sbq.workloads
    st = vp(stream.cuda_stream)
    pk = peaks()
    out = {}

    def int8_weights(n, k, copies):
        mods = []
        for c in range(copies):
            q = torch.randint(-127, 128, (n, k), dtype=torch.int8, device=dev)
            packed, rs = sbq.pack_int8(q, rowsum=True)
            mods.append((packed, (torch.rand(n, device=dev) + 0.5) * (1.0 / (127.0 * k ** 0.5)), rs))
        return mods

    if "gemv" in which:  # configuration 0: m=1, k=n=4096
        n = k = W.HIDDEN
        copies = 16
        ws = int8_weights(n, k, copies)
        x = W.activation(1, k, seed=0, device=dev)
        y = torch.empty(1, n, device=dev)

        def f():
            for p_, s_, _ in ws:
                L.call("sbq_gemv_w8", vp(x.data_ptr()), L.F16, k, vp(p_.data_ptr()), vp(s_.data_ptr()), None, 1, n, k,
                       vp(y.data_ptr()), L.F32, n, st)

        ms = _graph_time(f, stream, max(20, steps // 10), warmup) / copies
        b = n * k + 4 * n + 2 * k + 4 * n
        out["cfg0_gemv"] = {"us": round(ms * 1e3, 3), "gbs": round(b / ms / 1e6, 1),
                            "frac_hbm": round(b / ms / 1e6 / pk["hbm_gbs"], 4),
                            "frac_hbm_spec": round(b / ms / 1e6 / SPEC_HBM_GBS, 4), "bytes": b}
        del ws

    if "mlp" in which:  # configuration 1: fused gate/up + down at m in {1, 4, 16}
        k, n = W.HIDDEN, W.INTER
        gs, us_, ds = int8_weights(n, k, 2), int8_weights(n, k, 2), int8_weights(k, n, 2)
        res = {}
        for m in (1, 4, 16):
            x = W.activation(m, k, seed=m, device=dev)
            h = torch.empty(m, n, dtype=torch.float16, device=dev)
            y = torch.empty(m, k, device=dev)

            def f():
                for i in range(2):
                    g, u, d = gs[i], us_[i], ds[i]
                    L.call("sbq_mlp_gateup_w8", vp(x.data_ptr()), L.F16, k, vp(g[0].data_ptr()), vp(g[1].data_ptr()),
                           vp(u[0].data_ptr()), vp(u[1].data_ptr()), m, n, k, vp(h.data_ptr()), L.F16, n, st)
                    L.call("sbq_gemv_w8", vp(h.data_ptr()), L.F16, n, vp(d[0].data_ptr()), vp(d[1].data_ptr()), None,
                           m, k, n, vp(y.data_ptr()), L.F32, k, st)

            ms = _graph_time(f, stream, max(20, steps // 10), warmup) / 2
            b = 3 * n * k + 12 * n + 4 * k + 2 * m * k + 4 * m * n + 4 * m * k
            res[str(m)] = {"us": round(ms * 1e3, 3), "gbs": round(b / ms / 1e6, 1),
                           "frac_hbm": round(b / ms / 1e6 / pk["hbm_gbs"], 4),
                           "frac_hbm_spec": round(b / ms / 1e6 / SPEC_HBM_GBS, 4)}
        out["cfg1_mlp"] = res
        del gs, us_, ds

    if "gemm" in which:  # configuration 2: m=2048, k=4096, n=12288, fp16 out
        m, k, n = 2048, W.HIDDEN, W.INTER
        (p_, s_, _), = int8_weights(n, k, 1)
        x = W.activation(m, k, seed=2, device=dev)
        y = torch.empty(m, n, dtype=torch.float16, device=dev)

        def f():
            L.call("sbq_gemm_w8a16", vp(x.data_ptr()), L.F16, k, vp(p_.data_ptr()), vp(s_.data_ptr()), None, m, n, k,
                   vp(y.data_ptr()), L.F16, n, st)

        ms = _graph_time(f, stream, max(20, steps // 10), warmup)
        fl = 2 * m * n * k
        out["cfg2_prefill_gemm"] = {"us": round(ms * 1e3, 2), "tflops": round(fl / ms / 1e9, 1),
                                    "frac_bf16_peak": round(fl / ms / 1e9 / pk["bf16_tflops"], 4),
                                    "frac_f16_spec": round(fl / ms / 1e9 / SPEC_F16_TFLOPS, 4)}

    if "gemm_small" in which:  # configuration 4 at decode batch 64: the small-batch GEMM per projection
        res = {}
        for name, n, k in (("qkvd", 4 * W.HIDDEN, W.HIDDEN), ("o", W.HIDDEN, W.HIDDEN), ("down", W.HIDDEN, W.INTER)):
            copies = max(2, int(2 * 126e6 / (n * k)) + 1)
            ws = int8_weights(n, k, copies)
            x = W.activation(64, k, seed=4, device=dev)
            y = torch.empty(64, n, dtype=torch.float16, device=dev)

            def f():
                for p_, s_, _ in ws:
                    L.call("sbq_gemm_w8a16", vp(x.data_ptr()), L.F16, k, vp(p_.data_ptr()), vp(s_.data_ptr()), None, 64,
                           n, k, vp(y.data_ptr()), L.F16, n, st)

            ms = _graph_time(f, stream, max(20, steps // 10), warmup) / copies
            b = n * k
            res[name] = {"n": n, "k": k, "us": round(ms * 1e3, 2), "gbs": round(b / ms / 1e6, 1),
                         "frac_hbm": round(b / ms / 1e6 / pk["hbm_gbs"], 4)}
            del ws
        out["cfg4_b64_gemm_small"] = res

    if "gemm_f32" in which:  # configuration 2's shape with the reference's fp32 activations
        m, k, n = 2048, W.HIDDEN, W.INTER
        (p_, s_, _), = int8_weights(n, k, 1)
        x = W.activation(m, k, seed=2, dtype=torch.float32, device=dev)
        y = torch.empty(m, n, device=dev)
        wsb = int(L.load().sbq_linear_w8_workspace_bytes(m, k, L.F32))
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev)

        def f():
            L.call("sbq_linear_w8_ws", vp(x.data_ptr()), L.F32, k, vp(p_.data_ptr()), vp(s_.data_ptr()), None, m, n,
                   k, vp(y.data_ptr()), L.F32, n, vp(ws.data_ptr()), wsb, st)

        ms = _graph_time(f, stream, max(20, steps // 10), warmup)
        fl = 2 * m * n * k
        out["cfg2_prefill_gemm_f32x"] = {"us": round(ms * 1e3, 2), "tflops": round(fl / ms / 1e9, 1),
                                         "frac_bf16_peak": round(fl / ms / 1e9 / pk["bf16_tflops"], 4),
                                         "note": "fp32 x split into bf16 high/low parts (one extra kernel), two "
                                                 "MMAs per k-step; useful FLOPs 2mnk; fp32 out"}

    if "lora" in which:  # the hybrid block's rank-128 LoRA pair (2560 -> 128 -> 4096) at decode
        res = {}
        a = sbq.Int8Linear(W.float_weight(128, 2560, seed=1, device=dev), None, device=dev)
        b = sbq.Int8Linear(W.float_weight(4096, 128, seed=2, device=dev), None, device=dev)
        for m in (1, 16):
            x = W.activation(m, 2560, seed=m, dtype=torch.float32, device=dev)
            y = torch.empty(m, 4096, device=dev)
            t = torch.empty(m, 128, device=dev)

            def fused():
                L.call("sbq_lora_pair_w8", vp(x.data_ptr()), L.F32, 2560, vp(a.packed.data_ptr()),
                       vp(a.scale.data_ptr()), vp(b.packed.data_ptr()), vp(b.scale.data_ptr()), m, 128, 4096, 2560,
                       vp(y.data_ptr()), L.F32, 4096, st)

            def separate():
                L.call("sbq_linear_w8", vp(x.data_ptr()), L.F32, 2560, vp(a.packed.data_ptr()), vp(a.scale.data_ptr()),
                       None, m, 128, 2560, vp(t.data_ptr()), L.F32, 128, st)
                L.call("sbq_linear_w8", vp(t.data_ptr()), L.F32, 128, vp(b.packed.data_ptr()), vp(b.scale.data_ptr()),
                       None, m, 4096, 128, vp(y.data_ptr()), L.F32, 4096, st)

            res[str(m)] = {"fused_us": round(_graph_time(fused, stream, max(20, steps // 10), warmup, per=8) * 1e3, 2),
                           "two_launches_us": round(_graph_time(separate, stream, max(20, steps // 10), warmup, per=8) * 1e3, 2),
                           "calls_per_graph": 8}
        out["lora_pair"] = res

    if "groups" in which:  # a hybrid block's shared-input projections: one launch vs eleven
        from torch import nn
        res = {}
        names = [("sse_q_proj", 4096), ("sse_k_proj", 4096), ("sse_v_proj", 4096), ("lora_q_proj", 128),
                 ("lora_k_proj", 128), ("sse_a_proj", 64), ("sse_b_proj", 64), ("sse_e_proj", 4), ("swa_q_proj", 4096),
                 ("swa_k_proj", 1024), ("swa_v_proj", 1024)]
        blk = nn.Module()
        for i, (nm, n) in enumerate(names):
            setattr(blk, nm, sbq.Int8Linear(W.float_weight(n, 2560, seed=30 + i, device=dev), None, device=dev))
        mods = [getattr(blk, nm) for nm, _ in names]
        group = sbq.groups.SharedInputGroup(mods)
        for m in (1, 512):
            x = W.activation(m, 2560, seed=m, dtype=torch.float32, device=dev)
            outs = [torch.empty(m, mod.out_features, device=dev) for mod in mods]

            def separate():
                with torch.cuda.stream(stream):
                    for mod, o in zip(mods, outs):
                        mod.forward_into(x, o)

            def grouped():
                with torch.cuda.stream(stream):
                    group.forward_all(x)

            res["m%d" % m] = {"grouped_us": round(_graph_time(grouped, stream, max(20, steps // 10), warmup) * 1e3, 2),
                              "separate_us": round(_graph_time(separate, stream, max(20, steps // 10), warmup) * 1e3, 2),
                              "weight_bytes": sum(n * 2560 for _, n in names)}
        out["hybrid_shared_input_group"] = res

    if "dyn" in which:  # configuration 3: int8-dyn, m=512, k=n=4096
        m, k, n = 512, W.HIDDEN, W.HIDDEN
        (p_, s_, rs), = int8_weights(n, k, 1)
        x = W.activation(m, k, seed=3, device=dev)
        y = torch.empty(m, n, device=dev)
        wsb = int(L.load().sbq_dyn_workspace_bytes(m, k, 0))
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev)

        def f():
            L.call("sbq_linear_dyn", vp(x.data_ptr()), L.F16, k, 0, vp(p_.data_ptr()), vp(rs.data_ptr()),
                   vp(s_.data_ptr()), None, m, n, k, vp(y.data_ptr()), n, vp(ws.data_ptr()), wsb, st)

        # eight calls per graph replay (a model step's successive layers); one call per replay beside it
        ms = _graph_time(f, stream, max(20, steps // 10), warmup, per=8)
        ms_one = _graph_time(f, stream, max(20, steps // 10), warmup)
        ops = 2 * m * n * k
        byt = 2 * m * k + n * k + 4 * n + 4 * m * n  # x fp16, W, scales, y fp32
        t_roof = max(byt / (pk["hbm_gbs"] * 1e9), ops / (SPEC_I8_TOPS * 1e12))
        out["cfg3_dyn"] = {"us": round(ms * 1e3, 2), "tops": round(ops / ms / 1e9, 1),
                           "frac_int8_spec_4500": round(ops / ms / 1e9 / SPEC_I8_TOPS, 4),
                           "roofline_us": round(t_roof * 1e6, 2), "frac_roofline": round(t_roof * 1e3 / ms, 4),
                           "calls_per_graph": 8, "us_one_call_per_graph": round(ms_one * 1e3, 2)}
        # the GEMM alone on an already quantised activation (the same launch sbq_linear_dyn chains)
        xq = torch.empty(m, k, dtype=torch.uint8, device=dev)
        sx = torch.empty(1, device=dev)
        zp = torch.empty(1, dtype=torch.int32, device=dev)
        L.call("sbq_quant_act_per_tensor", vp(x.data_ptr()), L.F16, k, m, k, vp(xq.data_ptr()), vp(sx.data_ptr()),
               vp(zp.data_ptr()), vp(ws.data_ptr()), wsb, st)

        def g():
            L.call("sbq_gemm_w8a8", vp(xq.data_ptr()), 0, vp(p_.data_ptr()), vp(rs.data_ptr()), vp(sx.data_ptr()),
                   vp(zp.data_ptr()), vp(s_.data_ptr()), None, m, n, k, vp(y.data_ptr()), n, None, st)

        ms_g = _graph_time(g, stream, max(20, steps // 10), warmup, per=8)
        out["cfg3_dyn"]["gemm_only_us"] = round(ms_g * 1e3, 2)
        out["cfg3_dyn"]["quantise_us"] = round((ms - ms_g) * 1e3, 2)
        # the configuration's own wording: symmetric per-token scales (s8 x s8; the reference's
        # DynamicInt8Linear quantises per tensor, the line above)
        wsb_t = int(L.load().sbq_dyn_workspace_bytes(m, k, L.ACT_PER_TOKEN))
        ws_t = torch.empty(wsb_t, dtype=torch.uint8, device=dev)

        def f_tok():
            L.call("sbq_linear_dyn", vp(x.data_ptr()), L.F16, k, L.ACT_PER_TOKEN, vp(p_.data_ptr()), None,
                   vp(s_.data_ptr()), None, m, n, k, vp(y.data_ptr()), n, vp(ws_t.data_ptr()), wsb_t, st)

        ms_t = _graph_time(f_tok, stream, max(20, steps // 10), warmup, per=8)
        out["cfg3_dyn"]["per_token"] = {"us": round(ms_t * 1e3, 2), "tops": round(ops / ms_t / 1e9, 1),
                                        "frac_roofline": round(t_roof * 1e3 / ms_t, 4), "calls_per_graph": 8}
    return out


def stack_cases(sbq, stack, dev, stream, warmup: int) -> dict:
    """Configuration 4's other points on the same stack: decode at batch 8 and 64, prefill of 8192
    tokens (weight GB/s for decode, TFLOPS for prefill; CUDA graph per step, CUDA events)."""
    import torch

    out = {}
    total = stack.weight_bytes()
    for m in (8, 64):
        x = sbq.workloads.activation(m, stack.hidden, seed=m, device=dev)
        ms = _graph_time(lambda: stack(x), stream, 10, warmup)
        out["decode_b%d" % m] = {"ms": round(ms, 3), "gbs": round(total / ms / 1e6, 1),
                                 "frac_hbm": round(total / ms / 1e6 / peaks()["hbm_gbs"], 4),
                                 "frac_hbm_spec": round(total / ms / 1e6 / SPEC_HBM_GBS, 4)}
    m = 8192
    x = sbq.workloads.activation(m, stack.hidden, seed=m, device=dev)
    with torch.cuda.stream(stream):
        stack(x)  # warm-up (allocator)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        reps = 2
        for _ in range(reps):
            stack(x)
        end.record(stream)
    end.synchronize()
    ms = start.elapsed_time(end) / reps
    fl = 2.0 * m * total
    pk = peaks()
    out["prefill_8192"] = {"ms": round(ms, 2), "tflops": round(fl / ms / 1e9, 1),
                           # a step of ~0.16 s runs under the power cap: the sustained figure applies
                           "frac_bf16_sustained": round(fl / ms / 1e9 / pk["bf16_tflops_sustained"], 4),
                           "frac_bf16_peak": round(fl / ms / 1e9 / pk["bf16_tflops"], 4),
                           "frac_f16_spec": round(fl / ms / 1e9 / SPEC_F16_TFLOPS, 4),
                           "note": "per-projection GEMMs; gate GEMM then up GEMM with the SiLU*mul epilogue"}
    return out


def sharded_prefill_case(sbq, stack, dev, stream, world: int) -> dict:
    """Configuration 4's prefill (8192 tokens, 36 layers) on the output-channel sharded stack: every
    rank runs its shard of each projection's GEMM and NCCL all-gathers assemble the activations.
    CUDA events on the launching stream, max over ranks."""
    import torch
    import torch.distributed as dist

    m = 8192
    x = sbq.workloads.activation(m, stack.hidden, seed=m, device=dev)
    with torch.cuda.stream(stream):
        stack(x)  # warm-up (allocator, communicators)
    stream.synchronize()
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 2
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(reps):
            stack(x)
        end.record(stream)
    end.synchronize()
    t = torch.tensor([start.elapsed_time(end) / reps], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    fl = 2.0 * m * sbq.workloads.stack_bytes(len(stack.layers))
    pk = peaks()
    gathered = 2 * m * (4 * stack.hidden + stack.inter + 2 * stack.hidden + stack.hidden) * len(stack.layers)
    return {"ms": round(ms, 2), "tflops": round(fl / ms / 1e9, 1),
            "frac_bf16_sustained_per_gpu": round(fl / ms / 1e9 / world / pk["bf16_tflops_sustained"], 4),
            "allgather_bytes_per_step": gathered,
            "note": "per-projection GEMMs on each rank's output-channel shard; NCCL all_gather_into_tensor "
                    "after each sharded projection (4 per layer)"}


def module_api_cases(sbq, stack, dev, steps: int, warmup: int) -> dict:
    """The decode step (batch 1) through the drop-in's public module calls, eager (no CUDA graph):
    with host tensors (every projection copies its input in and its output back and waits, the
    path the reference's CPU model loop gets by swapping in the modules) and with device tensors.
    CUDA events on the launching stream around the whole step sequence (host gaps included)."""
    import torch

    total = stack.weight_bytes()
    x_dev = sbq.workloads.activation(1, stack.hidden, seed=5, device=dev)
    out = {}
    for name, x in (("host_tensors", x_dev.cpu()), ("device_tensors", x_dev)):
        for _ in range(warmup):
            stack.forward_modules(x)
        torch.cuda.synchronize()
        st = torch.cuda.current_stream(dev)
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_ev.record(st)
        for _ in range(steps):
            y = stack.forward_modules(x)
        e_ev.record(st)
        e_ev.synchronize()
        ms = s_ev.elapsed_time(e_ev) / steps
        out[name] = {"ms_per_step": round(ms, 3), "gbs": round(total / ms / 1e6, 1),
                     "module_calls_per_step": 4 * len(stack.layers), "launches_per_step": 5 * len(stack.layers)}
        if name == "host_tensors":
            out[name]["h2d_d2h_pairs_per_step"] = 4 * len(stack.layers)
            assert y.device.type == "cpu"
    return out


def load_pack_case(sbq, dev) -> dict:
    """The checkpoint's int8 load on the GPU: every linear weight of SpikingBrain2.0's shapes (539
    weights, 5.17 G parameters, bf16 on the host as the loader reads them) through the streaming
    packer (host -> pinned staging -> device -> quantise + pack), against the reference's 33.2 s
    int8 load (which also reads the shards from storage; the storage read is not included here)."""
    import torch

    shapes = sbq.workloads.checkpoint_linears()
    biggest = max(n * k for _, n, k in shapes)
    g = torch.Generator().manual_seed(7)
    host = (torch.randn(biggest, generator=g) * 0.02).to(torch.bfloat16)  # values do not change the timing
    packer = sbq.loader.StreamingPacker(device=dev)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    mods = [packer.make_linear("int8", host[:n * k].view(n, k)) for _, n, k in shapes]
    packer.finish()
    torch.cuda.synchronize()
    secs = time.perf_counter() - t0
    params = sum(n * k for _, n, k in shapes)
    res = {"seconds": round(secs, 3), "weights": len(mods), "params": params, "h2d_bytes": 2 * params,
           "h2d_gbs": round(2 * params / secs / 1e9, 1), "packed_bytes": sum(int(m.packed.numel()) for m in mods),
           "reference_int8_load_s": 33.2, "note": "host bf16 -> device quantise + pack; storage read not included"}
    del mods, packer
    torch.cuda.empty_cache()
    return res


def kernel_mode(args) -> None:
    """--kernel NAME: one configuration's kernel alone (also the command the ncu captures use)."""
    import torch

    sbq = importlib.import_module("spikingbrain-cpu_b200")
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.Stream(dev)
    res = kernel_cases(sbq, dev, stream, args.steps, args.warmup, which=(args.kernel,))
    print(json.dumps({"kernel": args.kernel, "steps": args.steps, "warmup": args.warmup, "results": res}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="sbq", choices=("sbq", "reference"))
    ap.add_argument("--layers", type=int, default=36)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline measurement")
    ap.add_argument("--no-extra", action="store_true", help="skip the per-configuration kernel timings")
    ap.add_argument("--kernel", choices=("gemv", "mlp", "gemm", "gemm_f32", "gemm_small", "dyn", "lora", "groups"),
                    help="time one configuration's kernel alone")
    ap.add_argument("--program", action="store_true",
                    help="run the decode step as one persistent decode-program launch instead of grouped launches")
    ap.add_argument("--exchange", choices=("peer", "nccl"), default="peer",
                    help="how sharded ranks assemble activations (N > 1): peer stores over NVLink or NCCL all-gather")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be at least 3")
    if args.impl == "reference":
        reference_arm(args)
        return
    if args.kernel:
        kernel_mode(args)
        return

    import torch
    import torch.distributed as dist

    world, rank, local = dist_setup(args)
    sbq = importlib.import_module("spikingbrain-cpu_b200")
    from ctypes import c_void_p

    dev = torch.device("cuda", torch.cuda.current_device())
    group = dist.group.WORLD if world > 1 else None
    stack = sbq.stack.ProjectionStack(layers=args.layers, device=dev, group=group, exchange=args.exchange)
    torch.cuda.synchronize()
    hidden = stack.hidden
    total_bytes = sbq.workloads.stack_bytes(args.layers)  # whole job, all ranks
    stream = torch.cuda.Stream(dev)

    # ---- device-resident timing: one graph replay per step
    runner = sbq.stack.CapturedStack(stack, m=1, stream=stream, use_program=args.program)
    x_static = runner.x
    x_static.copy_(sbq.workloads.activation(1, hidden, seed=5, device=dev))
    torch.cuda.synchronize()
    graph = runner.graph
    for _ in range(args.warmup):
        runner.run()
    torch.cuda.synchronize()
    uuids = ["GPU-" + str(torch.cuda.get_device_properties(dev).uuid)]
    if world > 1:
        allu = [None] * world
        dist.all_gather_object(allu, uuids[0])
        uuids = allu
    torch.cuda.synchronize()
    with ClockSampler(uuids if rank == 0 else []) as clocks:
        # every rank enters the timed region together, after rank 0's sampler is running
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        ms = timed_graph(graph, args.steps, stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = total_bytes / (ms * 1e-3) / 1e9

    # ---- end to end through the public API: pinned host input -> device -> stack -> host output
    x_host = runner.x_host
    x_host.copy_(x_static.cpu())
    e2e_steps = max(10, args.steps // 4)
    for _ in range(3):
        runner(x_host)
    if world > 1:
        dist.barrier()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_ev.record(stream)
    for _ in range(e2e_steps):
        runner(x_host)
    e_ev.record(stream)
    e_ev.synchronize()
    e2e_ms = s_ev.elapsed_time(e_ev) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = total_bytes / (e2e_ms * 1e-3) / 1e9

    # ---- dominant kernel alone: fused gate/up GEMV over the layers' distinct weights
    L = sbq._lib
    n_inter = stack.layers[0].mlp.gate_proj.out_features
    h_buf = torch.empty(1, n_inter, dtype=torch.float16, device=dev)
    st = c_void_p(stream.cuda_stream)

    def gateup_all():
        for layer in stack.layers:
            g, u = layer.mlp.gate_proj, layer.mlp.up_proj
            L.call("sbq_mlp_gateup_w8", c_void_p(x_static.data_ptr()), L.F16, hidden, c_void_p(g.packed.data_ptr()),
                   c_void_p(g.scale.data_ptr()), c_void_p(u.packed.data_ptr()), c_void_p(u.scale.data_ptr()), 1,
                   n_inter, hidden, c_void_p(h_buf.data_ptr()), L.F16, n_inter, st)

    g2, _ = capture(gateup_all, stream)
    with torch.cuda.stream(stream):
        for _ in range(3):
            g2.replay()
    stream.synchronize()
    reps = max(5, min(50, args.steps // 20))
    gu_ms = timed_graph(g2, reps, stream) / len(stack.layers)
    gu_bytes = 2 * n_inter * hidden + 2 * 4 * n_inter + 2 * hidden + 2 * n_inter
    pk = peaks()
    achieved = gu_bytes / (gu_ms * 1e-3) / 1e9
    del g2

    extra = None
    module_api = None
    if world == 1 and not args.no_extra:
        extra = kernel_cases(sbq, dev, stream, args.steps, args.warmup)
        extra["cfg4_stack"] = stack_cases(sbq, stack, dev, stream, args.warmup)
        module_api = module_api_cases(sbq, stack, dev, steps=max(5, min(20, args.steps)), warmup=2)
        extra["load_pack"] = load_pack_case(sbq, dev)
    elif world > 1 and not args.no_extra:
        extra = {"cfg4_prefill_8192_sharded": sharded_prefill_case(sbq, stack, dev, stream, world)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        from oracle import cpu_port

        r = cpu_port.time_stack_decode(layers=2, warmup=1, max_steps=400, min_seconds=8.0, max_seconds=30.0)
        r4 = cpu_port.time_stack_decode(layers=2, warmup=1, max_steps=200, min_seconds=4.0, max_seconds=10.0,
                                        threads=cpu_port.REFERENCE_THREADS)
        cpu = {"value": round(r["gbs"], 3), "unit": "GB/s", "cores": r["cores"], "kind": "port",
               "sample": "reference int8 algorithm (blocked fp32 dequant + sgemm) on 2 of 36 stack layers, "
                         "batch 1, %d steps" % r["steps"],
               "reference_threads_setting": {"value": round(r4["gbs"], 3), "unit": "GB/s", "cores": r4["cores"],
                                             "note": "SB_THREADS=4, the reference's default thread count",
                                             "steps": r4["steps"]}}

    launches = stack.launches_per_step(1, program=runner.program is not None)
    per_gpu = value / world  # each rank streams 1/world of the weights per step
    if world == 1:
        parallelism = "single"
    elif stack.exchange == "peer":
        parallelism = ("output-channel tp%d; GEMV outputs stored to every rank over NVLink (peer memory), "
                       "per-launch arrival counters" % world)
    else:
        parallelism = "output-channel tp%d + NCCL all-gather" % world
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8*fp16->fp32", "data": "synthetic (seeded N(0,0.02) weights, "
                                                                     "per-channel int8; N(0,1) fp16 input)",
            "config": {"workload": "cfg4-stack36-decode-b1", "layers": args.layers, "hidden": hidden,
                       "intermediate": stack.inter, "batch": 1, "weight_bytes_per_step": total_bytes,
                       "parallelism": parallelism,
                       "l2": "no flush: each step streams %.2f GB per GPU > 126 MB L2"
                             % (stack.weight_bytes() / 1e9),
                       "timing": "one CUDA graph replay per step, CUDA events, max over ranks"},
            "roofline": {"kernel": "gemv_w8_kernel (grouped decode GEMV; every launch of the timed step)",
                         "bound": "hbm", "achieved": round(per_gpu, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(per_gpu / pk["hbm_gbs"], 4), "peak_source": pk["source"],
                         "frac_of_spec_8000": round(per_gpu / SPEC_HBM_GBS, 4),
                         "per": "GPU" if world > 1 else "job",
                         "bytes_per_launch": total_bytes // world // launches,
                         "us_per_launch": round(ms * 1e3 / launches, 3),
                         "traffic": traffic_per_launch(launches, len(stack.layers)) if world == 1 else None,
                         "standalone_gateup": {"achieved": round(achieved, 1),
                                               "frac": round(achieved / pk["hbm_gbs"], 4),
                                               "bytes_per_launch": gu_bytes, "us_per_launch": round(gu_ms * 1e3, 3)}},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": 2 * hidden,
                    "d2h_bytes_per_step": 2 * hidden, "ms_per_step": round(e2e_ms, 4),
                    "path": "CapturedStack.__call__ on pinned host tensors (one CUDA graph per step)",
                    "module_api": module_api},
            "gpu_launches": launches * args.steps,
            "clocks": clocks.summary(),
            "configs_0_3": extra,
        }
        print(json.dumps(line), flush=True)
    runner.release()
    if world > 1:
        dist.barrier()
        if stack.peer is not None:
            stack.peer.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
