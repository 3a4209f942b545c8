"""Torch-CPU port of the reference's quantised-linear forward passes, timed as the CPU baseline.

TEST / BASELINE INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  The reference project is pure
Python and is not present on the GPU host, so ``bench.py`` times this port there instead.  It runs
the reference's algorithm with the same torch CPU kernels:

* ``int8_forward``  Int8Linear.forward (spikingbrain_cpu/quant.py:41-53): fp32 activations, the
  weight dequantised to fp32 in 128-row blocks, one fp32 sgemm per block, then the per-row scale.
* ``dyn_forward``   DynamicInt8Linear.forward (quant.py:56-66): fbgemm's prepacked int8 weight and
  ``quantized::linear_dynamic`` (engine ``x86``), exactly the library call the reference makes.
* ``StackSample``   the synthetic projection stack of ``spikingbrain-cpu_b200/stack.py`` built from
  those two, on a bounded number of layers.
"""

from __future__ import annotations

import os
import time

import torch
import torch.nn.functional as F


def use_all_cores() -> int:
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


# The reference's own thread setting (SB_THREADS, default 4: spikingbrain_cpu/bench.py:231).
REFERENCE_THREADS = 4


def int8_forward(x: torch.Tensor, q: torch.Tensor, scale: torch.Tensor, block: int = 128) -> torch.Tensor:
    """fp32 x [m, k] times int8 q [n, k] dequantised block by block, then scaled (quant.py:46-53)."""
    x2 = x.reshape(-1, q.shape[1]).float()
    out = torch.empty(x2.shape[0], q.shape[0], dtype=torch.float32)
    for lo in range(0, q.shape[0], block):
        hi = min(lo + block, q.shape[0])
        torch.matmul(x2, q[lo:hi].float().t(), out=out[:, lo:hi])
    return out * scale


def dyn_prepack(q: torch.Tensor, scale: torch.Tensor):
    """fbgemm prepack of the per-channel int8 weight (quant.py:60-61)."""
    torch.backends.quantized.engine = "x86"
    qw = torch._make_per_channel_quantized_tensor(q, scale.double(), torch.zeros(q.shape[0], dtype=torch.long), 0)
    return torch.ops.quantized.linear_prepack(qw, None)


def dyn_forward(x: torch.Tensor, packed) -> torch.Tensor:
    return torch.ops.quantized.linear_dynamic(x.reshape(-1, x.shape[-1]).float().contiguous(), packed)


class StackSample:
    """``layers`` layers of the projection stack on the CPU (random int8 weights, unit-ish scales)."""

    def __init__(self, layers: int = 2, hidden: int = 4096, inter: int = 12288, seed: int = 0):
        g = torch.Generator().manual_seed(seed)
        self.hidden, self.inter = hidden, inter

        def w(n, k):
            q = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
            return q, torch.full((n,), 1.0 / (127.0 * k ** 0.5))

        self.layers = [{"qkvd": w(4 * hidden, hidden), "o": w(hidden, hidden), "dout": w(hidden, hidden),
                        "gate": w(inter, hidden), "up": w(inter, hidden), "down": w(hidden, inter)}
                       for _ in range(layers)]

    def weight_bytes(self) -> int:
        return sum(q.numel() for layer in self.layers for q, _ in layer.values())

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        hd = self.hidden
        for L in self.layers:  # the device stack's data flow: o(v) is the next layer's input
            qkvd = int8_forward(x, *L["qkvd"]).half()
            h = (F.silu(int8_forward(x, *L["gate"])) * int8_forward(x, *L["up"])).half()
            int8_forward(h, *L["down"])
            int8_forward(qkvd[:, 3 * hd:], *L["dout"])
            x = int8_forward(qkvd[:, 2 * hd:3 * hd], *L["o"]).half()
        return x


def time_stack_decode(layers: int = 2, m: int = 1, warmup: int = 1, max_steps: int = 1000,
                      min_seconds: float = 0.0, max_seconds: float = 120.0, threads: int | None = None) -> dict:
    """Weight GB/s of the reference algorithm on ``layers`` stack layers.

    Runs ``warmup`` untimed steps, then timed steps until ``max_steps`` are done or ``max_seconds``
    have passed (and at least ``min_seconds``, if ``max_steps`` allows).  ``threads``: torch's
    intra-op threads (default: every core of the host).
    """
    before = torch.get_num_threads()
    if threads is None:
        cores = use_all_cores()
    else:
        torch.set_num_threads(threads)
        cores = torch.get_num_threads()
    sample = StackSample(layers)
    x = torch.randn(m, sample.hidden).half()
    for _ in range(max(0, warmup)):
        sample.forward(x)
    steps, t0 = 0, time.perf_counter()
    while steps < max_steps:
        sample.forward(x)
        steps += 1
        el = time.perf_counter() - t0
        if el >= max_seconds or (min_seconds and el >= min_seconds):
            break
    dt = (time.perf_counter() - t0) / steps
    torch.set_num_threads(before)
    return {"gbs": sample.weight_bytes() / dt / 1e9, "s_per_step": dt, "steps": steps, "cores": cores,
            "layers": layers, "m": m, "bytes": sample.weight_bytes()}
