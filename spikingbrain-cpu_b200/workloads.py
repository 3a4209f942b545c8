"""Seeded synthetic workloads of the benchmark configurations (no checkpoint or dataset exists here).

Weights follow the recipe of the reference's own quantiser (spikingbrain_cpu/quant.py:25-29):
``w ~ N(0, 0.02)`` in fp32, per-row ``scale = max|w| / 127`` and ``q = rint(w / scale)``, which
gives int8 values in [-127, 127].  Activations are ``N(0, 1)`` fp16.  Every generator takes an
explicit seed and uses its own ``torch.Generator`` so the same inputs come out on any machine.

Shapes (BASELINE configurations):
  0  decode GEMV          m=1,  k=4096,  n=4096
  1  fused MLP decode     m in {1,4,16}, gate/up [12288 x 4096], down [4096 x 12288]
  2  prefill GEMM         m=2048, k=4096, n=12288, fp16 out
  3  int8-dyn GEMM        m=512, k=4096, n=4096
  4  36-layer stack       per layer 6 x [4096 x 4096] + gate/up [12288 x 4096] + down [4096 x 12288];
                          decode batch {1, 8, 64}, prefill 8192 tokens
"""

from __future__ import annotations

import torch

HIDDEN = 4096
INTER = 12288
LAYERS = 36

CONFIGS = {
    0: {"name": "decode-gemv", "m": 1, "k": HIDDEN, "n": HIDDEN},
    1: {"name": "mlp-decode", "m": (1, 4, 16), "k": HIDDEN, "n": INTER},
    2: {"name": "prefill-gemm", "m": 2048, "k": HIDDEN, "n": INTER},
    3: {"name": "int8-dyn-gemm", "m": 512, "k": HIDDEN, "n": HIDDEN},
    4: {"name": "stack36", "layers": LAYERS, "hidden": HIDDEN, "inter": INTER, "decode_m": (1, 8, 64),
        "prefill_m": 8192},
}

# Per-layer projections of the synthetic stack: (name, n, k).  q/k/v/o and the delta-net in/out
# projections are [4096 x 4096]; the MLP is gate/up [12288 x 4096] and down [4096 x 12288].
STACK_LAYER = (("q", HIDDEN, HIDDEN), ("k", HIDDEN, HIDDEN), ("v", HIDDEN, HIDDEN), ("o", HIDDEN, HIDDEN),
               ("delta_in", HIDDEN, HIDDEN), ("delta_out", HIDDEN, HIDDEN), ("gate", INTER, HIDDEN),
               ("up", INTER, HIDDEN), ("down", HIDDEN, INTER))


def float_weight(n: int, k: int, seed: int, device="cpu") -> torch.Tensor:
    """fp32 ``N(0, 0.02)`` weight [n, k]."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    return torch.randn(n, k, generator=g, device=dev, dtype=torch.float32) * 0.02


def activation(m: int, k: int, seed: int, dtype=torch.float16, device="cpu") -> torch.Tensor:
    """``N(0, 1)`` activation [m, k] in ``dtype``."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    return torch.randn(m, k, generator=g, device=dev, dtype=torch.float32).to(dtype)


def stack_bytes(layers: int = LAYERS) -> int:
    """int8 weight bytes streamed by one decode step of the stack."""
    return layers * sum(n * k for _, n, k in STACK_LAYER)


def stack_flops(m: int, layers: int = LAYERS) -> int:
    return 2 * m * stack_bytes(layers)
