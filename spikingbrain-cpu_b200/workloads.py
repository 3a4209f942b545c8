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


# ---- the checkpoint's linear layers (for load-time measurement) ---------------------------------
# SpikingBrain2.0's projections as the reference's model declares them (spikingbrain_cpu/model.py:
# GatedMLP :232-240, SoftmaxAttention :243-258, HybridSSEAttention :271-301) with the checkpoint's
# sizes (config.py defaults: hidden 2560, 32 heads of 128, 8 key/value heads, MLP 9728, vocabulary
# 151936, 4 sparse partitions, 36 blocks of which 10 are softmax attention) and the tied int8 head
# (loader.py:94).  Which block indices are attention does not change the list of shapes.
CKPT = {"hidden": 2560, "heads": 32, "head_dim": 128, "kv_heads": 8, "inter": 9728, "vocab": 151936,
        "partitions": 4, "layers": 36, "attn_layers": 10}


def checkpoint_linears() -> list[tuple[str, int, int]]:
    """(name, out_features, in_features) of every linear weight the loader hands to make_linear."""
    c = CKPT
    hid, hd, kvd = c["hidden"], c["heads"] * c["head_dim"], c["kv_heads"] * c["head_dim"]
    out = []
    for i in range(c["layers"]):
        p = "model.layers.%d." % i
        if i < c["attn_layers"]:
            a = p + "attn."
            out += [(a + "q_proj", hd, hid), (a + "k_proj", kvd, hid), (a + "v_proj", kvd, hid), (a + "o_proj", hid, hd)]
        else:
            a = p + "attn."
            out += [(a + "sse_q_proj", hd, hid), (a + "sse_k_proj", hd, hid), (a + "sse_v_proj", hd, hid),
                    (a + "lora_q_proj.0", c["head_dim"], hid), (a + "lora_q_proj.1", hd, c["head_dim"]),
                    (a + "lora_k_proj.0", c["head_dim"], hid), (a + "lora_k_proj.1", hd, c["head_dim"]),
                    (a + "sse_a_proj", 2 * c["heads"], hid), (a + "sse_b_proj", 2 * c["heads"], hid),
                    (a + "sse_e_proj", c["partitions"], hid), (a + "sse_o_proj", hid, hd),
                    (a + "swa_q_proj", hd, hid), (a + "swa_k_proj", kvd, hid), (a + "swa_v_proj", kvd, hid),
                    (a + "swa_o_proj", hid, hd)]
        m = p + "mlp."
        out += [(m + "gate_proj", c["inter"], hid), (m + "up_proj", c["inter"], hid), (m + "down_proj", hid, c["inter"])]
    out.append(("lm_head", c["vocab"], hid))
    return out
