"""Generate the golden fixtures for the int8 / int8-dyn path from the reference itself.

Run in a container where the reference project is importable; its root
directory (the one holding ``spikingbrain_cpu/``) is the required argument:

    python tests/golden/make_golden.py REFERENCE_ROOT [--only small|cfg3]

It imports ``spikingbrain_cpu.quant`` from the reference, builds each case with
seeded inputs, runs the reference's own ``quantize_per_channel``,
``Int8Linear`` and ``DynamicInt8Linear`` (quantized engine ``x86``, i.e.
fbgemm), and writes beside this script:

* ``golden.npz`` + ``golden_meta.json``: 26 small cases, every array in full;
* ``golden_cfg3.npz`` + ``golden_cfg3.json``: benchmark configuration 3
  (int8-dyn, m=512, k=n=4096, the package's seeded workload generators) as
  SHA-256 digests of the full reference outputs (quantised activation, weight,
  fp32 output) plus the activation scale / zero point and 16 sampled output
  rows in full.

The tests read only these files; the reference is not needed at test time.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _adversarial_ties(gen: torch.Generator, m: int, k: int) -> torch.Tensor:
    """Activations whose x/s lands on or next to .5 for a fixed per-tensor scale."""
    a, b = 2.5, 3.25
    x = torch.zeros(m, k)
    x[0, 0], x[0, 1] = -a, b
    s = np.float32((np.float64(b) + a) / 255.0)
    kk = torch.randint(-110, 110, (m, k), generator=gen).double()
    jitter = torch.tensor([0.0, 1e-7, -1e-7, 3e-8, -3e-8], dtype=torch.float64)[
        torch.randint(0, 5, (m, k), generator=gen)]
    v = ((kk + 0.5 + jitter) * float(s)).float().clamp(-a, b)
    v[0, 0], v[0, 1] = -a, b
    return v


def _tie_weight(n: int, k: int, gen: torch.Generator) -> torch.Tensor:
    """Weights with exact .5 quotients (scale 1 per row) and an all-zero row."""
    w = (torch.randint(-254, 255, (n, k), generator=gen).float() / 2.0).clamp(-126.5, 126.5)
    w[:, 0] = 127.0
    w[1] = 0.0
    return w


CFG3_SEEDS = {"w": 30, "x": 31}  # workloads.float_weight(4096, 4096, 30), workloads.activation(512, 4096, 31)
CFG3_ROWS = [0, 1, 77, 127, 128, 200, 255, 256, 300, 383, 384, 450, 509, 510, 511, 63]


def sha256(a) -> str:
    import hashlib

    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def cfg3_inputs():
    """Configuration 3's seeded weight (fp32 [4096, 4096]) and activation (fp16 [512, 4096])."""
    import importlib

    sys.path.insert(0, str(HERE.parents[1]))
    wl = importlib.import_module("spikingbrain-cpu_b200.workloads")
    cfg = wl.CONFIGS[3]
    w = wl.float_weight(cfg["n"], cfg["k"], seed=CFG3_SEEDS["w"])
    x = wl.activation(cfg["m"], cfg["k"], seed=CFG3_SEEDS["x"])
    return w, x


def make_cfg3(quant) -> None:
    w, x = cfg3_inputs()
    xf = x.float()  # the reference takes fp32 activations (quant.py:47); fp16 -> fp32 is exact
    q, scale = quant.quantize_per_channel(w)
    y = quant.DynamicInt8Linear(w, None)(xf).detach().numpy()
    # the activation quantisation linear_dynamic applies (fbgemm per-tensor uint8, no range reduction)
    xq_t = torch.quantize_per_tensor_dynamic(xf, torch.quint8, False)
    rows = np.array(CFG3_ROWS)
    info = {"generated_by": "tests/golden/make_golden.py", "torch": torch.__version__,
            "quantized_engine": torch.backends.quantized.engine, "seeds": CFG3_SEEDS,
            "shape": {"m": int(x.shape[0]), "n": int(w.shape[0]), "k": int(w.shape[1])},
            "w_sha256": sha256(w.numpy()), "x_sha256": sha256(x.numpy()),
            "q_sha256": sha256(q.numpy()), "scale_sha256": sha256(scale.numpy()),
            "xq_sha256": sha256(xq_t.int_repr().numpy()),
            "s_x_bits": int(np.float32(xq_t.q_scale()).view(np.uint32)), "zp": int(xq_t.q_zero_point()),
            "y_sha256": sha256(y), "rows": CFG3_ROWS}
    np.savez_compressed(HERE / "golden_cfg3.npz", y_rows=y[rows])
    (HERE / "golden_cfg3.json").write_text(json.dumps(info, indent=1, sort_keys=True) + "\n")
    print("wrote configuration 3: y", y.shape, "digest", info["y_sha256"][:16])


def main(ref_root: str, only: str | None = None) -> None:
    sys.path.insert(0, ref_root)
    from spikingbrain_cpu import quant  # the reference, imported read-only

    torch.backends.quantized.engine = "x86"
    if only in (None, "cfg3"):
        make_cfg3(quant)
    if only == "cfg3":
        return
    arrays: dict[str, np.ndarray] = {}
    meta: dict[str, dict] = {}

    def put(name: str, kind: str, w: torch.Tensor, x: torch.Tensor, bias: torch.Tensor | None, **extra):
        q, scale = quant.quantize_per_channel(w)
        if kind == "int8":
            y = quant.Int8Linear(w, bias)(x)
        else:
            y = quant.DynamicInt8Linear(w, bias)(x)
        arrays[name + "/w"] = w.float().numpy()
        arrays[name + "/x"] = (x.float() if x.dtype == torch.bfloat16 else x).numpy()
        if bias is not None:
            arrays[name + "/bias"] = bias.float().numpy()
        arrays[name + "/q"] = q.numpy()
        arrays[name + "/scale"] = scale.numpy()
        arrays[name + "/y"] = y.detach().numpy()
        meta[name] = {"kind": kind, "w_dtype": str(w.dtype).replace("torch.", ""),
                      "x_dtype": str(x.dtype).replace("torch.", ""), "bias": bias is not None,
                      "shape": {"m": int(x.reshape(-1, x.shape[-1]).shape[0]), "n": int(w.shape[0]),
                                "k": int(w.shape[1])}, **extra}

    g = torch.Generator().manual_seed(20261201)

    def randw(n, k, dtype=torch.float32):
        return (torch.randn(n, k, generator=g) * 0.02).to(dtype)

    def randx(m, k, dtype=torch.float16, scale=1.0, shift=0.0):
        return (torch.randn(m, k, generator=g) * scale + shift).to(dtype)

    # ---- int8 weight-only (Int8Linear)
    put("w8_m1_n64_k128", "int8", randw(64, 128), randx(1, 128), None)
    put("w8_m3_n48_k192", "int8", randw(48, 192), randx(3, 192), None)
    put("w8_m17_n130_k320", "int8", randw(130, 320), randx(17, 320), None)
    put("w8_m16_n256_k512", "int8", randw(256, 512), randx(16, 512), None)
    put("w8_m1_n4_k256", "int8", randw(4, 256), randx(1, 256), None)
    put("w8_m2_n32_k64_bias", "int8", randw(32, 64), randx(2, 64), torch.randn(32, generator=g))
    put("w8_m5_n64_k256_fp32x", "int8", randw(64, 256), randx(5, 256, torch.float32), None)
    put("w8_m4_n64_k128_bf16w", "int8", randw(64, 128, torch.bfloat16), randx(4, 128), None)
    put("w8_m4_n64_k128_bf16x", "int8", randw(64, 128), randx(4, 128, torch.bfloat16), None)
    put("w8_m3_n16_k128_ties", "int8", _tie_weight(16, 128, g), randx(3, 128), None)
    put("w8_m64_n128_k256", "int8", randw(128, 256), randx(64, 256), None)
    put("w8_m2x3_n32_k64_batched", "int8", randw(32, 64), randx(6, 64).reshape(2, 3, 64), None)

    # ---- int8-dyn (DynamicInt8Linear, fbgemm dynamic per-tensor activation quantisation)
    put("dyn_m3_n64_k128", "int8-dyn", randw(64, 128), randx(3, 128, torch.float32), None)
    put("dyn_m8_n128_k256", "int8-dyn", randw(128, 256), randx(8, 256, torch.float32), None)
    put("dyn_m5_n40_k192_ties", "int8-dyn", randw(40, 192), _adversarial_ties(g, 5, 192), None)
    put("dyn_m4_n32_k77_ties", "int8-dyn", randw(32, 77), _adversarial_ties(g, 4, 77), None)
    put("dyn_m2_n32_k64_zero", "int8-dyn", randw(32, 64), torch.zeros(2, 64), None)
    put("dyn_m3_n32_k64_tiny", "int8-dyn", randw(32, 64), randx(3, 64, torch.float32, 1e-6), None)
    put("dyn_m3_n32_k64_tinypos", "int8-dyn", randw(32, 64), randx(3, 64, torch.float32, 1e-6).abs(), None)
    put("dyn_m3_n32_k64_tinyneg", "int8-dyn", randw(32, 64), -randx(3, 64, torch.float32, 1e-6).abs(), None)
    put("dyn_m3_n32_k64_pos", "int8-dyn", randw(32, 64), randx(3, 64, torch.float32).abs() + 0.25, None)
    put("dyn_m3_n32_k64_neg", "int8-dyn", randw(32, 64), -randx(3, 64, torch.float32).abs() - 0.25, None)
    put("dyn_m2_n32_k64_bias", "int8-dyn", randw(32, 64), randx(2, 64, torch.float32), torch.randn(32, generator=g))
    put("dyn_m33_n192_k512", "int8-dyn", randw(192, 512), randx(33, 512, torch.float32, 3.0, 0.5), None)
    put("dyn_m8_n64_k256_fp16x", "int8-dyn", randw(64, 256), randx(8, 256), None)
    put("dyn_m1_n64_k128", "int8-dyn", randw(64, 128), randx(1, 128, torch.float32), None)

    np.savez_compressed(HERE / "golden.npz", **arrays)
    info = {"generated_by": "tests/golden/make_golden.py", "torch": torch.__version__,
            "quantized_engine": torch.backends.quantized.engine, "seed": 20261201, "cases": meta}
    (HERE / "golden_meta.json").write_text(json.dumps(info, indent=1, sort_keys=True) + "\n")
    print("wrote", len(meta), "cases,", sum(a.nbytes for a in arrays.values()), "bytes raw")


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("reference_root", help="directory holding the reference's spikingbrain_cpu package")
    ap.add_argument("--only", choices=("small", "cfg3"), help="regenerate one fixture set")
    a = ap.parse_args()
    main(a.reference_root, a.only)
