"""B200 (sm_100a) int8 / int8-dyn quantised-linear path of spikingbrain-cpu.

A drop-in for ``spikingbrain_cpu.quant`` (same names and contracts) backed by libsbq.so, the
hand-written CUDA kernels behind the C ABI in ``include/sbq.h``.  Import it by its directory
name: ``importlib.import_module("spikingbrain-cpu_b200")``.
"""

from . import _lib, groups, loader, stack, workloads
from .mlp import FusedGatedMLP, FusedLoRAPair, fuse_gated_mlp, fuse_lora_pairs
from .quant import (FORMATS, BF16Linear, DynamicInt8Linear, FloatLinear, FP16Linear, Int8Linear, make_linear,
                    pack_int8, pack_weight, quantize_per_channel, unpack_int8)

__all__ = ["FORMATS", "BF16Linear", "DynamicInt8Linear", "FloatLinear", "FP16Linear", "Int8Linear", "make_linear",
           "pack_int8", "pack_weight", "quantize_per_channel", "unpack_int8", "_lib", "groups", "loader", "workloads", "stack", "FusedGatedMLP", "fuse_gated_mlp", "FusedLoRAPair", "fuse_lora_pairs"]
