"""Peak-FLOPs table and MFU (reference: tinytron/utils/profile.py:3-45).

Adds Blackwell entries (the reference has none, so it reports MFU 0 on B200).  The
B200 bf16 entry is the dense nominal peak; ``measured_peak_flops`` reads the
driver-measured cuBLAS figure from MEASURED_PEAKS.json when present.
"""
from __future__ import annotations

import json
import os
from pathlib import Path

import torch

GPU_PEAK_FLOPS = {
    "T4": {"fp32": 8.1e12, "fp16": 65e12, "bf16": 0},
    "V100": {"fp32": 15.7e12, "fp16": 125e12, "bf16": 0},
    "A100": {"fp32": 19.5e12, "fp16": 312e12, "bf16": 312e12},
    "A40": {"fp32": 37.4e12, "fp16": 149e12, "bf16": 149e12},
    "A30": {"fp32": 10.3e12, "fp16": 165e12, "bf16": 165e12},
    "RTX 6000 Ada": {"fp32": 91e12, "fp16": 181e12, "bf16": 181e12},
    "L4": {"fp32": 30e12, "fp16": 120e12, "bf16": 120e12},
    "L40": {"fp32": 91e12, "fp16": 181e12, "bf16": 181e12},
    "L40S": {"fp32": 91e12, "fp16": 181e12, "bf16": 181e12},
    "3090": {"fp32": 35.6e12, "fp16": 142e12, "bf16": 142e12},
    "4090": {"fp32": 82.6e12, "fp16": 330e12, "bf16": 330e12},
    "H100": {"fp32": 60e12, "fp16": 989e12, "bf16": 989e12, "fp8": 1979e12},
    "H800": {"fp32": 34e12, "fp16": 734e12, "bf16": 734e12, "fp8": 1468e12},
    "H200": {"fp32": 67e12, "fp16": 989e12, "bf16": 989e12, "fp8": 1979e12},
    "H20": {"fp32": 21e12, "fp16": 494e12, "bf16": 494e12, "fp8": 988e12},
    "B200": {"fp32": 80e12, "fp16": 2250e12, "bf16": 2250e12, "fp8": 4500e12, "fp4": 9000e12},
    "B300": {"fp32": 80e12, "fp16": 2250e12, "bf16": 2250e12, "fp8": 4500e12, "fp4": 13500e12},
}


def get_gpu_peak_flops(dtype: str = "bf16", per_device: bool = True) -> float:
    name = torch.cuda.get_device_name(0) if torch.cuda.is_available() else ""
    peak = None
    for k, v in GPU_PEAK_FLOPS.items():
        if k in name:
            peak = v.get(dtype.lower())
            break
    if not peak:
        print(f"Warning: unknown or unsupported FLOPs for GPU {name!r} with dtype {dtype}")
        peak = 0
    return peak if per_device else peak * torch.cuda.device_count()


def measured_peak_flops(default: float | None = None) -> float | None:
    """cuBLAS bf16 burst TFLOP/s measured on this pool (MEASURED_PEAKS.json), in FLOP/s."""
    p = Path(os.environ.get("TT_MEASURED_PEAKS", Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"))
    try:
        return float(json.loads(p.read_text())["bf16_tflops"]) * 1e12
    except Exception:
        return default


def compute_mfu(model, batch_size, seq_len, time, ga=1, dtype="bf16"):
    """(mfu, achieved FLOP/s, peak FLOP/s) with the reference FLOP formula."""
    flops = model.get_flops_per_fwd_bwd(batch_size, seq_len) * ga
    achieved = flops / time if time > 0 else 0.0
    peak = get_gpu_peak_flops(dtype=dtype, per_device=True)
    return (achieved / peak if peak else 0), achieved, peak


# ---------------------------------------------------------------------------- NVTX
_NVTX = None


def nvtx_enabled() -> bool:
    global _NVTX
    if _NVTX is None:
        import os

        _NVTX = os.environ.get("TT_NVTX", "0") == "1"
    return _NVTX


class nvtx_range:
    """NVTX range around a block (``TT_NVTX=1``; a no-op otherwise), so Nsight/CUPTI timelines
    show model-level regions (layers, attention, MLP/MoE, ZeRO-1 sync) around the kernels."""

    __slots__ = ("name", "on")

    def __init__(self, name: str):
        self.name = name
        self.on = nvtx_enabled()

    def __enter__(self):
        if self.on:
            import torch

            torch.cuda.nvtx.range_push(self.name)
        return self

    def __exit__(self, *exc):
        if self.on:
            import torch

            torch.cuda.nvtx.range_pop()
        return False
