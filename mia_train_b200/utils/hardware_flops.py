"""Dense per-GPU peak throughput, the MFU denominator (reference `src/utils/hardware_flops.py:38-131`).

Figures are the vendors' dense (non-sparse) tensor-core rates; the 2:4-sparsity headline numbers
are exactly twice these and would halve every reported MFU. Entries are matched most-specific
first on `torch.cuda.get_device_name()`. The fp32 peak depends on whether TF32 matmuls are
enabled, so it reads `torch.backends.cuda.matmul.allow_tf32` unless told.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

_T = 1.0e12


@dataclass(frozen=True)
class DevicePeak:
    label: str
    bf16: float
    tf32: float
    fp32: float


_TABLE: tuple[tuple[tuple[str, ...], DevicePeak], ...] = (
    (("B200",), DevicePeak("NVIDIA B200", 2250 * _T, 1100 * _T, 80 * _T)),
    (("H200",), DevicePeak("NVIDIA H200 SXM", 989.4 * _T, 494.7 * _T, 67 * _T)),
    (("H100 NVL",), DevicePeak("NVIDIA H100 NVL", 835.5 * _T, 417.7 * _T, 60 * _T)),
    (("H100 PCIE",), DevicePeak("NVIDIA H100 PCIe", 756.5 * _T, 378.2 * _T, 51 * _T)),
    (("H100",), DevicePeak("NVIDIA H100 SXM", 989.4 * _T, 494.7 * _T, 67 * _T)),
    (("A100",), DevicePeak("NVIDIA A100", 312 * _T, 156 * _T, 19.5 * _T)),
    (("L40S",), DevicePeak("NVIDIA L40S", 362 * _T, 183 * _T, 91.6 * _T)),
    (("L40",), DevicePeak("NVIDIA L40", 181.05 * _T, 90.5 * _T, 90.5 * _T)),
    (("L4",), DevicePeak("NVIDIA L4", 121 * _T, 60.5 * _T, 30.3 * _T)),
    (("A40",), DevicePeak("NVIDIA A40", 149.7 * _T, 74.8 * _T, 37.4 * _T)),
    (("A6000",), DevicePeak("NVIDIA RTX A6000", 154.8 * _T, 77.4 * _T, 38.7 * _T)),
)
_NO_BF16 = ("T4", "V100")


def _normalize(name: str) -> str:
    return name.upper().replace("-", " ")


def lookup_device(device_name: str) -> DevicePeak | None:
    normalized = _normalize(device_name)
    for keys, peak in _TABLE:
        if any(key in normalized for key in keys):
            return peak
    return None


def peak_flops(
    device_name: str, precision: str, allow_tf32: bool | None = None
) -> tuple[float | None, str]:
    """(peak FLOP/s, "") or (None, reason) for this device at this training precision."""
    normalized = _normalize(device_name)
    if precision == "bf16" and any(key in normalized for key in _NO_BF16):
        return None, f"{device_name} has no bf16 tensor cores, so it has no rated bf16 peak"
    peak = lookup_device(device_name)
    if peak is None:
        return None, (
            f"{device_name!r} is not in the peak-FLOPS table; set [trainer].peak_tflops to enable MFU"
        )
    if precision == "bf16":
        return peak.bf16, ""
    if precision == "fp32":
        if allow_tf32 is None:
            allow_tf32 = torch.backends.cuda.matmul.allow_tf32
        return (peak.tf32 if allow_tf32 else peak.fp32), ""
    return None, f"unknown precision {precision!r}"


def known_devices() -> tuple[str, ...]:
    return tuple(peak.label for _, peak in _TABLE)
