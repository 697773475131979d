"""Device guard and loader for the sm_100a native extension.

Mirrors ``python/kernels/native.py`` of the reference (its ``require_dcu`` /
``_extension`` pair, lines 19-62): every public operator validates its inputs
in pure Python first, then calls :func:`require_dcu` -- which here requires a
CUDA build of PyTorch, a visible GPU of compute capability 10.x (B200,
sm_100a) and inputs on one CUDA device -- and finally loads
``bysj_b200._C`` and requires the entry point it needs.  There is no CPU
fallback: on a host without the GPU or without the built extension the
operators raise ``RuntimeError``.  The guard keeps the reference's name so
code (and tests) that patch ``require_dcu`` keep working.
"""
from __future__ import annotations

import importlib

import torch

_EXTENSION_MODULE = "bysj_b200._C"
_SUPPORTED_MAJOR = 10  # Blackwell datacenter parts: sm_100 / sm_100a


def _require_cuda_runtime():
    if getattr(torch.version, "hip", None):
        raise RuntimeError("B200 operators require a CUDA build of PyTorch, not ROCm/HIP")
    if not torch.version.cuda:
        raise RuntimeError("B200 operators require a CUDA-enabled PyTorch build")
    if not torch.cuda.is_available():
        raise RuntimeError("B200 operators require a visible, available CUDA GPU")


def require_dcu(*tensors):
    """Require a supported GPU runtime and inputs on one CUDA device.

    Returns the ``torch.device`` the operator will run on.  (The name is the
    reference's; the check is for an sm_100 B200 GPU.)
    """
    _require_cuda_runtime()
    device = None
    for tensor in tensors:
        if tensor is None or not isinstance(tensor, torch.Tensor):
            continue
        if tensor.device.type != "cuda":
            raise RuntimeError(
                f"B200 operator inputs must be on a CUDA device, got {tensor.device}"
            )
        if device is not None and tensor.device != device:
            raise RuntimeError("B200 operator inputs must share one device")
        device = tensor.device
    index = torch.cuda.current_device() if device is None or device.index is None else device.index
    try:
        major, minor = torch.cuda.get_device_capability(index)
    except (AssertionError, RuntimeError) as exc:
        raise RuntimeError(f"cannot inspect CUDA device {index}") from exc
    if major != _SUPPORTED_MAJOR:
        raise RuntimeError(
            f"unsupported GPU architecture sm_{major}{minor}; "
            "this build targets sm_100a (B200)"
        )
    return torch.device("cuda", index)


require_b200 = require_dcu


def _extension(required_symbol: str):
    """Load ``bysj_b200._C`` and require the requested operator."""
    _require_cuda_runtime()
    try:
        extension = importlib.import_module(_EXTENSION_MODULE)
    except (ImportError, OSError) as exc:
        raise RuntimeError(
            "build the B200 extension first (python -m bysj_b200._build): "
            "segment, RMSNorm and GIE operators live in bysj_b200._C"
        ) from exc
    if not hasattr(extension, required_symbol):
        raise RuntimeError(
            f"the loaded {_EXTENSION_MODULE} extension has no {required_symbol!r} entry point"
        )
    return extension


__all__ = ["require_b200", "require_dcu"]
