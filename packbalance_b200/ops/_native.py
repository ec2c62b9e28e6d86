"""Loader for the in-tree native extension ``packbalance_b200._C``.

There is deliberately no silent fallback: a CUDA op whose extension cannot be
imported raises, so a missing build never turns into a slow PyTorch run.
"""

from __future__ import annotations

import functools

import torch


@functools.lru_cache(maxsize=1)
def module():
    try:
        from packbalance_b200 import _C
    except ImportError as exc:  # pragma: no cover - depends on the build
        raise RuntimeError(
            "packbalance_b200 native extension is not built; run `python setup.py build_ext --inplace` "
            "(or __graft_entry__.build())"
        ) from exc
    return _C


def available() -> bool:
    try:
        module()
    except RuntimeError:
        return False
    return True


_DETERMINISTIC = False


def set_deterministic(on: bool) -> bool:
    """Fixed-order reductions in the native step (the reference's ``train.deterministic``).

    While on: weight-gradient and CE-backward GEMMs run without split-K (one writer per
    output tile, no reduce-adds); RMSNorm dw, the gradient norm and the embedding
    gradient are summed in a fixed order instead of with fp32 atomics; the attention
    backward runs as an fp32 per-document recomputation (no reduce-adds across key tiles or
    heads).  Two runs on the same inputs then give bitwise identical weights, at the cost
    of speed (a debugging mode).  Returns the previous setting."""
    global _DETERMINISTIC
    prev = _DETERMINISTIC
    _DETERMINISTIC = bool(on)
    if available():
        module().set_deterministic(_DETERMINISTIC)
    return prev


def deterministic() -> bool:
    return _DETERMINISTIC


class KernelTimeout(RuntimeError):
    """A device-side bounded wait gave up (see the status code for which one)."""


STATUS_NAMES = {
    101: "gemm producer: smem slot never freed",
    102: "gemm producer: drain of in-flight copies",
    103: "gemm mma: accumulator never released",
    104: "gemm mma: tile copy never landed",
    105: "gemm mma: drain",
    106: "gemm epilogue: accumulator never ready",
}


def check_status(device: torch.device | int | None = None, clear: bool = True) -> None:
    """Raise :class:`KernelTimeout` if any kernel on ``device`` recorded a timeout."""
    if device is None:
        dev = torch.cuda.current_device()
    elif isinstance(device, torch.device):
        dev = device.index if device.index is not None else torch.cuda.current_device()
    else:
        dev = int(device)
    code = int(module().status_read(dev, clear))
    if code:
        raise KernelTimeout(f"device {dev}: kernel wait timed out (code {code}: {STATUS_NAMES.get(code, 'see csrc')})")
