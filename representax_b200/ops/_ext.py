"""Loader for the in-tree sm_100a extension and its device status word.

CUDA tensors always take the native path: when the extension is missing on a
machine with a GPU the ops raise instead of silently falling back to PyTorch.
"""

from __future__ import annotations

import os
import threading

import torch

_lock = threading.Lock()
_module = None
_status: dict[int, torch.Tensor] = {}

STATUS_MESSAGES = {
    1: "TMA producer wait exceeded its budget",
    2: "tensor-core issuer wait exceeded its budget",
    3: "epilogue wait exceeded its budget",
    4: "peer wait exceeded its budget",
    5: "drain of in-flight copies exceeded its budget",
    6: "bad kernel argument",
}


class KernelTimeoutError(RuntimeError):
    """A bounded device-side wait ran out; the kernel unwound and reported it."""


# Kernels launched per binding call (used to count our own launches).
KERNELS_PER_CALL = {"attention_backward": 3, "attention_backward_bias": 3, "grad_norm_sq": 1}


class _CountingModule:
    """Proxy that counts kernel launches made through the extension."""

    def __init__(self, module) -> None:
        self._module = module
        self.launches = 0
        self.counting = False

    def __getattr__(self, name):
        fn = getattr(self._module, name)
        if not callable(fn):
            return fn
        weight = KERNELS_PER_CALL.get(name, 1)

        def wrapped(*args, **kwargs):
            if self.counting:
                self.launches += weight
            return fn(*args, **kwargs)

        return wrapped


def ext():
    """Return the compiled extension module (behind a launch counter)."""

    global _module
    if _module is None:
        with _lock:
            if _module is None:
                try:
                    from representax_b200 import _C  # type: ignore[attr-defined]
                except ImportError as error:  # pragma: no cover - depends on build
                    raise RuntimeError(
                        "representax_b200 CUDA extension is not built; run "
                        "`python setup.py build_ext --inplace` (sm_100a)"
                    ) from error
                if os.environ.get("RX_ATTENTION_TC", "1") == "0":
                    _C.set_attention_tcgen05(False)
                _module = _CountingModule(_C)
    return _module


def launch_counter():
    """The counting proxy: set ``.counting`` and read ``.launches``."""

    return ext()


def available() -> bool:
    try:
        ext()
    except RuntimeError:
        return False
    return True


def status(device: torch.device | int) -> torch.Tensor:
    """Per-device int32 status word that waiting kernels write error codes to."""

    index = torch.device("cuda", device).index if isinstance(device, int) else device.index
    if index is None:
        index = torch.cuda.current_device()
    tensor = _status.get(index)
    if tensor is None:
        tensor = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", index))
        _status[index] = tensor
        ext().register_status_word(tensor)
    return tensor


def check_status(device: torch.device | int) -> None:
    """Raise :class:`KernelTimeoutError` if a kernel on ``device`` reported one."""

    word = status(device)
    code = int(word[0].item())
    if code != 0:
        word.zero_()
        raise KernelTimeoutError(STATUS_MESSAGES.get(code, f"kernel status {code}"))
