"""Backend dispatch with exactly one backend: the sm_100a CUDA library.

Keeps the reference dispatcher's observable contract
(mxflashattn/dispatch.py:15-30, :89-170): a thread-local ``DispatchInfo``
recorded for every successful call, ``get_last_dispatch_info()``, and
``BackendUnavailableError`` carrying an actionable reason when the call
cannot run natively.  What changed by design: the MetaX vendor branch and the
ATen bring-up branch are gone, and so is the CPU reference fallback -- the
PyTorch oracle is test infrastructure only, so ``MXFLASHATTN_ALLOW_FALLBACK``
no longer routes anywhere; the error says so.
"""

from __future__ import annotations

import importlib
import os
import threading
from dataclasses import dataclass
from typing import Any

import torch

BACKEND_LABEL = "cuda_sm100"
_EXTENSION_MODULE = "mxflashattn_b200.backend"


class BackendUnavailableError(RuntimeError):
    """Raised when the CUDA backend cannot execute the call."""


@dataclass(frozen=True)
class DispatchInfo:
    backend: str
    operation: str
    fallback_reason: str | None = None


_state = threading.local()


def get_last_dispatch_info() -> DispatchInfo | None:
    return getattr(_state, "dispatch_info", None)


_EXTENSION: list[Any] = []  # the imported backend module, once found


def _native_extension() -> Any | None:
    """The backend module, or None when it cannot be imported (tests replace this)."""
    if _EXTENSION:
        return _EXTENSION[0]
    try:
        module = importlib.import_module(_EXTENSION_MODULE)
    except (ImportError, OSError):
        return None
    _EXTENSION.append(module)
    return module


_INFOS: dict[str, DispatchInfo] = {}  # immutable records, one per operation


def native_unavailable_reason(tensor: Any, operation: str) -> str | None:
    """Why ``operation`` on ``tensor`` cannot run natively, or None if it can."""
    if tensor.device.type != "cuda":
        return "native_backend_requires_accelerator_tensor"
    if tensor.dtype not in (torch.float16, torch.bfloat16):
        return "native_backend_supports_only_float16_and_bfloat16"
    extension = _native_extension()
    if extension is None:
        return "native_extension_not_built_or_not_importable"
    try:
        available = bool(extension.is_available())
    except Exception as exc:  # a broken library is reported, not hidden
        return f"native_availability_check_failed:{type(exc).__name__}:{exc}"
    if not available:
        return "native_extension_reports_unavailable_runtime"
    if not callable(getattr(extension, operation, None)):
        return f"native_extension_does_not_implement_{operation}"
    return None


def dispatch(operation: str, tensor: Any, extension_args: tuple[Any, ...]) -> Any:
    """Run ``operation`` on the CUDA backend or raise ``BackendUnavailableError``."""
    _state.dispatch_info = None
    reason = native_unavailable_reason(tensor, operation)
    if reason is None:
        extension = _native_extension()
        try:
            result = getattr(extension, operation)(*extension_args)
        except RuntimeError as exc:
            if type(exc).__name__ != "NativeLibraryError":
                raise
            reason = f"native_call_failed:{exc}"
        else:
            info = _INFOS.get(operation)
            if info is None:
                info = _INFOS[operation] = DispatchInfo(backend=BACKEND_LABEL, operation=operation)
            _state.dispatch_info = info
            return result
    hint = ""
    if os.getenv("MXFLASHATTN_ALLOW_FALLBACK", "").strip() == "1":
        hint = ("; MXFLASHATTN_ALLOW_FALLBACK=1 is ignored: this build ships no CPU reference path "
                "(the PyTorch oracle is test infrastructure only)")
    raise BackendUnavailableError(f"MXFlashAttn dispatch failed ({reason}){hint}")
