"""Loader for the in-tree sm_100a extension (``tornado_gcm_b200/_C*.so``).

The CUDA code paths require it: when a CUDA tensor reaches an op and the
extension did not load, :func:`require` raises instead of silently falling
back to eager torch.
"""

from __future__ import annotations

import glob
import os

import torch

_LOADED = None
_ERROR = None


def load() -> bool:
    global _LOADED, _ERROR
    if _LOADED is not None:
        return _LOADED
    try:
        from tornado_gcm_b200 import _C  # noqa: F401  (registers torch.ops.tgcm.*)

        _LOADED = hasattr(torch.ops.tgcm, "sht_synth")
    except Exception as exc:  # pragma: no cover - depends on the build
        _ERROR = exc
        _LOADED = False
    return _LOADED


def available() -> bool:
    return load()


def require(what: str = "kernel"):
    if not load():
        here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        found = glob.glob(os.path.join(here, "_C*.so"))
        raise RuntimeError(
            f"tornado_gcm_b200 CUDA extension required for {what} but not loaded "
            f"(found {found}; error: {_ERROR}). Build it with `python setup.py build_ext --inplace`.")
    from tornado_gcm_b200.ops import accounting

    if accounting.active() is not None:
        return accounting.CountingOps(torch.ops.tgcm)
    return torch.ops.tgcm


_POISON = os.environ.get("TGCM_POISON", "0") not in ("", "0")


def poison_enabled() -> bool:
    """Poison mode: op outputs and scratch start as NaN (see ``csrc/alloc.h``)."""
    return _POISON


def set_poison_mode(on: bool) -> None:
    """Switch poison mode for both the Python wrappers and the native allocations."""
    global _POISON
    _POISON = bool(on)
    if load():
        torch.ops.tgcm.set_poison_mode(_POISON)


def empty(*shape, dtype, device) -> torch.Tensor:
    """``torch.empty`` that honours poison mode (NaN / all-ones fill)."""
    t = torch.empty(*shape, dtype=dtype, device=device)
    if poison_enabled():
        t.fill_(float("nan") if t.is_floating_point() else -1)
    return t


def set_bounds_check(on: bool) -> None:
    """Bounds-checked mode of the table-driven kernels: every index read from a
    table (recipe terms: channels, stencils, diagonals, matrices) is checked on
    the device before use; a bad one records error code 5 in the device error
    flag and is skipped instead of dereferenced (:func:`check_error_flag` raises)."""
    require("bounds checks").set_bounds_check(bool(on))


def _flag_key(device) -> str:
    d = torch.device(device)
    if d.type == "cuda" and d.index is None:
        d = torch.device("cuda", torch.cuda.current_device())
    return str(d)


def error_flag(device) -> torch.Tensor:
    """Per-device int32 flag that kernels set on a bounded-wait timeout."""
    key = _flag_key(device)
    t = _FLAGS.get(key)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _FLAGS[key] = t
    return t


_FLAGS: dict = {}


def check_error_flag(device) -> int:
    """Read (and clear) the device error flag; raises on a recorded timeout."""
    f = _FLAGS.get(_flag_key(device))
    if f is None:
        return 0
    code = int(f.item())
    if code:
        f.zero_()
        what = "index out of bounds" if code == 5 else "bounded wait expired"
        raise RuntimeError(f"tornado_gcm_b200 kernel reported error code {code} ({what})")
    return 0
