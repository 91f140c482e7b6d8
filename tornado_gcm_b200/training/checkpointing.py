"""``.pt`` checkpoints — same keys as reference ``training/checkpointing.py:20-95``:
``{"model_state_dict", "optimizer_state_dict", "training_state": {step, phase,
best_val_loss}, "ema_params"?}`` and the inference export
``{"model_state_dict": <bf16 floats>, "format": "inference"}``.  Writes are
atomic (temp file + rename) so an interrupted save never corrupts the last
good checkpoint."""

from __future__ import annotations

import dataclasses
import os
import pathlib
import tempfile

import torch
import torch.nn as nn


@dataclasses.dataclass
class TrainingState:
    step: int = 0
    phase: int = 0
    best_val_loss: float = float("inf")


def _atomic_save(obj, path: pathlib.Path) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    fd, tmp = tempfile.mkstemp(dir=str(path.parent), prefix="ckpt_tmp_", suffix=".pt")
    os.close(fd)
    try:
        torch.save(obj, tmp)
        os.replace(tmp, path)
    finally:
        if os.path.exists(tmp):
            os.remove(tmp)


def _unwrap(model: nn.Module) -> nn.Module:
    while hasattr(model, "module"):
        model = model.module
    return model


def save_checkpoint(path, model: nn.Module, optimizer: torch.optim.Optimizer, training_state: TrainingState,
                    ema_params: dict | None = None) -> None:
    ckpt = {"model_state_dict": _unwrap(model).state_dict(), "optimizer_state_dict": optimizer.state_dict(),
            "training_state": dataclasses.asdict(training_state)}
    if ema_params is not None:
        ckpt["ema_params"] = {k: v.detach().cpu() for k, v in ema_params.items()}
    _atomic_save(ckpt, pathlib.Path(path))


def load_checkpoint(path, model: nn.Module, optimizer: torch.optim.Optimizer | None = None,
                    strict: bool = True) -> TrainingState:
    ckpt = torch.load(path, map_location="cpu", weights_only=False)
    _unwrap(model).load_state_dict(ckpt["model_state_dict"], strict=strict)
    if optimizer is not None and "optimizer_state_dict" in ckpt:
        optimizer.load_state_dict(ckpt["optimizer_state_dict"])
    return TrainingState(**ckpt.get("training_state", {}))


def load_ema(path) -> dict | None:
    return torch.load(path, map_location="cpu", weights_only=False).get("ema_params")


def export_inference_checkpoint(model: nn.Module, path, ema_params: dict | None = None,
                                nn_dtype: torch.dtype = torch.bfloat16, meta: dict | None = None) -> None:
    """Parameters (EMA copies when given) in ``nn_dtype``; buffers (normalisation
    statistics, reference profiles, interpolation matrices) keep their dtype."""
    raw = _unwrap(model)
    sd = {k: v for k, v in raw.state_dict().items()}
    params = dict(raw.named_parameters())
    if ema_params is not None:
        sd.update({k: v for k, v in ema_params.items() if k in sd})
    conv = {}
    for k, v in sd.items():
        v = v.detach().cpu()
        conv[k] = v.to(nn_dtype) if (k in params and v.is_floating_point()) else v
    _atomic_save({"model_state_dict": conv, "format": "inference", "meta": dict(meta or {})}, pathlib.Path(path))


def load_inference_checkpoint(path, model: nn.Module, strict: bool = False) -> None:
    ckpt = torch.load(path, map_location="cpu", weights_only=True)
    sd = ckpt.get("model_state_dict", ckpt)
    target = _unwrap(model).state_dict()
    sd = {k: v.to(target[k].dtype) if k in target and v.is_floating_point() else v for k, v in sd.items()}
    _unwrap(model).load_state_dict(sd, strict=strict)
