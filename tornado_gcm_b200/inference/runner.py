"""Mixed-precision inference engine — reference ``inference/runner.py:33-370``.

:class:`MPInference` runs autoregressive rollouts of a
:class:`~tornado_gcm_b200.models.api.NeuralGCMModel` (Z3 BF16 towers, Z1 TF32
transforms, Z2 FP64-accumulated fixer).  On CUDA every outer step can be
replayed from a captured CUDA graph (:class:`FusedAdvanceKernel`), and
streamed outputs leave the GPU through pinned host buffers with
non-blocking copies.

Beyond the reference API (``run``, ``run_chunked``, ``run_streaming``,
``audit``) this module provides what the reference CLI calls but never
defines: :meth:`MPInference.from_state_dict` and :meth:`MPInference.rollout`.
"""

from __future__ import annotations

import logging
from concurrent.futures import Future, ThreadPoolExecutor
from typing import Any, Callable, Optional

import torch
import torch.nn as nn

from tornado_gcm_b200.precision.policy import PrecisionPolicy

logger = logging.getLogger(__name__)


def _offload(obj: Any, device: str | torch.device = "cpu", async_transfer: bool = True) -> Any:
    """Move a State / tensor to ``device``; CUDA → CPU copies go through pinned memory."""
    dev = torch.device(device)

    def move(t: torch.Tensor) -> torch.Tensor:
        if dev.type == "cpu" and t.is_cuda and async_transfer:
            out = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
            out.copy_(t, non_blocking=True)
            return out
        return t.to(dev, non_blocking=async_transfer)

    if hasattr(obj, "tree_map"):
        return obj.tree_map(move)
    if isinstance(obj, torch.Tensor):
        return move(obj)
    if isinstance(obj, dict):
        return {k: _offload(v, device, async_transfer) for k, v in obj.items()}
    return obj


def _map_tensors(obj: Any, fn: Callable) -> Any:
    if hasattr(obj, "tree_map"):
        return obj.tree_map(fn)
    if isinstance(obj, (torch.Tensor, Future)):
        return fn(obj)
    if isinstance(obj, dict):
        return {k: _map_tensors(v, fn) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_map_tensors(v, fn) for v in obj)
    return obj


class HostOffloader:
    """Device → host copies of forecast outputs, overlapped with later steps.

    ``submit(obj)`` issues, for every CUDA tensor of ``obj``, a non-blocking
    copy into a pinned staging block and records an event; a worker thread
    waits for the event and moves the block into ordinary host memory.  The
    staging block is then freed, and PyTorch's caching host allocator hands it
    to a later copy once that copy's predecessor has completed — after the
    first steps no new memory is page-locked (allocating fresh pinned memory
    for every output costs more than the copy itself).  ``resolve`` waits and
    returns the host objects in the structure that was submitted.
    """

    def __init__(self, workers: int = 2):
        self._pool = ThreadPoolExecutor(max_workers=workers, thread_name_prefix="tgcm-offload")

    def _one(self, t):
        if not (isinstance(t, torch.Tensor) and t.is_cuda):
            done: Future = Future()
            done.set_result(t)
            return done
        stage = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        stage.copy_(t, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()

        def finish(stage=stage, ev=ev):
            ev.synchronize()
            out = torch.empty(stage.shape, dtype=stage.dtype)  # pageable
            out.copy_(stage)
            return out  # the pinned block returns to the allocator's cache

        return self._pool.submit(finish)

    def submit(self, obj: Any) -> Any:
        return _map_tensors(obj, self._one)

    def resolve(self, obj: Any) -> Any:
        return _map_tensors(obj, lambda f: f.result() if isinstance(f, Future) else f)

    def close(self) -> None:
        self._pool.shutdown(wait=True)


def _has_nan(obj: Any) -> bool:
    if hasattr(obj, "tensors"):
        return any(bool(torch.isnan(t).any()) for t in obj.tensors() if t.is_floating_point())
    if isinstance(obj, torch.Tensor):
        return bool(torch.isnan(obj).any())
    if isinstance(obj, dict):
        return any(_has_nan(v) for v in obj.values())
    return False


def auto_estimate_chunk_size(model: nn.Module, sample_state: Any, headroom: float = 0.6) -> int:
    """Largest power of two (≤ 256) of states that fits ``headroom`` of free device memory."""
    try:
        device = next(model.parameters()).device
    except StopIteration:
        return 64
    if device.type != "cuda":
        return 64
    state = sample_state.state if hasattr(sample_state, "state") else sample_state
    nbytes = sum(t.numel() * t.element_size() for t in state.tensors()) if hasattr(state, "tensors") else 0
    if nbytes == 0:
        return 64
    free, _ = torch.cuda.mem_get_info(device)
    raw = max(1, int(free * headroom) // nbytes)
    chunk = 1
    while chunk * 2 <= min(raw, 256):
        chunk *= 2
    return chunk


class MPInference:
    """Mixed-precision inference engine.

    ``model`` is a :class:`NeuralGCMModel` or a
    :class:`~tornado_gcm_b200.models.builders.HybridGCM` (encoder → model →
    decoder).  With ``use_graph`` (default on CUDA) every outer-step physics
    step replays a captured CUDA graph.
    """

    def __init__(self, model: nn.Module, policy: Optional[PrecisionPolicy] = None, monitor=None,
                 use_graph: bool = True):
        self.hybrid = model if hasattr(model, "encoder") and hasattr(model, "physics_steps_per_output") else None
        self.model = self.hybrid.model if self.hybrid is not None else model
        self.policy = policy or getattr(self.model, "policy", None) or PrecisionPolicy()
        self.monitor = monitor
        (self.hybrid or self.model).eval()
        self.policy.apply_tf32_setting()
        self.use_graph = use_graph
        self._kernel = None

    # ── construction from a checkpoint ──
    @classmethod
    def from_state_dict(cls, state_dict: dict, device: str | torch.device = "cuda", resolution: Optional[str] = None,
                        policy: Optional[PrecisionPolicy] = None, **kwargs) -> "MPInference":
        """Build the hybrid model of the checkpoint's resolution and load its weights.

        ``state_dict`` is either an inference checkpoint written by
        :func:`tornado_gcm_b200.training.checkpointing.export_inference_checkpoint`
        (``{"model": ..., "meta": {"resolution": ...}}``) or a bare model state dict
        (then ``resolution`` names the architecture, default ``"2.8deg"``).
        """
        from tornado_gcm_b200.models.builders import build_hybrid_gcm

        meta = state_dict.get("meta", {}) if isinstance(state_dict, dict) else {}
        weights = state_dict.get("model", state_dict.get("model_state_dict", state_dict))
        res = resolution or meta.get("resolution", "2.8deg")
        gcm, _ = build_hybrid_gcm(res, device, policy=policy)
        missing, unexpected = gcm.load_state_dict({k: v for k, v in weights.items()}, strict=False)
        if unexpected:
            logger.warning("checkpoint entries not used by the %s model: %s", res, unexpected[:8])
        if missing:
            logger.warning("model entries missing from the checkpoint: %s", missing[:8])
        return cls(gcm, policy=policy, **kwargs)

    # ── stepping ──
    def _step_fn(self) -> Callable:
        if self.use_graph and torch.cuda.is_available():
            if self._kernel is None:
                from tornado_gcm_b200.precision.accelerator.graphed_step import FusedAdvanceKernel

                self._kernel = FusedAdvanceKernel(self.model, self.policy)
            return self._kernel
        return self.model.step

    def _inner(self, inner_steps: Optional[int]) -> int:
        if inner_steps is not None:
            return int(inner_steps)
        if self.hybrid is not None:
            return int(self.hybrid.physics_steps_per_output)
        return int(getattr(self.model.config, "inner_steps", 1))

    def _forcings(self, forcings):
        if forcings is None or self.hybrid is None:
            return forcings
        return self.hybrid.normalize_forcings(forcings)

    @torch.no_grad()
    def _unroll(self, state, n: int, inner_steps: Optional[int], forcings, post_process_fn=None):
        step = self._step_fn()
        f = self._forcings(forcings)
        inner = self._inner(inner_steps)
        out = []
        for _ in range(n):
            for _ in range(inner):
                state = step(state, f)
            out.append(post_process_fn(state) if post_process_fn is not None else state)
        return state, out

    @torch.no_grad()
    def run(self, initial_state: Any, outer_steps: int, inner_steps: Optional[int] = None,
            post_process_fn: Optional[Callable] = None, forcings: Optional[dict] = None) -> list:
        _, traj = self._unroll(initial_state, outer_steps, inner_steps, forcings, post_process_fn)
        return traj

    @torch.no_grad()
    def run_chunked(self, initial_state: Any, total_steps: int, chunk_size: int = 100, inner_steps: int = 1,
                    post_process_fn: Optional[Callable] = None, forcings: Optional[dict] = None) -> list:
        results, state, remaining = [], initial_state, total_steps
        while remaining > 0:
            n = min(chunk_size, remaining)
            state, chunk = self._unroll(state, n, inner_steps, forcings, post_process_fn)
            results.extend(chunk)
            remaining -= n
        return results

    @torch.no_grad()
    def run_streaming(self, initial_state: Any, outer_steps: int, inner_steps: int = 1,
                      forcings: Optional[dict] = None, *, chunk_size: int = 1, keep_steps: Optional[set] = None,
                      on_step_fn: Optional[Callable[[int, Any], None]] = None,
                      post_process_fn: Optional[Callable] = None, offload_device: str | torch.device = "cpu",
                      async_offload: bool = True, nan_guard: bool = False,
                      checkpoint_interval: int = 0) -> tuple[Any, list]:
        """Chunked rollout with per-step offload; returns ``(final_state, [(step, saved), ...])``.

        ``keep_steps`` are 1-based outer-step indices to keep (None keeps all).
        With ``nan_guard`` a NaN in an output rolls the run back to the last
        host checkpoint (taken every ``checkpoint_interval`` outer steps), at
        most three times.
        """
        saved: list = []
        state = initial_state
        step = 0
        ckpt = None
        retries = 0
        device = state.vorticity.device if hasattr(state, "vorticity") else None
        off = (HostOffloader() if async_offload and torch.device(offload_device).type == "cpu"
               and torch.cuda.is_available() else None)
        keep = (lambda o: off.submit(o)) if off is not None else (lambda o: _offload(o, offload_device, async_offload))
        while step < outer_steps:
            if checkpoint_interval > 0 and step % checkpoint_interval == 0:
                ckpt = (step, _offload(state, "cpu", False))
            n = min(max(1, chunk_size), outer_steps - step)
            state, chunk = self._unroll(state, n, inner_steps, forcings, post_process_fn)
            reverted = False
            for i, out in enumerate(chunk):
                gstep = step + i + 1
                if nan_guard and _has_nan(out):
                    logger.warning("NaN detected at outer step %d", gstep)
                    retries += 1
                    if ckpt is not None and retries <= 3:
                        step = ckpt[0]
                        state = _offload(ckpt[1], device, False) if device is not None else ckpt[1]
                        saved = [(s, v) for s, v in saved if s <= step]
                        reverted = True
                        break
                    raise RuntimeError(f"NaN at step {gstep} (retries={retries}, no viable checkpoint)")
                if on_step_fn is not None:
                    on_step_fn(gstep, out)
                if keep_steps is None or gstep in keep_steps:
                    saved.append((gstep, keep(out)))
            if reverted:
                continue
            step += n
        if off is not None:
            saved = [(g, off.resolve(v)) for g, v in saved]
            off.close()
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        return state, saved

    # ── data-space rollout (the CLI entry point) ──
    @torch.no_grad()
    def rollout(self, initial_state: Any, steps: int, forcings: Optional[dict] = None, decode: bool = True,
                offload: bool = False) -> list:
        """``steps`` outer (6-h) steps from a State or, with an encoder, from normalised data fields.

        Returns the decoded data fields per step (when the engine wraps a model
        with a decoder and ``decode``), else the model States.
        """
        state = initial_state
        f = forcings
        if self.hybrid is not None and isinstance(initial_state, dict):
            f = forcings if forcings is not None else {}
            state = self.hybrid.encoder(initial_state, self.hybrid.normalize_forcings(f))
        dec = None
        if decode and self.hybrid is not None:
            nf = self.hybrid.normalize_forcings(f) if f else {}
            dec = (lambda s: self.hybrid.decoder(s, nf))
        off = HostOffloader() if offload and torch.cuda.is_available() else None
        post = dec
        if off is not None:  # each 6-h output leaves the GPU while the next steps run
            post = (lambda s: off.submit(dec(s) if dec is not None else s))
        _, traj = self._unroll(state, steps, None, f, post)
        if off is not None:
            traj = [off.resolve(t) for t in traj]
            off.close()
        elif offload:
            traj = [_offload(t, "cpu", False) for t in traj]
        return traj

    def audit(self) -> dict:
        if self.monitor is None:
            return {}
        return self.monitor.summary() if hasattr(self.monitor, "summary") else {}

    def stats(self) -> dict:
        return self._kernel.stats() if self._kernel is not None else {"graph": False}
