"""Production inference — reference ``inference/production.py:29-414``.

* :class:`InferenceRunner` — chunked forecast with a NaN guard that rolls back
  to the last host checkpoint, optional forcing provider and output writer;
* :class:`EnsembleRunner` — ensemble members.  Members that share an initial
  state run as ONE batch (the member index is the leading batch dimension of
  every kernel) with per-member Gaussian-random-field perturbations, instead
  of the reference's sequential member loop;
* writers: :class:`NumpyWriter` (in memory, ``.npz``), :class:`StoreWriter`
  (the mixed-precision storage manager's directory store, one step per
  record) and :class:`AsyncStoreWriter` (the same on a background thread).
  ``ZarrWriter`` / ``AsyncZarrWriter`` are the store writers under the
  reference's names: this image has no zarr package, so the layout is the
  storage manager's ``.bin`` + ``_metadata.json`` files;
* :func:`load_initial_condition` / :func:`save_forecast` — the functions the
  reference CLI calls but does not define (``cli.py:115-124``).
"""

from __future__ import annotations

import dataclasses
import logging
import pathlib
import queue
import threading
from typing import Any, Callable, Optional, Sequence

import numpy as np
import torch

logger = logging.getLogger(__name__)


@dataclasses.dataclass
class InferenceConfig:
    outer_steps: int = 100
    inner_steps: int = 1
    chunk_size: int = 50
    nan_guard: bool = True
    checkpoint_interval: int = 0
    output_path: Optional[str | pathlib.Path] = None
    output_variables: Optional[Sequence[str]] = None


def _has_nan(chunk: list) -> bool:
    for s in chunk:
        ts = s.tensors() if hasattr(s, "tensors") else (list(s.values()) if isinstance(s, dict) else [s])
        for t in ts:
            if torch.is_tensor(t) and t.is_floating_point() and bool(torch.isnan(t).any()):
                return True
    return False


def _clone_state(state):
    if hasattr(state, "tree_map"):
        return state.tree_map(lambda t: t.detach().clone())
    if isinstance(state, dict):
        return {k: v.detach().clone() if torch.is_tensor(v) else v for k, v in state.items()}
    return state


def _state_to_dict(state) -> dict[str, np.ndarray]:
    if isinstance(state, dict):
        return {k: v.detach().float().cpu().numpy() for k, v in state.items() if torch.is_tensor(v)}
    out = {"vorticity": state.vorticity, "divergence": state.divergence,
           "temperature_variation": state.temperature_variation,
           "log_surface_pressure": state.log_surface_pressure}
    out.update({f"tracers.{k}": v for k, v in state.tracers.items()})
    return {k: v.detach().float().cpu().numpy() for k, v in out.items()}


class InferenceRunner:
    """Chunked forecast with NaN rollback and optional writer."""

    def __init__(self, engine, config: InferenceConfig, forcing_fn: Optional[Callable[[float], dict]] = None,
                 post_process_fn: Optional[Callable] = None):
        self.engine = engine
        self.config = config
        self.forcing_fn = forcing_fn
        self.post_process_fn = post_process_fn
        self._last_checkpoint: Optional[tuple[int, Any]] = None

    @torch.no_grad()
    def run(self, initial_state: Any, writer=None) -> list:
        cfg = self.config
        out, state, step, retries = [], initial_state, 0, 0
        while step < cfg.outer_steps:
            n = min(cfg.chunk_size, cfg.outer_steps - step)
            if cfg.checkpoint_interval > 0 and step % cfg.checkpoint_interval == 0:
                self._last_checkpoint = (step, _clone_state(state))
            forcings = None
            if self.forcing_fn is not None:
                forcings = self.forcing_fn(getattr(state, "sim_time", float(step)))
            state, chunk = self.engine._unroll(state, n, cfg.inner_steps, forcings, self.post_process_fn)
            if cfg.nan_guard and _has_nan(chunk):
                retries += 1
                logger.warning("NaN in outputs of steps %d..%d", step + 1, step + n)
                if self._last_checkpoint is not None and retries <= 3:
                    step, saved = self._last_checkpoint
                    state = _clone_state(saved)
                    out = out[:step]
                    continue
                logger.error("NaN detected and no checkpoint to roll back to")
                break
            if writer is not None:
                writer.write_chunk(chunk, start_step=step)
            out.extend(chunk)
            step += n
        return out


class EnsembleRunner:
    """Ensemble members as one batch (default) or one after another.

    ``perturb(state, generator)`` adds a member's perturbation; by default a
    Gaussian random field (σ = ``perturbation_std`` in model units,
    correlation length ``correlation_km``) is added to temperature and
    vorticity.  With ``batched`` the members are stacked on the leading
    dimension of the initial state (which must have batch size 1).
    """

    def __init__(self, runner: InferenceRunner, n_members: int = 10, base_seed: int = 42, batched: bool = True,
                 perturb: Optional[Callable] = None, perturbation_std: float = 0.0,
                 correlation_km: float = 1000.0):
        self.runner = runner
        self.n_members = n_members
        self.base_seed = base_seed
        self.batched = batched
        self.perturb = perturb
        self.perturbation_std = perturbation_std
        self.correlation_km = correlation_km

    def _default_perturb(self):
        if self.perturbation_std <= 0:
            return None
        from tornado_gcm_b200.neural.stochastic import GaussianRandomField

        grid = self.runner.engine.model.config.coords.horizontal
        grf = GaussianRandomField(grid, correlation_length_km=self.correlation_km, variance=1.0)

        def perturb(state, gen):
            def add(t):
                noise = grf.sample_modal(t.shape[:-2], generator=gen, device=t.device, dtype=t.dtype)
                return t + self.perturbation_std * noise
            return type(state)(add(state.vorticity), state.divergence, add(state.temperature_variation),
                               state.log_surface_pressure, state.tracers, state.sim_time)

        return perturb

    @torch.no_grad()
    def run(self, initial_state: Any, writer=None) -> list:
        perturb = self.perturb or self._default_perturb()
        dev = initial_state.vorticity.device
        if self.batched:
            members = initial_state.tree_map(
                lambda t: t.expand(self.n_members, *t.shape[1:]).contiguous() if t.shape[0] == 1 else t)
            if perturb is not None:
                gen = torch.Generator(device=dev).manual_seed(self.base_seed)
                members = perturb(members, gen)
            traj = self.runner.run(members, writer=writer)
            return [[s.tree_map(lambda t, i=i: t[i:i + 1]) for s in traj] for i in range(self.n_members)]
        out = []
        for m in range(self.n_members):
            gen = torch.Generator(device=dev).manual_seed(self.base_seed + m)
            s0 = perturb(initial_state, gen) if perturb is not None else initial_state
            out.append(self.runner.run(s0, writer=writer))
        return out


class NumpyWriter:
    """Collects outputs in host memory; ``finalize()`` stacks them per variable."""

    def __init__(self, output_variables: Optional[Sequence[str]] = None):
        self.output_variables = output_variables
        self._buf: dict[str, list] = {}

    def write_chunk(self, chunk: list, start_step: int = 0) -> None:
        for s in chunk:
            for k, v in _state_to_dict(s).items():
                if self.output_variables is None or k in self.output_variables:
                    self._buf.setdefault(k, []).append(v)

    def finalize(self) -> dict[str, np.ndarray]:
        return {k: np.stack(v) for k, v in self._buf.items()}

    def save(self, path: str | pathlib.Path) -> None:
        np.savez(path, **self.finalize())


class StoreWriter:
    """One record per step through :class:`SDAStorageManager` (exact/lossy per variable)."""

    def __init__(self, path: str | pathlib.Path, output_variables: Optional[Sequence[str]] = None,
                 storage_config=None):
        from tornado_gcm_b200.precision.storage import SDAStorageManager

        self.path = pathlib.Path(path)
        self.output_variables = output_variables
        self.manager = SDAStorageManager(storage_config)
        self.steps_written: list[int] = []

    def _write_one(self, step: int, state) -> None:
        d = {k: torch.from_numpy(v) for k, v in _state_to_dict(state).items()
             if self.output_variables is None or k in self.output_variables}
        self.manager.write(d, str(self.path), step=step)
        self.steps_written.append(step)

    def write_chunk(self, chunk: list, start_step: int = 0) -> None:
        for i, s in enumerate(chunk):
            self._write_one(start_step + i, s)


class AsyncStoreWriter(StoreWriter):
    """:class:`StoreWriter` on a background thread (host copies made eagerly)."""

    def __init__(self, path, output_variables=None, storage_config=None, max_queue: int = 8):
        super().__init__(path, output_variables, storage_config)
        self._q: queue.Queue = queue.Queue(maxsize=max_queue)
        self._err: Optional[BaseException] = None
        self._t = threading.Thread(target=self._loop, daemon=True)
        self._t.start()

    def _loop(self):
        while True:
            item = self._q.get()
            if item is None:
                self._q.task_done()
                return
            try:
                self._write_one(*item)
            except BaseException as exc:  # pragma: no cover - surfaced in flush
                self._err = exc
            finally:
                self._q.task_done()

    def write_chunk(self, chunk: list, start_step: int = 0) -> None:
        for i, s in enumerate(chunk):
            self._q.put((start_step + i, _clone_state(s.tree_map(lambda t: t.cpu())
                                                      if hasattr(s, "tree_map") else s)))

    def flush(self) -> None:
        self._q.join()
        if self._err is not None:
            raise self._err

    def close(self) -> None:
        self.flush()
        self._q.put(None)
        self._t.join(timeout=30)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


ZarrWriter = StoreWriter
AsyncZarrWriter = AsyncStoreWriter


def load_initial_condition(path: str | pathlib.Path, device: str | torch.device = "cpu") -> dict:
    """Normalised data fields from a ``.pt`` (dict of tensors) or ``.npz`` file.

    Keys are the data fields of the encoder (``u, v, t, q, z, clwc, ciwc`` on
    pressure levels); an optional ``forcings`` entry (``.pt``) or ``forcing.*``
    keys (``.npz``) carry the forcing fields.
    """
    path = pathlib.Path(path)
    if path.suffix == ".npz":
        raw = dict(np.load(path))
        data = {k: torch.as_tensor(v) for k, v in raw.items() if not k.startswith("forcing.")}
        forc = {k[len("forcing."):]: torch.as_tensor(v) for k, v in raw.items() if k.startswith("forcing.")}
        if forc:
            data["forcings"] = forc
    else:
        data = torch.load(path, map_location="cpu", weights_only=True)
    out = {}
    for k, v in data.items():
        if isinstance(v, dict):
            out[k] = {kk: vv.to(device).float() for kk, vv in v.items()}
        else:
            out[k] = v.to(device).float()
    return out


def save_forecast(trajectory: list, path: str | pathlib.Path) -> None:
    """``.npz`` (stacked per variable) for a ``.npz`` path, else a storage-manager directory."""
    path = pathlib.Path(path)
    if path.suffix == ".npz":
        w = NumpyWriter()
        w.write_chunk(trajectory)
        w.save(path)
        return
    w = StoreWriter(path)
    w.write_chunk(trajectory)
