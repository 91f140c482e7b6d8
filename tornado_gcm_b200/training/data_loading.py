"""Gap-tolerant trajectory windows and data loaders (reference ``training/data_loading.py:20-195``).

Windows: the time axis is split at gaps (Δt > 1.5 × median); segments at
least W·(1−r_max) long give full sliding windows (weight 1), segments of
at least W/2 give shorter windows with weight 0.5.  The loader pins host
memory so the trainer's host→device copies are asynchronous.
"""

from __future__ import annotations

import dataclasses
from typing import Optional

import numpy as np
import torch
from torch.utils.data import DataLoader, Dataset


@dataclasses.dataclass
class TemporalWindow:
    start_idx: int
    length: int
    weight: float = 1.0


def find_contiguous_segments(times: np.ndarray, gap_factor: float = 1.5) -> list:
    times = np.asarray(times)
    if len(times) < 2:
        return [(0, len(times))]
    dt = np.diff(times.astype(np.float64))
    gaps = np.nonzero(dt > gap_factor * np.median(dt))[0]
    bounds = [0] + [int(i) + 1 for i in gaps] + [len(times)]
    return [(bounds[i], bounds[i + 1]) for i in range(len(bounds) - 1)]


def gap_tolerant_sampling(times: np.ndarray, window_length: int, max_missing_rate: float = 0.05,
                          gap_factor: float = 1.5) -> list:
    full = int(window_length * (1.0 - max_missing_rate))
    short = window_length // 2
    out = []
    for a, b in find_contiguous_segments(times, gap_factor):
        n = b - a
        if n >= full:
            out += [TemporalWindow(i, window_length, 1.0) for i in range(a, b - window_length + 1)]
        elif n >= short:
            out += [TemporalWindow(i, n, 0.5) for i in range(a, b - n + 1)]
    return out


class TrajectoryDataset(Dataset):
    def __init__(self, data: dict, times: np.ndarray, window_length: int, max_missing_rate: float = 0.05):
        self.data = data
        self.times = times
        self.windows = gap_tolerant_sampling(times, window_length, max_missing_rate)
        w = np.array([x.weight for x in self.windows], dtype=np.float64)
        self._weights = w / w.sum() if len(w) else w

    def __len__(self) -> int:
        return len(self.windows)

    def __getitem__(self, idx: int) -> dict:
        win = self.windows[idx]
        sl = slice(win.start_idx, win.start_idx + win.length)
        out = {k: torch.from_numpy(np.ascontiguousarray(v[sl])).float() for k, v in self.data.items()}
        out["weight"] = torch.tensor(win.weight, dtype=torch.float32)
        return out


class WeightedRandomSampler(torch.utils.data.Sampler):
    def __init__(self, dataset: TrajectoryDataset, num_samples: Optional[int] = None, seed: int = 0):
        self.weights = torch.from_numpy(dataset._weights).double()
        self.num_samples = num_samples or len(dataset)
        self.gen = torch.Generator().manual_seed(seed)

    def __iter__(self):
        return iter(torch.multinomial(self.weights, self.num_samples, replacement=True,
                                      generator=self.gen).tolist())

    def __len__(self) -> int:
        return self.num_samples


def _collate(batch: list) -> dict:
    lengths = {b["weight"].item() for b in batch}
    keys = batch[0].keys()
    return {k: torch.stack([b[k] for b in batch]) for k in keys} if len(lengths) <= 2 else batch


def build_dataloader(data: dict, times: np.ndarray, window_length: int, batch_size: int, num_workers: int = 0,
                     max_missing_rate: float = 0.05, use_distributed_sampler: bool = False,
                     pin_memory: bool = True, seed: int = 0) -> DataLoader:
    ds = TrajectoryDataset(data, times, window_length, max_missing_rate)
    sampler = None
    if use_distributed_sampler:
        from tornado_gcm_b200.parallel.ddp import build_distributed_sampler

        sampler = build_distributed_sampler(ds, shuffle=True, seed=seed)
    if sampler is None:
        sampler = WeightedRandomSampler(ds, seed=seed)
    return DataLoader(ds, batch_size=batch_size, sampler=sampler, num_workers=num_workers,
                      pin_memory=pin_memory and torch.cuda.is_available(), drop_last=True)
