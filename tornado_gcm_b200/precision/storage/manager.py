"""Variable-level mixed-precision storage — reference ``precision/storage/manager.py:34-227``.

Critical variables are stored exactly, the rest through the lossy codec
(mode ``"mixed"``); ``"exact"`` / ``"lossy"`` force one codec.  On-disk
layout (the same as the reference, so stores are interchangeable):
``<dir>/<name>[_s<step>].bin`` plus ``_metadata[_s<step>].json`` with codec,
shape, dtype, original dtype, compressor and size per variable.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any, Optional

import torch

from tornado_gcm_b200.precision.storage.codec import ExactCodec, LossyCodec, _EncodedTensor

_RATIO = {"zstd": 0.7, "lz4": 0.8, "zlib": 0.75, "lzma": 0.65}


class SDAStorageManager:
    def __init__(self, config=None) -> None:
        if config is None:
            from tornado_gcm_b200.precision.sda import StorageConfig

            config = StorageConfig()
        self._config = config
        self._exact = ExactCodec(config.compressor, config.compression_level)
        self._lossy = LossyCodec(config.lossy_dtype, config.compressor, config.compression_level)

    @property
    def config(self):
        return self._config

    def _is_critical(self, name: str) -> bool:
        mode = self._config.mode
        if mode == "exact":
            return True
        if mode == "lossy":
            return False
        if name in self._config.critical_variables:
            return True
        if name in self._config.non_critical_variables:
            return False
        return True

    @staticmethod
    def _flatten(variables: dict) -> dict[str, torch.Tensor]:
        flat = {}
        for k, v in variables.items():
            if isinstance(v, dict):
                for kk, vv in v.items():
                    flat[f"{k}.{kk}"] = vv
            else:
                flat[k] = v
        return flat

    def write(self, variables: dict, output_dir: str, step: Optional[int] = None) -> dict[str, Any]:
        out = Path(output_dir)
        out.mkdir(parents=True, exist_ok=True)
        suffix = f"_s{step}" if step is not None else ""
        meta, summary = {}, {}
        for name, t in self._flatten(variables).items():
            crit = self._is_critical(name) and self._is_critical(name.split(".")[0])
            enc = self._exact.encode(t, self._config.exact_dtype if t.is_floating_point() else None) if crit \
                else self._lossy.encode(t, verify=True)
            (out / f"{name}{suffix}.bin").write_bytes(enc.data)
            meta[name] = {"codec": "exact" if crit else "lossy", "shape": list(enc.shape), "dtype": enc.dtype_name,
                          "original_dtype": enc.original_dtype_name, "compressor": enc.compressor,
                          "size_bytes": len(enc.data)}
            summary[name] = {"codec": meta[name]["codec"], "size_bytes": len(enc.data),
                             "original_bytes": t.nelement() * t.element_size()}
        with open(out / f"_metadata{suffix}.json", "w", encoding="utf-8") as fh:
            json.dump(meta, fh, indent=2)
        return summary

    def read(self, input_dir: str, step: Optional[int] = None,
             restore_dtype: torch.dtype = torch.float32) -> dict[str, torch.Tensor]:
        inp = Path(input_dir)
        suffix = f"_s{step}" if step is not None else ""
        with open(inp / f"_metadata{suffix}.json", encoding="utf-8") as fh:
            meta = json.load(fh)
        res = {}
        for name, m in meta.items():
            enc = _EncodedTensor((inp / f"{name}{suffix}.bin").read_bytes(), tuple(m["shape"]), m["dtype"],
                                 m["original_dtype"], m["compressor"])
            t = self._exact.decode(enc) if m["codec"] == "exact" else self._lossy.decode(enc)
            res[name] = t.to(restore_dtype) if t.is_floating_point() else t
        return res

    def estimate_storage(self, variables: dict, num_steps: int = 1) -> dict[str, Any]:
        eb = torch.tensor([], dtype=self._config.exact_dtype).element_size()
        lb = torch.tensor([], dtype=self._config.lossy_dtype).element_size()
        ratio = _RATIO.get(self._exact._compressor, 1.0)
        per, tot_e, tot_l = {}, 0, 0
        for name, shape in variables.items():
            n = 1
            for s in shape:
                n *= int(s)
            crit = self._is_critical(name)
            raw = n * (eb if crit else lb) * num_steps
            est = int(raw * ratio)
            per[name] = {"codec": "exact" if crit else "lossy", "raw_bytes": raw, "estimated_bytes": est}
            if crit:
                tot_e += est
            else:
                tot_l += est
        return {"per_variable": per, "total_exact_bytes": tot_e, "total_lossy_bytes": tot_l,
                "total_bytes": tot_e + tot_l, "total_mb": round((tot_e + tot_l) / 2 ** 20, 2)}
