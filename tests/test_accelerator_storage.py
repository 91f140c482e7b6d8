"""Accelerator registry / torch oracles and the mixed-precision storage manager (CPU)."""

import numpy as np
import pytest
import torch

from tornado_gcm_b200.precision.accelerator import registry, reductions, sm100_sht
from tornado_gcm_b200.precision.sda import StorageConfig
from tornado_gcm_b200.precision.storage import ExactCodec, LossyCodec, SDAStorageManager


def test_registry_priorities_and_backend_filter():
    reg = registry.AcceleratorRegistry()
    reg.register("op", lambda: "low", priority=1, backend="torch")
    reg.register("op", lambda: "high", priority=9, backend="sm100")
    assert reg.get("op")() == "high"
    assert reg.get("op", backend="torch")() == "low"
    assert reg.available("op") == ["sm100", "torch"]
    assert "op" in reg and len(reg) == 1
    with pytest.raises(KeyError):
        reg.get("missing")
    g = registry.get_global_registry()
    for name in ("sht_legendre_inverse", "sht_legendre_forward", "sphere_integrate", "spectral_norm",
                 "conservation_fix"):
        assert g.available(name) == ["sm100", "torch"]


def test_torch_oracles():
    rng = np.random.default_rng(0)
    basis = rng.standard_normal((5, 4, 3))
    x = torch.randn(2, 5, 3)
    ref = np.einsum("mjl,bml->bmj", basis, x.double().numpy())
    np.testing.assert_allclose(sm100_sht.sht_legendre_inverse(basis, x).numpy(), ref, rtol=1e-5, atol=1e-5)
    y = torch.randn(2, 5, 4)
    ref = np.einsum("mjl,bmj->bml", basis, y.double().numpy())
    np.testing.assert_allclose(sm100_sht.sht_legendre_forward(basis, y).numpy(), ref, rtol=1e-5, atol=1e-5)
    z = torch.randn(3, 6, 4)
    w = torch.rand(4, dtype=torch.float64)
    np.testing.assert_allclose(reductions.sphere_integrate(z, w).numpy(),
                               (z.double() * w).sum(dim=(-2, -1)).numpy(), rtol=1e-12)
    acc = reductions.KahanAccumulator((2,))
    for _ in range(1000):
        acc.add(torch.tensor([0.1, 1e-8], dtype=torch.float64))
    np.testing.assert_allclose(acc.value().numpy(), [100.0, 1e-5], rtol=1e-12)


@pytest.mark.parametrize("compressor", ["zstd", "zlib", "lzma", "none"])
def test_codecs_roundtrip(compressor):
    t = torch.randn(3, 17, 9, dtype=torch.float32)
    ex = ExactCodec(compressor)
    enc = ex.encode(t)
    torch.testing.assert_close(ex.decode(enc), t, rtol=0, atol=0)
    lo = LossyCodec(torch.bfloat16, compressor)
    enc = lo.encode(t)
    back = lo.decode(enc, restore_dtype=torch.float32)
    torch.testing.assert_close(back, t.to(torch.bfloat16).float(), rtol=0, atol=0)


def test_storage_manager_mixed_routing(tmp_path):
    mgr = SDAStorageManager(StorageConfig(mode="mixed", compressor="zlib"))
    v = {"vorticity": torch.randn(2, 4, 5), "tracers": {"q": torch.randn(2, 4, 5)}}
    summ = mgr.write(v, str(tmp_path), step=3)
    assert summ["vorticity"]["codec"] == "exact" and summ["tracers.q"]["codec"] == "lossy"
    back = mgr.read(str(tmp_path), step=3)
    torch.testing.assert_close(back["vorticity"], v["vorticity"], rtol=0, atol=0)
    torch.testing.assert_close(back["tracers.q"], v["tracers"]["q"].to(torch.bfloat16).float(), rtol=0, atol=0)
    est = mgr.estimate_storage({"vorticity": (32, 127, 65), "tracers": (32, 127, 65)}, num_steps=10)
    assert est["total_exact_bytes"] > est["total_lossy_bytes"] > 0
