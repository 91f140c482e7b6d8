"""Sparse / split-precision spectral storage and the split-precision transform (CPU)."""

import numpy as np
import torch

from tornado_gcm_b200.core import spherical_harmonic as sh
from tornado_gcm_b200.precision import sparse


def test_triangular_mask_matches_grid_mask():
    g = sh.Grid.T21()
    np.testing.assert_array_equal(sparse.triangular_mask(*g.modal_shape).numpy(), g.mask)
    n_valid, n_total = sparse.count_structural_zeros(*g.modal_shape)
    assert n_valid == int(g.mask.sum()) and n_total == g.mask.size


def test_sparse_state_modes_roundtrip():
    g = sh.Grid.T21()
    x = torch.randn(2, 3, *g.modal_shape) * torch.as_tensor(g.mask)
    for mode in ("structural", "adaptive", "mixed"):
        st = sparse.SpectralSparseState.from_state_dict({"vorticity": x, "scalar": torch.tensor(1.0)},
                                                        sparse.SparseConfig(enabled=True, mode=mode))
        back = st.to_dense_dict()["vorticity"]
        if mode == "mixed":
            cut = st.fields["vorticity"].cutoff_l
            torch.testing.assert_close(back[..., :cut], x[..., :cut])
            torch.testing.assert_close(back[..., cut:], x[..., cut:].bfloat16().float())
            assert st.memory_savings > 0.2
        elif mode == "structural":
            torch.testing.assert_close(back, x)
    assert 0 < sparse.memory_savings_ratio(*g.modal_shape, mode="structural") < 1


def test_split_precision_transform_matches_dense():
    g = sh.Grid.T21(precision="highest")
    p = g.spherical_harmonics.legendre_table
    basis = np.concatenate([p[:1], np.repeat(p[1:], 2, axis=0)], axis=0)
    tr = sparse.SparseSpectralTransform(basis, sparse.SparseConfig(mode="mixed", high_order_cutoff=0.5),
                                        fourier_basis=g.spherical_harmonics.basis.f)
    m, l = g.modal_mesh
    x = torch.tensor(np.random.default_rng(0).standard_normal(g.modal_shape) * g.mask * (1.0 + l) ** -1.5)
    c = sparse.MixedPrecisionSparse.from_dense(x, tr.cutoff_l)
    nod = tr.inverse_transform(c)
    ref = g.to_nodal(x)
    assert float((nod.double() - ref).norm() / ref.norm()) < 1e-3
    back = tr.forward_transform(ref.float() * torch.as_tensor(g.spherical_harmonics.basis.w))
    assert back.to_dense().shape == x.shape


def test_packed_storage_saves_memory_and_roundtrips_exactly():
    g = sh.Grid.T21()
    mask = torch.as_tensor(g.mask)
    x = torch.randn(3, 4, *g.modal_shape) * mask
    lay = sparse.TriangleLayout(*g.modal_shape)
    assert lay.count == int(mask.sum())
    # l-major: the packed entries of total wavenumber l sit in [l_offsets[l], l_offsets[l+1])
    m, l = g.modal_mesh
    ls = torch.as_tensor(l).flatten()[lay.index]
    assert bool((ls[1:] >= ls[:-1]).all())
    st = sparse.SpectralSparseState.from_state_dict({"t": x}, sparse.SparseConfig(mode="structural"))
    torch.testing.assert_close(st.to_dense_dict()["t"], x, rtol=0, atol=0)
    assert abs(st.memory_savings - (1 - lay.count / mask.numel())) < 1e-12 and st.memory_savings > 0.4
    # adaptive: small entries dropped, the rest exact, fewer bytes than the packed triangle
    y = x.clone()
    y[..., 5:, :] *= 1e-9
    ad = sparse.SpectralSparseState.from_state_dict({"t": y}, sparse.SparseConfig(mode="adaptive",
                                                                                  adaptive_threshold=1e-6))
    back = ad.to_dense_dict()["t"]
    keep = y.abs() >= 1e-6
    torch.testing.assert_close(back[keep], y[keep], rtol=0, atol=0)
    assert float(back[~keep].abs().max()) == 0.0
    assert ad.memory_bytes < st.memory_bytes
    # mixed: split at one packed position; low part exact, high part BF16
    mx = sparse.MixedPrecisionSparse.from_dense(x, 11)
    assert mx.low.shape[-1] == lay.split(11) and mx.high.dtype == torch.bfloat16
    d = mx.to_dense()
    torch.testing.assert_close(d[..., :11], x[..., :11], rtol=0, atol=0)
    torch.testing.assert_close(d[..., 11:], x[..., 11:].bfloat16().float(), rtol=0, atol=0)
