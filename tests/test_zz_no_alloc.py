"""The allocation-free synthesis entry point ``tgcm_sht_synth_noalloc``.

That C function serves callers that cannot allocate device memory while they
run (a fixed memory arena, no PyTorch allocator, plain C code): it keeps its
intermediate buffer in a static array inside the extension.  Here it is called
through its exported C symbol with ctypes and compared with the regular
synthesis op, which takes its buffer from PyTorch.  Consecutive calls share
the static buffer, so several calls in a row with different shapes check that
no call depends on what the previous one left behind.

This file is named so that pytest collects it last.
"""

import ctypes

import numpy as np
import pytest
import torch

from tornado_gcm_b200.ops import _ext

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs CUDA")]

OK, ERR_ARGS, ERR_TOO_LARGE = 0, 1, 2
SCRATCH_FLOATS = 4 * 1024 * 1024


def _entry():
    _ext.require("allocation-free synthesis test")
    from tornado_gcm_b200 import _C

    fn = ctypes.CDLL(_C.__file__).tgcm_sht_synth_noalloc
    ll = ctypes.c_longlong
    fn.argtypes = [ctypes.c_void_p, ll, ll, ll, ll, ll, ctypes.c_void_p, ll, ll, ll, ctypes.c_void_p, ll, ll,
                   ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def _bases(name):
    from tornado_gcm_b200.core import spherical_harmonic as sh
    from tornado_gcm_b200.ops import sht as sht_ops

    g = getattr(sh.Grid, name)(precision="tf32")
    return g, sht_ops.bases(g.spherical_harmonics, torch.device("cuda"))


def _modal_padded(g, b, S, seed):
    """(S, M2, Lp) buffer holding a band-limited field in its first L columns."""
    rng = np.random.default_rng(seed)
    m, l = g.modal_mesh
    amp = np.where(g.mask, (1.0 + l) ** -1.5, 0.0)
    buf = torch.zeros(S, b.M2, b.Lp, dtype=torch.float32)
    buf[..., : b.L] = torch.tensor(rng.standard_normal((S,) + g.modal_shape) * amp, dtype=torch.float32)
    return buf.cuda()


def _call(fn, b, xbuf, S, out, lat_major, err):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(xbuf.data_ptr(), S, b.M2, b.L, b.Lp, b.M2 * b.Lp, b.P.data_ptr(), (b.M2 + 1) // 2, b.J, b.Lp,
              b.F.data_ptr(), b.I, b.M2p, out.data_ptr(), int(lat_major), err.data_ptr(), stream)


def _regular(b, xbuf, lat_major):
    ops = _ext.require("synthesis")
    S = xbuf.shape[0]
    ws = torch.empty(S * b.J * b.M2p, dtype=torch.float32, device=xbuf.device)
    return ops.sht_synth(xbuf[..., : b.L], b.L, b.P, b.F, ws, None, None, lat_major)


@pytest.mark.parametrize("calls", [[("TL63", 7, False), ("TL63", 3, True), ("T21", 11, False),
                                    ("TL127", 5, True), ("TL63", 7, False)]])
def test_noalloc_synthesis_matches_regular_op(calls):
    fn = _entry()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for i, (name, S, lat_major) in enumerate(calls):
        g, b = _bases(name)
        xbuf = _modal_padded(g, b, S, seed=10 + i)
        shape = (S, b.J, b.I) if lat_major else (S, b.I, b.J)
        out = torch.full(shape, float("nan"), device="cuda")
        assert _call(fn, b, xbuf, S, out, lat_major, err) == OK
        ref = _regular(b, xbuf, lat_major)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-6)


def test_noalloc_synthesis_rejects_oversized_request():
    fn = _entry()
    g, b = _bases("TL63")
    S = SCRATCH_FLOATS // (b.J * b.M2p) + 1  # one slice more than the static buffer holds
    xbuf = _modal_padded(g, b, 1, seed=0)
    out = torch.empty(1, b.I, b.J, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    # the size check runs before any pointer is dereferenced or kernel launched
    assert _call(fn, b, xbuf, S, out, False, err) == ERR_TOO_LARGE
    bad = xbuf.flatten()[1:]  # 4-byte offset: not 16-byte aligned
    assert _call(fn, b, bad, 1, out, False, err) == ERR_ARGS


def test_noalloc_synthesis_rejects_groups_without_k_blocks():
    """A wavenumber group whose triangular K range is empty would leave its W rows unwritten."""
    fn = _entry()
    g, b = _bases("TL63")
    xbuf = _modal_padded(g, b, 1, seed=0)
    out = torch.empty(1, b.I, b.J, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    L, Mw = 32, 33  # group m = 32 would start its K loop at l = 32 = L
    rc = fn(xbuf.data_ptr(), 1, 2 * Mw - 1, L, b.Lp, b.M2 * b.Lp, b.P.data_ptr(), Mw, b.J, b.Lp,
            b.F.data_ptr(), b.I, b.M2p, out.data_ptr(), 0, err.data_ptr(), stream)
    assert rc == ERR_ARGS
