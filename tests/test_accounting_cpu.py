"""Op accounting behind the step-level roofline: FLOP formulas and the counting proxy."""

import torch

from tornado_gcm_b200.ops import accounting


def test_gemm_flop_formulas():
    X, W = torch.empty(300, 208), torch.empty(72, 208)
    assert accounting._flops("linear_fwd", (X, W)) == (2 * 300 * 208 * 72, "bf16")
    dY = torch.empty(300, 72)
    assert accounting._flops("linear_dgrad", (dY, W)) == (2 * 300 * 72 * 208, "bf16")
    A, B = torch.empty(5, 128, 64), torch.empty(5, 80, 64)
    assert accounting._flops("bgemm_tf32", (A, B)) == (2 * 5 * 128 * 64 * 80, "tf32")
    # Legendre synthesis: sum over m < Mw of (L - m) coefficients per cos/sin row, J latitudes
    x, P, F = torch.empty(7, 5, 6), torch.empty(3, 4, 8), torch.empty(8, 8)
    fl, cls = accounting._flops("sht_synth", (x, 6, P, F))
    assert cls == "tf32" and fl == 2 * 7 * 4 * 2 * (6 + 5 + 4) + 2 * 7 * 4 * 8 * 5
    assert accounting._flops("spectral_linear", (x,)) == (0, None)


def test_counting_proxy_records_calls_and_restores():
    class FakeOps:
        @staticmethod
        def linear_fwd(X, W):
            return None

    assert accounting.active() is None
    with accounting.counting() as acc:
        ops = accounting.CountingOps(FakeOps())
        ops.linear_fwd(torch.empty(4, 8), torch.empty(16, 8))
        ops.linear_fwd(torch.empty(4, 8), torch.empty(16, 8))
    assert accounting.active() is None
    assert acc["linear_fwd"]["calls"] == 2 and acc["linear_fwd"]["flops"] == 2 * 2 * 4 * 8 * 16
    assert acc["linear_fwd"]["bytes"] == 0  # host tensors are not device traffic
    sm = accounting.summary({"k": {"calls": 1, "bytes": 6.5546e9, "flops": 0, "cls": None}}, 6554.6, 1690.5)
    assert abs(sm["t_hbm_ms"] - 1.0) < 1e-6 and sm["roofline_ms"] == sm["t_hbm_ms"]
