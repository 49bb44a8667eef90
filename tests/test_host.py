"""Host logic that needs no GPU: table lookup and caching."""

import numpy as np
import torch


def test_missing_table_is_fitted_and_cached(tmp_path, monkeypatch):
    from lookatmyquant_b200 import codes
    monkeypatch.setattr(codes, "fit_trellis_values", lambda *a, **kw: torch.arange(4096.0))
    monkeypatch.setenv("LAMQ_TABLE_CACHE", str(tmp_path))
    v = codes.trellis_values(12, 2, 48)
    assert (tmp_path / "trellis_L12_k2_T48_s0_ema.f64").exists()
    assert np.array_equal(codes.trellis_values(12, 2, 48).numpy(), v.numpy())
