"""Rotation loader and composition (reference intent: ``tests/test_numeric.py``
rotation loader, key tolerance, quality floor; ``tests/test_backend.py`` strict
missing rotation)."""
import warnings

import pytest
import torch

from oscar_b200.kv import calib as C
from oscar_b200.kv import format as fmt
from oscar_b200.kv import rotation as R


def _ortho(D, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.linalg.qr(torch.randn(D, D, generator=g, dtype=torch.float64))[0].float()


def test_quality_floor_u_h_pbr_beats_plain_eigenvectors():
    """Synthetic outlier channels: per-vector INT2 after the plain eigenvector basis
    stays at noise level, after U.H.P_br it does not."""
    D, N = 256, 512
    g = torch.Generator().manual_seed(7)
    chan = torch.ones(D)
    chan[:4], chan[4:12], chan[12:24] = 24.0, 8.0, 2.5
    amp = torch.exp(0.4 * torch.randn(N, 1, 1, generator=g))
    K = torch.randn(N, 1, D, generator=g) * chan * amp
    x = K.reshape(-1, D).double()
    cov = x.t() @ x / x.shape[0]
    evals, evecs = torch.linalg.eigh(cov + 1e-6 * torch.eye(D, dtype=torch.float64))
    order = torch.argsort(evals, descending=True)
    U = evecs[:, order].float()
    Rn = C.compose_rotation(evecs, evals).float()
    assert (Rn @ Rn.t() - torch.eye(D)).abs().max() < 1e-4

    def rel(xr):
        p, s, z = fmt.quantize(xr)
        return float((fmt.dequant(p, s, z, D) - xr).norm() / xr.norm())

    r_plain, r_new = rel(K @ U), rel(K @ Rn)
    assert r_plain >= 1.0, r_plain
    assert r_new <= 0.60, r_new


def test_loader_formats_and_key_tolerance(tmp_path):
    D = 64
    a, b = _ortho(D, 1), _ortho(D, 2)
    p2 = tmp_path / "v2.pt"
    R.save_rotations(p2, {3: {"rotation": a, "rotation_v": b}})
    assert torch.allclose(R.get_layer_rotation(str(p2), 3, D, "cpu", mode="k"), a)
    assert torch.allclose(R.get_layer_rotation(str(p2), "model.layers.3.self_attn.attn", D, "cpu", mode="v"), b)
    # {lid: matrix} with string keys, and a stacked [L, D, D] tensor (both legacy, not v2)
    pd = tmp_path / "dict.pt"
    torch.save({"3": a, "model.layers.7.self_attn": b}, pd)
    ps = tmp_path / "stack.pt"
    torch.save(torch.stack([a, b]), ps)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        assert torch.allclose(R.get_layer_rotation(str(pd), 7, D, "cpu"), b)
        assert torch.allclose(R.get_layer_rotation(str(ps), 1, D, "cpu"), b)
    assert R.layer_index_from_name("model.layers.11.self_attn.attn") == 11
    assert R.layer_index_from_name("lm_head") is None


def test_loader_strict_and_missing(tmp_path):
    D = 64
    p = tmp_path / "r.pt"
    R.save_rotations(p, {3: {"rotation": _ortho(D, 1), "rotation_v": _ortho(D, 2)}})
    # missing layer: identity when not strict, error when strict
    assert torch.equal(R.get_layer_rotation(str(p), 5, D, "cpu", strict=False), torch.eye(D))
    with pytest.raises(Exception):
        R.get_layer_rotation(str(p), 5, D, "cpu", strict=True)
    bad = tmp_path / "bad.pt"
    R.save_rotations(bad, {3: {"rotation": torch.randn(D, D), "rotation_v": _ortho(D, 2)}})
    with pytest.raises(Exception):
        R.get_layer_rotation(str(bad), 3, D, "cpu", strict=True)
    nan = tmp_path / "nan.pt"
    m = _ortho(D, 1)
    m[0, 0] = float("nan")
    R.save_rotations(nan, {3: {"rotation": m, "rotation_v": _ortho(D, 2)}})
    with pytest.raises(Exception):
        R.get_layer_rotation(str(nan), 3, D, "cpu", strict=True)


def test_calibration_merge_is_count_weighted():
    D = 8
    a = {"L": {"q": {"cov": torch.eye(D) * 2, "count": 1}, "v": {"cov": torch.eye(D), "count": 1}}}
    b = {"L": {"q": {"cov": torch.eye(D) * 5, "count": 3}, "v": {"cov": torch.eye(D), "count": 3}}}
    m = C.merge_rank_stats([a, b], D)
    assert m["L"]["q"]["count"] == 4
    assert torch.allclose(m["L"]["q"]["cov_sum"] / 4, torch.eye(D) * (2 + 15) / 4)
