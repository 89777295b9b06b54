"""Adaptive density control of the Gaussian table on CPU tensors (the
reference's tests/test_splatting.py:557-650 restated for torch): clone /
split / prune counts and layout, MCMC relocation, compact checkpoints,
opacity reset.  These are host-side table edits with torch operations; no
rendering is involved."""

import math

import numpy as np
import pytest
import torch

from mlx3d_b200.splatting import GaussianModel


def _model(n, seed, sh_degree=1):
    g = torch.Generator().manual_seed(seed)
    return GaussianModel.from_points(torch.randn(n, 3, generator=g), sh_degree=sh_degree)


def test_densify_and_prune_counts_and_layout():
    model = _model(50, 0)
    n0 = model.num_gaussians
    grads = torch.cat([torch.full((10,), 1.0), torch.zeros(n0 - 10)])
    counts = torch.ones(n0)
    with torch.no_grad():
        model.params["opacities"][-5:] -= 100.0
    before = {k: v.clone() for k, v in model.params.items()}
    stats = model.densify_and_prune(grads, counts, grad_threshold=0.5, scene_extent=10.0, percent_dense=0.5,
                                    return_optimizer_state=True, generator=torch.Generator().manual_seed(1))
    assert stats["pruned"] >= 5
    assert stats["cloned"] + stats["split"] == 10
    n1 = n0 - stats["pruned"] + stats["cloned"] + 2 * stats["split"]
    assert model.num_gaussians == n1
    assert stats["_new_count"] == stats["cloned"] + 2 * stats["split"]
    keep = stats["_keep_idx"]
    nk = keep.numel()
    # kept rows first, in order, unchanged
    for k, v in model.params.items():
        torch.testing.assert_close(v[:nk], before[k][keep], rtol=0, atol=0)
    # split rows: log-scales reduced by log 1.6, two per source
    if stats["split"]:
        s = model.params["scales"][nk + stats["cloned"]:]
        assert s.shape[0] == 2 * stats["split"]
    for v in model.params.values():
        assert v.is_contiguous()


def test_split_samples_follow_the_gaussian():
    """One large Gaussian with a high gradient is split into two rows whose
    offsets are R (s * z); with many draws their covariance is R S^2 R^T."""
    means = torch.zeros(1, 3)
    quats = torch.tensor([[0.9238795, 0.0, 0.0, 0.3826834]])  # 45 degrees about z
    scales = torch.log(torch.tensor([[0.3, 0.1, 0.05]]))
    params = {"means": means, "quats": quats, "scales": scales, "opacities": torch.zeros(1),
              "sh_dc": torch.zeros(1, 1, 3), "sh_rest": torch.zeros(1, 0, 3)}
    offs = []
    gen = torch.Generator().manual_seed(7)
    for _ in range(2000):
        m = GaussianModel({k: v.clone() for k, v in params.items()}, sh_degree=0)
        st = m.densify_and_prune(torch.ones(1), torch.ones(1), grad_threshold=0.5, scene_extent=10.0,
                                 percent_dense=0.001, generator=gen)
        assert st == {"cloned": 0, "split": 1, "pruned": 1}
        assert m.num_gaussians == 2
        torch.testing.assert_close(m.params["scales"], (scales - math.log(1.6)).repeat(2, 1))
        offs.append(m.params["means"])
    x = torch.cat(offs).double()
    cov = x.T @ x / x.shape[0]
    c, s_ = math.cos(math.pi / 4), math.sin(math.pi / 4)
    R = torch.tensor([[c, -s_, 0.0], [s_, c, 0.0], [0.0, 0.0, 1.0]], dtype=torch.float64)
    S2 = torch.diag(torch.tensor([0.3, 0.1, 0.05], dtype=torch.float64) ** 2)
    torch.testing.assert_close(cov, R @ S2 @ R.T, atol=3e-3, rtol=0.1)


def test_prune_only_when_no_gradient_is_high():
    model = _model(20, 3)
    with torch.no_grad():
        model.params["opacities"][:4] = -20.0
    st = model.densify_and_prune(torch.zeros(20), torch.ones(20), scene_extent=10.0)
    assert st == {"cloned": 0, "split": 0, "pruned": 4}
    assert model.num_gaussians == 16


def test_select_and_append_keep_leaves_trainable():
    model = _model(6, 4)
    for v in model.params.values():
        v.requires_grad_(True)
    model.select([5, 1, 3])
    assert model.num_gaussians == 3
    model.append({k: torch.zeros(2, *v.shape[1:]) for k, v in model.params.items()})
    assert model.num_gaussians == 5
    for v in model.params.values():
        assert v.is_leaf and v.requires_grad and v.is_contiguous()


def test_mcmc_relocation_keeps_the_count():
    g = torch.Generator().manual_seed(12)
    model = GaussianModel.from_points(torch.randn(30, 3, generator=g) * 0.2, sh_degree=0)
    n0 = model.num_gaussians
    with torch.no_grad():
        model.params["opacities"][:5] -= 100.0
    before = model.params["means"].clone()
    grads = torch.cat([torch.zeros(10), torch.linspace(0.0, 1.0, 20)])
    stats = model.relocate_mcmc(grads, torch.ones(n0), relocate_frac=0.2, min_opacity=0.05, jitter_scale=0.0)
    assert model.num_gaussians == n0
    assert stats["relocated"] == 5
    moved = stats["_moved_idx"].sort().values
    assert moved.tolist() == [0, 1, 2, 3, 4]
    after = model.params["means"]
    assert not torch.allclose(after[:5], before[:5])
    # sources: the five highest-gradient rows, copied with reset opacity and shrunk scales
    # (jitter 0: each relocated row is an exact copy of one of rows 25..29)
    assert torch.isin(after[:5, 0], before[25:, 0]).all()
    torch.testing.assert_close(model.params["opacities"][:5], torch.full((5,), math.log(0.05 / 0.95)))


def test_compact_prunes_by_opacity_and_cap_without_mutating():
    pts = torch.stack([torch.tensor([float(i), 0.0, 0.0]) for i in range(6)])
    model = GaussianModel.from_points(pts, sh_degree=2)
    model.active_sh_degree = 2
    model.params["opacities"] = torch.tensor([-8.0, 2.0, -4.0, 4.0, 1.0, -7.0])
    model.params["scales"] = torch.log(torch.tensor([[0.1] * 3, [0.2] * 3, [5.0] * 3, [1.0] * 3, [0.4] * 3,
                                                     [10.0] * 3]))
    compact = model.compact(min_opacity=0.01, max_gaussians=2)
    assert model.num_gaussians == 6 and compact.num_gaussians == 2
    np.testing.assert_allclose(compact.params["means"][:, 0].numpy(), [2.0, 3.0], atol=1e-6)
    assert compact.sh_degree == 2 and compact.active_sh_degree == 2


def test_compact_truncates_sh_degree_and_keeps_one_row():
    g = torch.Generator().manual_seed(2)
    model = GaussianModel.from_points(torch.randn(4, 3, generator=g) * 0.1, sh_degree=3)
    model.active_sh_degree = 3
    model.params["opacities"] = torch.full((4,), -20.0)
    compact = model.compact(min_opacity=0.99, target_sh_degree=1)
    assert compact.num_gaussians == 1 and compact.sh_degree == 1 and compact.active_sh_degree == 1
    assert compact.sh.shape == (1, 4, 3)


def test_compact_validates_inputs():
    model = _model(3, 5)
    with pytest.raises(ValueError, match="max_gaussians"):
        model.compact(max_gaussians=0)
    with pytest.raises(ValueError, match="target_sh_degree"):
        model.compact(target_sh_degree=2)


def test_reset_opacities_clamps_logits():
    model = _model(5, 6)
    with torch.no_grad():
        model.params["opacities"][:] = torch.tensor([-9.0, -2.0, 0.0, 3.0, 8.0])
    model.reset_opacities(0.01)
    cap = math.log(0.01 / 0.99)
    np.testing.assert_allclose(model.params["opacities"].numpy(), [-9.0, cap, cap, cap, cap], rtol=1e-6)
