"""Adaptive density control against the reference's own model.py (CPU).

``tests/golden/reference_outputs.npz`` holds what mlx3D's
GaussianModel.densify_and_prune (model.py:406-480) and relocate_mcmc
(model.py:482-531) produced on seeded parameters, executed on the numpy
stand-in for mlx.core, with numpy's generator seeded and the split draws
stored.  The oracle restatement (oracle/density.py) and the product
(mlx3d_b200/splatting/model.py, torch on CPU tensors, given the same draws)
must select the same rows exactly; new parameter values agree to float32
rounding (the reference forms split offsets in float64 and writes relocated
rows as a + (v - a)).  The relocation's destination/source pairing follows
the order of MLX's argpartition, which is unspecified, so relocated rows are
compared as a multiset.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import density as orc_density
from mlx3d_b200.splatting import GaussianModel

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_outputs.npz"
NAMES = ("means", "scales", "quats", "opacities", "sh_dc", "sh_rest")


@pytest.fixture(scope="module")
def g():
    with np.load(GOLDEN) as z:
        return {k: z[k] for k in z.files}


def _params(g, p):
    return {k: g[f"{p}in_{k}"] for k in NAMES}


def _close(a, b, what, tol=1e-6):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    assert a.shape == b.shape, (what, a.shape, b.shape)
    err = np.abs(a - b).max() if a.size else 0.0
    assert err <= tol * max(1.0, np.abs(b).max() if b.size else 1.0), (what, err)


DENSIFY = dict(grad_threshold=0.0002, scene_extent=3.0, percent_dense=0.02, min_opacity=0.005)


def test_oracle_densify_matches_reference(g):
    new, info = orc_density.densify_and_prune(_params(g, "density/"), g["density/grad_accum"],
                                              g["density/grad_count"], samples=g["density/split_samples"],
                                              **DENSIFY)
    assert [info["cloned"], info["split"], info["pruned"]] == g["density/counts"].tolist()
    np.testing.assert_array_equal(info["keep_idx"], g["density/keep_idx"])
    for k in NAMES:
        _close(new[k], g[f"density/out_{k}"], k)
    # every case occurs: clones, splits, prunes of each kind
    assert info["cloned"] > 0 and info["split"] > 0 and info["pruned"] > info["split"]


def test_product_densify_matches_reference(g):
    model = GaussianModel({k: torch.tensor(v) for k, v in _params(g, "density/").items()}, sh_degree=1)
    stats = model.densify_and_prune(torch.tensor(g["density/grad_accum"]), torch.tensor(g["density/grad_count"]),
                                    return_optimizer_state=True,
                                    samples=torch.tensor(g["density/split_samples"], dtype=torch.float32),
                                    **DENSIFY)
    assert [stats["cloned"], stats["split"], stats["pruned"]] == g["density/counts"].tolist()
    np.testing.assert_array_equal(stats["_keep_idx"].numpy(), g["density/keep_idx"])
    for k in NAMES:
        _close(model.params[k].detach().numpy(), g[f"density/out_{k}"], k)


def _rows_as_multiset(params, idx):
    rows = np.concatenate([np.asarray(params[k])[idx].reshape(len(idx), -1) for k in NAMES], axis=1)
    return rows[np.lexsort(rows.T[::-1])]


def test_oracle_and_product_relocation_match_reference(g):
    p = _params(g, "mcmc/")
    k, dst, src = orc_density.relocate_mcmc_selection(p, g["mcmc/grad_accum"], g["mcmc/grad_count"],
                                                      relocate_frac=0.05, min_opacity=0.01)
    assert k == int(g["mcmc/relocated"][0]) and k > 0
    np.testing.assert_array_equal(dst, g["mcmc/moved_idx"])
    ref_out = {kk: g[f"mcmc/out_{kk}"] for kk in NAMES}
    written = orc_density.relocated_rows(p, src)
    want = _rows_as_multiset(written, np.arange(k))
    _close(want, _rows_as_multiset(ref_out, dst), "relocated rows (oracle)")
    untouched = np.setdiff1d(np.arange(p["means"].shape[0]), dst)
    for kk in NAMES:
        np.testing.assert_array_equal(ref_out[kk][untouched], p[kk][untouched])
    # the product, given the same inputs
    model = GaussianModel({kk: torch.tensor(v) for kk, v in p.items()}, sh_degree=1)
    st = model.relocate_mcmc(torch.tensor(g["mcmc/grad_accum"]), torch.tensor(g["mcmc/grad_count"]),
                             relocate_frac=0.05, min_opacity=0.01, jitter_scale=0.0)
    assert st["relocated"] == k
    np.testing.assert_array_equal(np.sort(st["_moved_idx"].numpy()), dst)
    out = {kk: v.detach().numpy() for kk, v in model.params.items()}
    _close(_rows_as_multiset(out, dst), _rows_as_multiset(ref_out, dst), "relocated rows (product)")
    for kk in NAMES:
        np.testing.assert_array_equal(out[kk][untouched], p[kk][untouched])
