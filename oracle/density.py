"""CPU restatement of the reference's adaptive density control (test
infrastructure only; the product path is mlx3d_b200/splatting/model.py).

Follows src/mlx3d/splatting/model.py of mlx3D 0.2.0:

* ``densify_and_prune``  model.py:406-480 -- clone / split / prune selection
  and the new rows (splits: two draws R (s * z) around the mean, log-scales
  minus log 1.6), kept rows first, then clones, then split pairs;
* ``relocate_mcmc``      model.py:482-531 -- fixed-budget relocation of
  underused rows onto copies of high-gradient rows.

Random draws are inputs here (``samples`` / ``noise``), so a caller can feed
the same draws to the reference and to the product.  The MCMC selection is
returned as sets: the reference takes its k rows with ``mx.argpartition``,
whose order inside the selection is unspecified, and pairs destination i
with source i in that order; only the selected sets and the multiset of
written rows are fixed by the algorithm.
"""

from __future__ import annotations

import numpy as np

LOG_1_6 = float(np.log(1.6))


def _rotmat(q: np.ndarray) -> np.ndarray:
    """Rotation matrices of wxyz quaternions (transforms/rotations.py:30-49)."""
    q = q / np.linalg.norm(q, axis=1, keepdims=True)
    w, x, y, z = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    two = 2.0
    m = np.stack([1 - two * (y * y + z * z), two * (x * y - w * z), two * (x * z + w * y),
                  two * (x * y + w * z), 1 - two * (x * x + z * z), two * (y * z - w * x),
                  two * (x * z - w * y), two * (y * z + w * x), 1 - two * (x * x + y * y)], axis=-1)
    return m.reshape(-1, 3, 3)


def densify_and_prune(params: dict, grad_accum, grad_count, grad_threshold=0.0002, scene_extent=1.0,
                      percent_dense=0.01, min_opacity=0.005, samples=None) -> tuple[dict, dict]:
    """(new params, {"clone_idx", "split_idx", "keep_idx", "cloned", "split", "pruned"})."""
    p = {k: np.asarray(v) for k, v in params.items()}
    avg_grad = np.asarray(grad_accum) / np.maximum(np.asarray(grad_count), 1.0)
    scales = np.exp(p["scales"])
    max_scale = scales.max(axis=1)
    high = avg_grad > grad_threshold
    clone_mask = high & (max_scale <= percent_dense * scene_extent)
    split_mask = high & (max_scale > percent_dense * scene_extent)
    clone_idx = np.where(clone_mask)[0]
    split_idx = np.where(split_mask)[0]
    clones = {k: v[clone_idx] for k, v in p.items()}
    splits = {}
    if split_idx.size:
        R = _rotmat(p["quats"][split_idx])
        s = scales[split_idx]
        z = np.asarray(samples, dtype=np.float64).reshape(split_idx.size * 2, 3)
        offsets = np.einsum("nij,nj->ni", np.repeat(R, 2, axis=0), z * np.repeat(s, 2, axis=0))
        splits = {k: np.repeat(v[split_idx], 2, axis=0) for k, v in p.items()}
        splits["means"] = splits["means"] + offsets.astype(np.float32)
        splits["scales"] = splits["scales"] - np.float32(LOG_1_6)
    opac = 1.0 / (1.0 + np.exp(-np.clip(p["opacities"], -50.0, 50.0)))
    prune = (opac < min_opacity) | split_mask | (max_scale > 0.5 * scene_extent)
    keep_idx = np.where(~prune)[0]
    new = {k: np.concatenate([v[keep_idx], clones[k]] + ([splits[k]] if splits else []), axis=0)
           for k, v in p.items()}
    info = {"clone_idx": clone_idx, "split_idx": split_idx, "keep_idx": keep_idx, "cloned": int(clone_idx.size),
            "split": int(split_idx.size), "pruned": int(prune.sum())}
    return new, info


def relocate_mcmc_selection(params: dict, grad_accum, grad_count, relocate_frac=0.02, min_opacity=0.01):
    """(k, destination set, source set) of model.py:493-515, as sorted arrays."""
    p = {k: np.asarray(v) for k, v in params.items()}
    n = p["means"].shape[0]
    max_relocate = int(max(0.0, min(relocate_frac, 1.0)) * n)
    if max_relocate <= 0 or n <= 1:
        return 0, np.zeros(0, np.int64), np.zeros(0, np.int64)
    counts = np.asarray(grad_count, np.float32)
    avg_grad = np.asarray(grad_accum, np.float32) / np.maximum(counts, np.float32(1.0))
    opac = 1.0 / (1.0 + np.exp(-p["opacities"].astype(np.float32)))
    underused = (opac < min_opacity) | (counts <= 0)
    n_under = int(underused.sum())
    k = max_relocate if n_under == 0 else min(max_relocate, n_under)
    k = min(k, n - 1)
    if k == 0:
        return 0, np.zeros(0, np.int64), np.zeros(0, np.int64)
    target = np.where(underused, 2.0 - opac, -opac)
    dst = np.argsort(-target, kind="stable")[:k]
    source = avg_grad.copy()
    source[dst] = -1e30
    src = np.argsort(-source, kind="stable")[:k]
    return k, np.sort(dst), np.sort(src)


def relocated_rows(params: dict, src: np.ndarray) -> dict:
    """The rows relocate_mcmc writes for sources ``src`` without jitter
    (model.py:516-530): copies with opacity logit(0.05) and log-scales minus
    log 1.6."""
    p = {k: np.asarray(v) for k, v in params.items()}
    out = {k: v[src].copy() for k, v in p.items()}
    out["opacities"] = np.full_like(out["opacities"], np.float32(np.log(0.05 / 0.95)))
    out["scales"] = out["scales"] - np.float32(LOG_1_6)
    return out
