"""3DGS PLY checkpoints (src/mlx3d/splatting/model.py:338-392, io/ply_io.py:56-271).

The standard Gaussian-splatting vertex layout, all float32, in this order:
``x y z nx ny nz f_dc_0..2 f_rest_0..(3(K-1)-1) opacity scale_0..2 rot_0..3``
with ``f_rest`` channel-major (all coefficients of red, then green, then
blue), raw (pre-activation) parameters.  Written as binary_little_endian;
read from binary_little_endian or ascii files with float / double / integer
vertex properties.  Host-side file IO (numpy), not a device path.
"""

from __future__ import annotations

import os

import numpy as np
import torch

__all__ = ["save_gaussians_ply", "load_gaussians_ply"]

_PLY_TYPES = {
    "char": "i1", "int8": "i1", "uchar": "u1", "uint8": "u1", "short": "i2", "int16": "i2", "ushort": "u2",
    "uint16": "u2", "int": "i4", "int32": "i4", "uint": "u4", "uint32": "u4", "float": "f4", "float32": "f4",
    "double": "f8", "float64": "f8",
}


def _host(t) -> np.ndarray:
    return (t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else np.asarray(t)).astype(np.float32)


def save_gaussians_ply(path: str, params: dict) -> None:
    """Write raw GaussianModel parameters in the 3DGS layout (model.py:338-361)."""
    means = _host(params["means"])
    n = means.shape[0]
    dc = _host(params["sh_dc"]).reshape(n, 3)
    rest = _host(params["sh_rest"]).reshape(n, -1, 3)
    rest_t = rest.transpose(0, 2, 1).reshape(n, -1)  # channel-major
    cols = [("x", means[:, 0]), ("y", means[:, 1]), ("z", means[:, 2])]
    cols += [(f"n{a}", np.zeros(n, np.float32)) for a in "xyz"]
    cols += [(f"f_dc_{c}", dc[:, c]) for c in range(3)]
    cols += [(f"f_rest_{i}", rest_t[:, i]) for i in range(rest_t.shape[1])]
    cols += [("opacity", _host(params["opacities"]).reshape(n))]
    scales, quats = _host(params["scales"]), _host(params["quats"])
    cols += [(f"scale_{i}", scales[:, i]) for i in range(3)]
    cols += [(f"rot_{i}", quats[:, i]) for i in range(4)]
    rec = np.empty(n, dtype=[(k, "<f4") for k, _ in cols])
    for k, v in cols:
        rec[k] = v
    header = ["ply", "format binary_little_endian 1.0", f"element vertex {n}"]
    header += [f"property float {k}" for k, _ in cols]
    header += ["end_header"]
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    with open(path, "wb") as f:
        f.write(("\n".join(header) + "\n").encode("ascii"))
        f.write(rec.tobytes())


def _read_vertices(path: str) -> np.ndarray:
    with open(path, "rb") as f:
        data = f.read()
    end = data.find(b"end_header\n")
    if end < 0:
        raise ValueError(f"{path!r} is not a valid PLY file (no end_header).")
    lines = data[:end].decode("ascii", errors="replace").splitlines()
    if not lines or lines[0].strip() != "ply":
        raise ValueError(f"{path!r} is not a PLY file.")
    body = data[end + len(b"end_header\n"):]
    fmt, elements = None, []
    for line in lines[1:]:
        parts = line.split()
        if not parts or parts[0] == "comment":
            continue
        if parts[0] == "format":
            fmt = parts[1]
        elif parts[0] == "element":
            elements.append([parts[1], int(parts[2]), []])
        elif parts[0] == "property":
            if parts[1] == "list":
                raise ValueError("list properties are not supported in Gaussian PLY files")
            elements[-1][2].append((parts[2], _PLY_TYPES[parts[1]]))
    if not elements or elements[0][0] != "vertex":
        raise ValueError("the first PLY element must be 'vertex'.")
    name, count, props = elements[0]
    if fmt == "binary_little_endian":
        dt = np.dtype([(k, "<" + t) for k, t in props])
        return np.frombuffer(body, dtype=dt, count=count)
    if fmt == "ascii":
        text = body.decode("ascii").split("\n")[:count]
        arr = np.loadtxt(text, dtype=np.float64, ndmin=2)
        dt = np.dtype([(k, t) for k, t in props])
        rec = np.empty(count, dtype=dt)
        for j, (k, _) in enumerate(props):
            rec[k] = arr[:, j]
        return rec
    raise ValueError(f"unsupported PLY format {fmt!r}")


def load_gaussians_ply(path: str, sh_degree: int = 3, device="cuda") -> tuple[dict, int]:
    """Read a 3DGS PLY (model.py:363-392): returns (raw parameters, SH degree),
    the degree inferred from the file when its f_rest count disagrees."""
    v = _read_vertices(path)
    names = v.dtype.names
    n = v.shape[0]
    n_rest = len([k for k in names if k.startswith("f_rest_")])
    K = (sh_degree + 1) ** 2
    if n_rest != 3 * (K - 1):
        K = n_rest // 3 + 1
        sh_degree = int(round(np.sqrt(K))) - 1
    f = lambda k: np.asarray(v[k], dtype=np.float32)  # noqa: E731
    rest = np.stack([f(f"f_rest_{i}") for i in range(n_rest)], 1) if n_rest else np.zeros((n, 0), np.float32)
    rest = rest.reshape(n, 3, K - 1).transpose(0, 2, 1)
    params = {
        "means": np.stack([f("x"), f("y"), f("z")], 1),
        "scales": np.stack([f(f"scale_{i}") for i in range(3)], 1),
        "quats": np.stack([f(f"rot_{i}") for i in range(4)], 1),
        "opacities": f("opacity"),
        "sh_dc": np.stack([f(f"f_dc_{c}") for c in range(3)], 1)[:, None, :],
        "sh_rest": rest,
    }
    return {k: torch.from_numpy(np.ascontiguousarray(a)).to(device) for k, a in params.items()}, sh_degree
