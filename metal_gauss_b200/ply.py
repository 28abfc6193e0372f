"""INRIA-convention .ply export and import for trained Gaussians.

The reference writes its model with `train.export_ply` (metal_gauss/train.py:
583-624) and reads it with `io.load_ply` (metal_gauss/io.py:87-121), both
through the `plyfile` package (>= 1.0). The on-disk layout is the 3DGS
convention and must not change (io.py:1-11): one binary little-endian
`vertex` element of float32 properties, in this order:

    x y z, f_dc_0..2, f_rest_0..(3*(B-1)-1), opacity, scale_0..2, rot_0..3

with the parameters in their stored (pre-activation) form: opacity a logit,
scales logarithms, the quaternion (w, x, y, z) as trained (not normalised),
and the higher SH bands channel-major, f_rest_[c*(B-1) + (b-1)] holding band
b of channel c. The header is the PLY 1.0 header plyfile writes for such an
element: `ply`, `format binary_little_endian 1.0`, `element vertex N`, one
`property float <name>` line per field, `end_header`, each line ended by a
line feed, followed directly by the packed records.

This module writes and reads that layout with numpy alone (plyfile is not a
dependency here).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch


def field_names(rest_per_channel: int = 15) -> list[str]:
    """Property names in file order for (rest_per_channel + 1) SH bands."""
    return (["x", "y", "z"] + [f"f_dc_{i}" for i in range(3)]
            + [f"f_rest_{i}" for i in range(3 * rest_per_channel)] + ["opacity"]
            + [f"scale_{i}" for i in range(3)] + [f"rot_{i}" for i in range(4)])


def header(n: int, rest_per_channel: int = 15) -> bytes:
    lines = ["ply", "format binary_little_endian 1.0", f"element vertex {n}"]
    lines += [f"property float {name}" for name in field_names(rest_per_channel)]
    lines.append("end_header")
    return ("\n".join(lines) + "\n").encode("ascii")


def _np(t) -> np.ndarray:
    if isinstance(t, torch.Tensor):
        t = t.detach().to("cpu", torch.float32)
        return t.numpy()
    return np.asarray(t, dtype=np.float32)


def records(p: dict) -> np.ndarray:
    """The structured float32 records of parameter dict `p` (the trainer's
    storage form: means (N,3), quats (N,4), log_scales (N,3), logit_opac
    (N,), and either sh_dc (N,1,3) + sh_rest (N,B-1,3) or sh (N,B,3))."""
    means = _np(p["means"])
    n = means.shape[0]
    if "sh_dc" in p:
        sh = np.concatenate([_np(p["sh_dc"]).reshape(n, 1, 3),
                             _np(p["sh_rest"]).reshape(n, -1, 3)], axis=1)
    else:
        sh = _np(p["sh"]).reshape(n, -1, 3)
    per_channel = sh.shape[1] - 1
    rec = np.zeros(n, dtype=np.dtype([(name, "<f4") for name in field_names(per_channel)]))
    rec["x"], rec["y"], rec["z"] = means[:, 0], means[:, 1], means[:, 2]
    for c in range(3):
        rec[f"f_dc_{c}"] = sh[:, 0, c]
        for b in range(per_channel):
            rec[f"f_rest_{c * per_channel + b}"] = sh[:, b + 1, c]
    rec["opacity"] = _np(p["logit_opac"]).reshape(n)
    ls = _np(p["log_scales"]).reshape(n, 3)
    for i in range(3):
        rec[f"scale_{i}"] = ls[:, i]
    q = _np(p["quats"]).reshape(n, 4)
    for i in range(4):
        rec[f"rot_{i}"] = q[:, i]
    return rec


def bake_3d_filter(p: dict, filter_3d) -> dict:
    """`p` with Mip-Splatting's 3D filter baked into its stored scales and
    opacity (train.py:609-616): the filter is applied to exp(log_scales) and
    sigmoid(logit_opac) (mipfilter.py:79-93) and the results are written back
    in log / logit space, opacity clamped to [1e-6, 1 - 1e-6] so a fully
    suppressed Gaussian stays finite. float32 arithmetic on the host."""
    f = torch.as_tensor(filter_3d).detach().to("cpu", torch.float32)
    ls = torch.as_tensor(p["log_scales"]).detach().to("cpu", torch.float32)
    lo = torch.as_tensor(p["logit_opac"]).detach().to("cpu", torch.float32)
    n = ls.shape[0]
    f = f[:n]
    s2 = torch.exp(ls) ** 2
    s2f = s2 + (f ** 2).unsqueeze(-1)
    sc = torch.sqrt(s2f)
    op = torch.sigmoid(lo) * torch.sqrt((s2.prod(dim=-1) / s2f.prod(dim=-1)).clamp(0.0, 1.0))
    op = op.clamp(1e-6, 1.0 - 1e-6)
    out = dict(p)
    out["log_scales"] = torch.log(sc.clamp_min(1e-12))
    out["logit_opac"] = torch.log(op / (1.0 - op))
    return out


def export_ply(p: dict, path: str | Path, filter_3d=None) -> None:
    """Write `p` as an INRIA-convention .ply, the layout of the reference's
    `export_ply(p, path, filter_3d)` (train.py:583-624); with `filter_3d` the
    filter is baked into the stored scales and opacity, so any viewer renders
    the model as the trainer does."""
    if filter_3d is not None:
        p = bake_3d_filter(p, filter_3d)
    rec = records(p)
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    with open(path, "wb") as f:
        f.write(header(rec.shape[0], (len(rec.dtype.names) - 14) // 3))
        f.write(rec.tobytes())


def read_ply(path: str | Path) -> dict:
    """Parameters in the trainer's storage form (means, quats, log_scales,
    logit_opac, sh_dc (N,1,3), sh_rest (N,B-1,3); float32 tensors on the CPU)
    from a binary little-endian INRIA .ply whose vertex properties are all
    float32. Unlike the reference's load_ply (io.py:87-121) nothing is
    activated or normalised: the values are exactly those stored."""
    with open(path, "rb") as f:
        raw = f.read()
    end = raw.find(b"end_header\n")
    if not raw.startswith(b"ply\n") or end < 0:
        raise ValueError(f"{path}: not a PLY file")
    lines = raw[:end].decode("ascii").split("\n")
    if "format binary_little_endian 1.0" not in lines:
        raise ValueError(f"{path}: only binary little-endian PLY files are read")
    n, names, in_vertex = None, [], False
    for line in lines:
        parts = line.split()
        if not parts:
            continue
        if parts[0] == "element":
            in_vertex = parts[1] == "vertex"
            if in_vertex:
                n = int(parts[2])
            elif n is not None:
                raise ValueError(f"{path}: elements after 'vertex' are not read")
        elif parts[0] == "property" and in_vertex:
            if parts[1] != "float":
                raise ValueError(f"{path}: property {parts[-1]} is {parts[1]}, not float")
            names.append(parts[2])
    if n is None:
        raise ValueError(f"{path}: no vertex element")
    rec = np.frombuffer(raw, dtype=np.dtype([(nm, "<f4") for nm in names]), count=n,
                        offset=end + len(b"end_header\n"))
    n_rest = sum(1 for nm in names if nm.startswith("f_rest_"))
    if n_rest % 3:
        raise ValueError(f"{path}: {n_rest} f_rest coefficients is not a whole number per "
                         "channel")
    per_channel = n_rest // 3
    sh = np.zeros((n, per_channel + 1, 3), np.float32)
    for c in range(3):
        sh[:, 0, c] = rec[f"f_dc_{c}"]
        for b in range(per_channel):
            sh[:, b + 1, c] = rec[f"f_rest_{c * per_channel + b}"]
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    return {
        "means": t(np.stack([rec["x"], rec["y"], rec["z"]], 1)),
        "quats": t(np.stack([rec[f"rot_{i}"] for i in range(4)], 1)),
        "log_scales": t(np.stack([rec[f"scale_{i}"] for i in range(3)], 1)),
        "logit_opac": t(rec["opacity"]),
        "sh_dc": t(sh[:, :1]),
        "sh_rest": t(sh[:, 1:]),
    }
