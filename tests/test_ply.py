"""INRIA .ply export/import (the reference's train.export_ply layout,
metal_gauss/train.py:583-624, io.py:1-11): header text, property order,
channel-major f_rest, stored (pre-activation) values, and bit-exact round
trips. Runs on the CPU."""

import numpy as np
import pytest
import torch

from metal_gauss_b200 import ply


def _params(n=37, rest=15, seed=0):
    g = np.random.default_rng(seed)
    f = lambda *s: torch.from_numpy(g.standard_normal(s).astype(np.float32))
    return {"means": f(n, 3), "quats": f(n, 4), "log_scales": f(n, 3), "logit_opac": f(n),
            "sh_dc": f(n, 1, 3), "sh_rest": f(n, rest, 3)}


def test_header_and_property_order(tmp_path):
    p = _params(5)
    path = tmp_path / "m.ply"
    ply.export_ply(p, path)
    raw = path.read_bytes()
    head = raw[:raw.index(b"end_header\n") + len(b"end_header\n")].decode("ascii")
    lines = head.splitlines()
    assert lines[:3] == ["ply", "format binary_little_endian 1.0", "element vertex 5"]
    props = [ln.split()[2] for ln in lines[3:-1]]
    assert all(ln.split()[:2] == ["property", "float"] for ln in lines[3:-1])
    assert props == (["x", "y", "z", "f_dc_0", "f_dc_1", "f_dc_2"]
                     + [f"f_rest_{i}" for i in range(45)]
                     + ["opacity", "scale_0", "scale_1", "scale_2",
                        "rot_0", "rot_1", "rot_2", "rot_3"])
    assert lines[-1] == "end_header"
    assert len(raw) == len(head) + 5 * 59 * 4


def test_values_are_stored_form_and_channel_major(tmp_path):
    p = _params(3)
    path = tmp_path / "m.ply"
    ply.export_ply(p, path)
    raw = path.read_bytes()
    body = np.frombuffer(raw[raw.index(b"end_header\n") + 11:], dtype="<f4").reshape(3, 59)
    assert np.array_equal(body[:, 0:3], p["means"].numpy())
    assert np.array_equal(body[:, 3:6], p["sh_dc"].numpy()[:, 0, :])
    rest = p["sh_rest"].numpy()          # (n, 15 bands, 3 channels)
    for c in range(3):                   # f_rest_[c*15 + b] = band b+1 of channel c
        assert np.array_equal(body[:, 6 + 15 * c:6 + 15 * (c + 1)], rest[:, :, c])
    assert np.array_equal(body[:, 51], p["logit_opac"].numpy())      # a logit, as stored
    assert np.array_equal(body[:, 52:55], p["log_scales"].numpy())   # logarithms, as stored
    assert np.array_equal(body[:, 55:59], p["quats"].numpy())        # not normalised


@pytest.mark.parametrize("rest", [0, 3, 8, 15])
def test_round_trip_is_bit_exact(tmp_path, rest):
    p = _params(101, rest, seed=rest)
    path = tmp_path / f"r{rest}.ply"
    ply.export_ply(p, path)
    q = ply.read_ply(path)
    for k in p:
        assert torch.equal(q[k], p[k].reshape(q[k].shape)), k
    # a second export of what was read is byte-identical
    path2 = tmp_path / f"r{rest}_again.ply"
    ply.export_ply(q, path2)
    assert path.read_bytes() == path2.read_bytes()


def test_fused_sh_input_matches_split(tmp_path):
    p = _params(9)
    fused = dict(p)
    fused["sh"] = torch.cat([fused.pop("sh_dc"), fused.pop("sh_rest")], 1)
    ply.export_ply(p, tmp_path / "a.ply")
    ply.export_ply(fused, tmp_path / "b.ply")
    assert (tmp_path / "a.ply").read_bytes() == (tmp_path / "b.ply").read_bytes()


def test_reader_rejects_what_it_cannot_read(tmp_path):
    bad = tmp_path / "ascii.ply"
    bad.write_bytes(b"ply\nformat ascii 1.0\nelement vertex 0\nend_header\n")
    with pytest.raises(ValueError, match="binary little-endian"):
        ply.read_ply(bad)
    dbl = tmp_path / "double.ply"
    dbl.write_bytes(b"ply\nformat binary_little_endian 1.0\nelement vertex 1\n"
                    b"property double x\nend_header\n" + bytes(8))
    with pytest.raises(ValueError, match="not float"):
        ply.read_ply(dbl)


def test_export_bakes_the_3d_filter_as_the_reference_does(tmp_path):
    """train.export_ply with filter_3d (train.py:609-616): the filtered scales
    and opacity written in log / logit space, against the values the
    reference's own mipfilter and bake produced (tests/golden/filter3d.npz)."""
    from tests.golden.fixtures import load
    f = load("filter3d")
    n = f["filter"].shape[0]
    p = _params(n)
    p["log_scales"] = torch.from_numpy(f["log_scales"])
    p["logit_opac"] = torch.from_numpy(f["logit_opac"])
    ply.export_ply(p, tmp_path / "baked.ply", filter_3d=torch.from_numpy(f["filter"]))
    q = ply.read_ply(tmp_path / "baked.ply")
    assert np.abs(q["log_scales"].numpy() - f["baked_log_scales"]).max() < 1e-5
    assert np.abs(q["logit_opac"].numpy() - f["baked_logit_opac"]).max() < 1e-4
    assert torch.equal(q["means"], p["means"].float())
    # a zero filter changes the scales by at most rounding
    ply.export_ply(p, tmp_path / "zero.ply", filter_3d=torch.zeros(n))
    z = ply.read_ply(tmp_path / "zero.ply")
    assert np.abs(z["log_scales"].numpy() - f["log_scales"]).max() < 1e-6
