"""Generates the golden fixtures in this directory from the REFERENCE's own code.

    python tests/golden/make_golden.py --reference /path/to/metal-gauss

The reference (nandometzger/metal-gauss) is pure PyTorch apart from its Metal
kernels, so everything it can compute on a CPU is used here as ground truth:
torch_ref.render / torch_ref.project (torch_ref.py:49-337), sh.eval_sh,
metal_backend.build_tile_lists with the exact ellipse test
(metal_backend.py:111-214), metal_backend.antialias_scale (:367-393),
ssim.ssim (ssim.py:49-108), selective_adam.SelectiveAdam, and
mipfilter.compute_3d_filter / apply_3d_filter with its autograd and the .ply
bake of train.export_ply (train.py:609-616), and mcmc.relocate / grow /
add_noise with their torch.multinomial / torch.randn_like draws recorded. Inputs are seeded
and stored in the fixtures, so tests never need the reference or this script.
The binning fixture takes its inputs from the CPU oracle's preprocess (the
reference's own binning consumes the Metal preprocess outputs, which cannot run
here); its outputs are the reference's build_tile_lists on those inputs.
"""

from __future__ import annotations

import argparse
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]


def np32(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy().astype(np.float32)


def scene_inputs(p: dict):
    means = p["means"].clone()
    quats = p["quats"].clone()
    scales = torch.exp(p["log_scales"])
    opac = torch.sigmoid(p["logit_opac"])
    sh = torch.cat([p["sh_dc"], p["sh_rest"]], 1)
    return means, quats, scales, opac, sh


def render_case(torch_ref, means, quats, scales, opac, sh, K, vm, W, H, sh_degree, tile,
                background, colors=None, loss="square", target=None, antialias=False):
    leaves = [t.clone().requires_grad_(True) for t in (means, quats, scales, opac)]
    shl = None if sh is None else sh.clone().requires_grad_(True)
    col = None if colors is None else colors.clone().requires_grad_(True)
    rgb, alpha, info = torch_ref.render(*leaves, shl, K, vm, W, H, sh_degree=sh_degree, tile=tile,
                                        background=background, colors=col, antialias=antialias)
    if loss == "square":
        L = rgb.square().mean() + 0.1 * alpha.square().mean()
    elif loss == "l1":
        L = (rgb - target).abs().mean()
    else:
        raise ValueError(loss)
    L.backward()
    out = dict(rgb=np32(rgb), alpha=np32(alpha), isect_total=np.int64(info["isect_total"]),
               g_means=np32(leaves[0].grad), g_quats=np32(leaves[1].grad),
               g_scales=np32(leaves[2].grad), g_opac=np32(leaves[3].grad))
    if shl is not None:
        out["g_sh"] = np32(shl.grad)
    if col is not None:
        out["g_colors"] = np32(col.grad)
    return out


def project_case(torch_ref, sh_mod, means, quats, scales, sh, K, vm, W, H, sh_degree):
    fx, fy, cx, cy = (float(K[0, 0]), float(K[1, 1]), float(K[0, 2]), float(K[1, 2]))
    cov3d = torch_ref.build_cov3d(quats, scales)
    uv, conic, depth, radius, valid, _ = torch_ref.project(means, cov3d, vm, fx, fy, cx, cy, W, H,
                                                           0.01, 100.0)
    cam_center = -vm[:3, :3].T @ vm[:3, 3]
    dirs = means - cam_center
    dirs = dirs / dirs.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    colors = (sh_mod.eval_sh(sh_degree, sh[:, : sh_mod.num_sh_bases(sh_degree)], dirs)
              + 0.5).clamp_min(0.0)
    return dict(p_uv=np32(uv), p_conic=np32(conic), p_depth=np32(depth),
                p_radius=np32(radius), p_valid=valid.numpy(), p_color=np32(colors))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of nandometzger/metal-gauss")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference).resolve()))
    sys.path.insert(0, str(ROOT))
    from metal_gauss import metal_backend, selective_adam, torch_ref  # noqa: E402
    from metal_gauss import sh as sh_mod  # noqa: E402
    from metal_gauss import ssim as ssim_mod  # noqa: E402

    import oracle  # noqa: E402
    from metal_gauss_b200 import scenes  # noqa: E402

    torch.set_num_threads(8)

    # -------------------------------------------------------- cfg1 (BASELINE)
    p, views, spec = scenes.config("cfg1")
    v = views[0]
    W, H = v.width, v.height
    means, quats, scales, opac, sh = scene_inputs(p)
    sh0 = sh[:, :1]
    target = scenes.random_target(W, H, seed=100)
    r = render_case(torch_ref, means, quats, scales, opac, sh0, v.K, v.viewmat, W, H, 0, 16,
                    spec["background"], loss="l1", target=target)
    pr = project_case(torch_ref, sh_mod, means, quats, scales, sh0, v.K, v.viewmat, W, H, 0)
    np.savez_compressed(HERE / "cfg1.npz", means=np32(means), quats=np32(quats),
                        scales=np32(scales), opac=np32(opac), sh=np32(sh0), K=np32(v.K),
                        viewmat=np32(v.viewmat), W=W, H=H, target=np32(target),
                        background=np.array(spec["background"], np.float32), **r, **pr)
    print("cfg1", r["isect_total"], float(r["alpha"].max()))

    # ---------------------------------------------------------- SH degree 3
    g = torch.Generator().manual_seed(3)
    n, W, H = 2000, 96, 72
    means = torch.randn(n, 3, generator=g) * 0.6 + torch.tensor([0.0, 0.0, 4.0])
    quats = torch.randn(n, 4, generator=g)
    scales = torch.rand(n, 3, generator=g) * 0.08 + 0.02
    opac = torch.rand(n, generator=g) * 0.7 + 0.15
    sh = torch.randn(n, 16, 3, generator=g) * 0.25
    K = scenes.intrinsics(W, H, 60.0)
    vm = scenes.look_at((0.3, -0.2, -0.5), (0.0, 0.0, 4.0), down=(0.0, 1.0, 0.0))
    r = render_case(torch_ref, means, quats, scales, opac, sh, K, vm, W, H, 3, 16, (0.0, 0.0, 0.0))
    pr = project_case(torch_ref, sh_mod, means, quats, scales, sh, K, vm, W, H, 3)
    np.savez_compressed(HERE / "sh3.npz", means=np32(means), quats=np32(quats),
                        scales=np32(scales), opac=np32(opac), sh=np32(sh), K=np32(K),
                        viewmat=np32(vm), W=W, H=H, **r, **pr)
    print("sh3", r["isect_total"])

    # --------------------------- every tile size, explicit colours (test_metal)
    torch.manual_seed(17)
    n = 300
    means = torch.randn(n, 3) * 0.6 + torch.tensor([0.0, 0.0, 4.0])
    quats = torch.randn(n, 4)
    scales = (torch.rand(n, 3) * 0.10 + 0.03) * torch.tensor([4.0, 0.5, 1.0])
    opac = torch.rand(n) * 0.7 + 0.15
    cols = torch.rand(n, 3)
    W, H = 100, 63
    K = torch.eye(3)
    f = 0.8 * max(W, H)
    K[0, 0], K[1, 1], K[0, 2], K[1, 2] = f, f, W / 2, H / 2
    vm = torch.eye(4)
    tiles = {}
    for tile in (8, 12, 16, 32):
        r = render_case(torch_ref, means, quats, scales, opac, None, K, vm, W, H, 3, tile,
                        (0.0, 0.0, 0.0), colors=cols)
        tiles.update({f"t{tile}_{k}": val for k, val in r.items()})
    np.savez_compressed(HERE / "tiles.npz", means=np32(means), quats=np32(quats),
                        scales=np32(scales), opac=np32(opac), colors=np32(cols), K=np32(K),
                        viewmat=np32(vm), W=W, H=H, **tiles)
    print("tiles done")

    # ------------------------------------------------------------- binning
    g = torch.Generator().manual_seed(1)
    n, W, H = 8000, 240, 320
    means = torch.randn(n, 3, generator=g) * 0.5
    means[:, 2] += 3.0
    quats = torch.randn(n, 4, generator=g)
    scales = torch.rand(n, 3, generator=g) * 0.08 + 0.005
    op = torch.rand(n, generator=g) * 0.9 + 0.05
    torch.randn(n, 16, 3, generator=g)  # keeps the stream aligned with test_metal_binning
    K = torch.tensor([[200.0, 0, W / 2], [0, 200.0, H / 2], [0, 0, 1.0]])
    vm = torch.eye(4)
    cam = oracle.camera(vm.numpy(), K.numpy(), W, H)
    pre = oracle.preprocess_forward(means.numpy(), quats.numpy(), scales.numpy(), None, None,
                                    op.numpy(), cam, -1)
    del pre["color"]
    out = dict(means=np32(means), quats=np32(quats), scales=np32(scales), opac=np32(op),
               K=np32(K), viewmat=np32(vm), W=W, H=H,
               **{f"pre_{k}": v for k, v in pre.items()})
    uv, rxy, conic, depth = (torch.from_numpy(pre[k]) for k in ("uv", "rxy", "conic", "depth"))
    valid = torch.from_numpy(pre["valid"]).bool()
    for tile in (16, 32):
        ids, offs, tx = metal_backend.build_tile_lists(uv, rxy[:, 0], depth, valid, W, H, tile,
                                                       ry=rxy[:, 1], conic=conic, opacity=op)
        ids_c, offs_c, _ = metal_backend.build_tile_lists(uv, rxy[:, 0], depth, valid, W, H, tile,
                                                          ry=rxy[:, 1])
        out[f"t{tile}_ids"] = ids.numpy().astype(np.int32)
        out[f"t{tile}_offsets"] = offs.numpy().astype(np.int32)
        out[f"t{tile}_box_count"] = np.int64(ids_c.numel())
        print("binning", tile, ids.numel(), "of", ids_c.numel())
    np.savez_compressed(HERE / "binning.npz", **out)

    # ----------------------------------------------------------- antialias
    torch.manual_seed(0)
    m = 512
    sx = torch.rand(m).double() * 5.0 + 0.01
    sy = torch.rand(m).double() * 5.0 + 0.01
    rho = (torch.rand(m).double() - 0.5) * 1.2
    a0, c0, b0 = sx * sx + 0.3, sy * sy + 0.3, rho * sx * sy
    det = a0 * c0 - b0 * b0
    conic = torch.stack([c0 / det, -b0 / det, a0 / det], -1).float()
    np.savez_compressed(HERE / "antialias.npz", conic=np32(conic),
                        scale=np32(metal_backend.antialias_scale(conic, 0.3)))

    # ---------------------------------------------------------------- SSIM
    g = torch.Generator().manual_seed(5)
    H, W = 37, 53
    a = torch.rand(H, W, 3, generator=g)
    b = torch.rand(H, W, 3, generator=g)
    k15 = ssim_mod.gaussian_kernel(device="cpu", groups=15)
    k9 = ssim_mod.gaussian_kernel(device="cpu", groups=9)
    al = a.clone().requires_grad_(True)
    s = ssim_mod.ssim(al, b, k15, k9)
    (gs,) = torch.autograd.grad(s, al)
    al2 = a.clone().requires_grad_(True)
    loss = 0.8 * (al2 - b).abs().mean() + 0.2 * (1.0 - ssim_mod.ssim(al2, b, k15, k9))
    (gl,) = torch.autograd.grad(loss, al2)
    np.savez_compressed(HERE / "ssim.npz", a=np32(a), b=np32(b), ssim=np.float64(s.item()),
                        g_ssim=np32(gs), loss=np.float64(loss.item()), g_loss=np32(gl),
                        window=np32(k15[0, 0, 0]))

    # ------------------------------------------------------ selective adam
    g = torch.Generator().manual_seed(9)
    rows = 40
    shapes = [(rows, 3), (rows, 15, 3), (rows,)]
    params = [torch.randn(*sh_, generator=g) for sh_ in shapes]
    grads, masks = [], []
    for step in range(6):
        grads.append([torch.randn(*sh_, generator=g) for sh_ in shapes])
        frac = 0.8 if step % 2 == 0 else 0.2          # masked and indexed paths
        masks.append(torch.rand(rows, generator=g) < frac)
    ps = [t.clone().requires_grad_(True) for t in params]
    opt = selective_adam.SelectiveAdam([{"params": [t], "lr": lr}
                                        for t, lr in zip(ps, (1e-2, 2.5e-3, 5e-2))], eps=1e-15)
    for step in range(6):
        for t, gr in zip(ps, grads[step]):
            t.grad = gr.clone()
        opt.step(masks[step])
    out = {f"p{i}": np32(t) for i, t in enumerate(params)}
    out.update({f"final{i}": np32(t) for i, t in enumerate(ps)})
    out.update({f"steps{i}": np32(opt.state[t]["steps"]) for i, t in enumerate(ps)})
    for step in range(6):
        out[f"mask{step}"] = masks[step].numpy()
        for i, gr in enumerate(grads[step]):
            out[f"g{step}_{i}"] = np32(gr)
    np.savez_compressed(HERE / "selective_adam.npz", lrs=np.array([1e-2, 2.5e-3, 5e-2]), **out)

    # ----------------------------------------------- boundary energy sweep
    W = H = 128
    F, Z = 100.0, 2.0
    Kb = torch.tensor([[F, 0, W / 2], [0, F, H / 2], [0, 0, 1.0]])
    qb = torch.tensor([[1.0, 0, 0, 0]])
    sb = torch.full((1, 3), 0.04)
    shb = torch.zeros(1, 16, 3)
    shb[:, 0] = 1.0
    ob = torch.tensor([0.99])
    us = np.arange(28.0, 36.0, 0.1)
    energy = []
    for u in us:
        x = (u - W / 2) * Z / F
        m = torch.tensor([[x, 0.0, Z]], dtype=torch.float32)
        rgb, _, _ = torch_ref.render(m, qb, sb, ob, shb, Kb, torch.eye(4), W, H, tile=32,
                                     sh_degree=3)
        energy.append(rgb.sum().item())
    np.savez_compressed(HERE / "boundary.npz", us=us, energy=np.array(energy))
    # ------------------------------------------------- Mip-Splatting 3D filter
    from metal_gauss import mipfilter  # noqa: E402

    class _FView:
        def __init__(self, K, vm, W, H):
            self.K, self.viewmat = K, vm
            self.image = torch.zeros(H, W, 3, dtype=torch.uint8)

    g = torch.Generator().manual_seed(17)
    nf = 400
    fmeans = torch.randn(nf, 3, generator=g) * 1.5
    fmeans[:5, 2] = 50.0                       # behind every camera: unseen
    fviews, fk, fvm, fwh = [], [], [], []
    for i, (ang, f, W, H) in enumerate([(0.0, 300.0, 160, 120), (0.7, 450.0, 200, 100),
                                        (-0.5, 250.0, 128, 128)]):
        vm = torch.eye(4)
        c, s_ = math.cos(ang), math.sin(ang)
        vm[:3, :3] = torch.tensor([[c, 0.0, -s_], [0.0, 1.0, 0.0], [s_, 0.0, c]])
        vm[2, 3] = 5.0 + i
        K = torch.tensor([[f, 0.0, W / 2], [0.0, f, H / 2], [0.0, 0.0, 1.0]])
        fviews.append(_FView(K, vm, W, H))
        fk.append(np32(K)); fvm.append(np32(vm)); fwh.append((W, H))
    filt = mipfilter.compute_3d_filter(fmeans, fviews)
    fs = (torch.rand(nf, 3, generator=g) * 0.2 + 1e-3).requires_grad_(True)
    fo = torch.rand(nf, generator=g).requires_grad_(True)
    ns, no = mipfilter.apply_3d_filter(fs, fo, filt)
    gs = torch.randn(nf, 3, generator=g)
    go = torch.randn(nf, generator=g)
    (ns * gs).sum().backward(retain_graph=True)
    (no * go).sum().backward()
    # the bake of train.export_ply (train.py:609-616) on log / logit parameters
    fls, flo = torch.log(fs.detach()), torch.logit(fo.detach().clamp(1e-4, 1 - 1e-4))
    sc, op = mipfilter.apply_3d_filter(torch.exp(fls), torch.sigmoid(flo), filt)
    baked_ls = torch.log(sc.clamp_min(1e-12))
    op = op.clamp(1e-6, 1.0 - 1e-6)
    baked_lo = torch.log(op / (1.0 - op))
    np.savez_compressed(HERE / "filter3d.npz", means=np32(fmeans), K=np.stack(fk),
                        viewmat=np.stack(fvm), wh=np.array(fwh), filter=np32(filt),
                        scales=np32(fs), opac=np32(fo), new_scales=np32(ns), new_opac=np32(no),
                        g_scales=np32(gs), g_opac=np32(go), d_scales=np32(fs.grad),
                        d_opac=np32(fo.grad), log_scales=np32(fls), logit_opac=np32(flo),
                        baked_log_scales=np32(baked_ls), baked_logit_opac=np32(baked_lo))
    # ------------------------------------------------------------ MCMC
    from metal_gauss import mcmc  # noqa: E402

    def mcmc_params(n, seed):
        gm = torch.Generator().manual_seed(seed)
        return {"means": torch.randn(n, 3, generator=gm),
                "quats": torch.randn(n, 4, generator=gm),
                "log_scales": torch.randn(n, 3, generator=gm) * 0.5 - 3.0,
                "logit_opac": torch.randn(n, generator=gm) * 3.0 - 2.0,
                "sh_dc": torch.randn(n, 1, 3, generator=gm),
                "sh_rest": torch.randn(n, 15, 3, generator=gm) * 0.1}

    captured = {}
    real_multinomial, real_randn_like = torch.multinomial, torch.randn_like

    def multinomial(w, k, replacement=False, **kw):
        out = real_multinomial(w, k, replacement=replacement, **kw)
        captured["draw"] = out.clone()
        return out

    def randn_like(t, **kw):
        out = real_randn_like(t, **kw)
        captured["eps"] = out.clone()
        return out

    torch.multinomial, torch.randn_like = multinomial, randn_like
    try:
        torch.manual_seed(23)
        pr = mcmc_params(300, 29)
        before = {k: v.clone() for k, v in pr.items()}
        opac_b = torch.sigmoid(before["logit_opac"])
        alive = (opac_b >= 0.005).nonzero(as_tuple=True)[0]
        moved = mcmc.relocate(pr)
        reloc_picks = alive[captured["draw"]]
        pg = mcmc_params(300, 31)
        gbefore = {k: v.clone() for k, v in pg.items()}
        new_active = mcmc.grow(pg, 260, 200)
        grow_picks = captured["draw"].clone()
        pn = mcmc_params(300, 37)
        nbefore = {k: v.clone() for k, v in pn.items()}
        mcmc.add_noise(pn, 1.6e-4, 4e4)
        eps = captured["eps"].clone()
    finally:
        torch.multinomial, torch.randn_like = real_multinomial, real_randn_like
    out = {"moved": np.int64(moved), "reloc_picks": reloc_picks.numpy().astype(np.int32),
           "new_active": np.int64(new_active), "grow_picks": grow_picks.numpy().astype(np.int32),
           "eps": np32(eps)}
    for tag, b, a in (("reloc", before, pr), ("grow", gbefore, pg), ("noise", nbefore, pn)):
        for k in b:
            out[f"{tag}_before_{k}"] = np32(b[k])
            out[f"{tag}_after_{k}"] = np32(a[k])
    np.savez_compressed(HERE / "mcmc.npz", **out)
    for f_ in sorted(HERE.glob("*.npz")):
        print(f_.name, f_.stat().st_size)


if __name__ == "__main__":
    main()
