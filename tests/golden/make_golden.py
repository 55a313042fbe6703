"""Generate the golden fixtures under tests/golden/ from the reference's own
Python implementation (depth_anything_v2/*.py, run on the CPU with torch).

Run where the reference checkout is importable:
    python tests/golden/make_golden.py /path/to/Depth-Anything-V2
The fixtures are small .npz files; the GPU box never needs the reference.

Contents:
  ops.npz        per-operator outputs of the reference model's own modules /
                 torch functional calls it makes (LayerNorm eps 1e-6, nn.GELU,
                 softmax, align-corners bilinear, Conv2d, ConvTranspose2d,
                 DINOv2.interpolate_pos_encoding, Attention.forward);
  model_vits.npz DepthAnythingV2('vits') forward with seeded weights
                 (dav2file.random_state_dict(seed=0)) on seeded tensors;
  image_vits.npz infer_image (cv2 bicubic preprocessing + model + bilinear to
                 the source size) on a seeded BGR8 image;
  model_vits_metric.npz  the metric-depth model (metric_depth/depth_anything_v2,
                 sigmoid head x max_depth 20) with the base and strong weights on
                 the model_vits inputs;
  image_vits_518.npz  the same at the benchmark's full size: a 518x518 BGR8
                 image (np.random.default_rng(0), the BASELINE CPU config's
                 image), input size 518, ViT-S with random_state_dict(seed=0);
                 depth stored as float16 (the tests compare at 1e-2).
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT / "depth-anything-v2_b200"))


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    import torch
    import torch.nn.functional as F
    from depth_anything_v2.dinov2_layers.attention import Attention
    from depth_anything_v2.dpt import DepthAnythingV2

    from dav2_b200 import dav2file

    torch.manual_seed(0)
    rng = np.random.default_rng(1234)
    out = {}
    # LayerNorm (nn.LayerNorm(eps=1e-6) as in dinov2.py)
    x = rng.standard_normal((37, 384)).astype(np.float32) * 2 + 0.3
    w = rng.standard_normal(384).astype(np.float32)
    b = rng.standard_normal(384).astype(np.float32)
    out["ln_x"], out["ln_w"], out["ln_b"] = x, w, b
    out["ln_y"] = F.layer_norm(torch.from_numpy(x), (384,), torch.from_numpy(w), torch.from_numpy(b), 1e-6).numpy()
    # GELU (nn.GELU, exact erf)
    g = rng.standard_normal(4096).astype(np.float32) * 4
    out["gelu_x"], out["gelu_y"] = g, torch.nn.GELU()(torch.from_numpy(g)).numpy()
    # softmax of q*scale . k (attention.py:53-58)
    s = rng.standard_normal((16, 300)).astype(np.float32) * 4
    out["sm_x"], out["sm_y"] = s, (torch.from_numpy(s) * 0.125).softmax(-1).numpy()
    # align-corners bilinear (util/blocks.py:165, dpt.py:149)
    bl = rng.standard_normal((3, 19, 23)).astype(np.float32)
    out["bl_x"] = bl
    out["bl_y"] = F.interpolate(torch.from_numpy(bl)[None], (37, 45), mode="bilinear", align_corners=True)[0].numpy()
    # Conv2d 3x3 pad 1 and stride 2
    cx = rng.standard_normal((5, 11, 9)).astype(np.float32)
    cw = rng.standard_normal((7, 5, 3, 3)).astype(np.float32) * 0.2
    cb = rng.standard_normal(7).astype(np.float32)
    out["cv_x"], out["cv_w"], out["cv_b"] = cx, cw, cb
    out["cv_y1"] = F.conv2d(torch.from_numpy(cx)[None], torch.from_numpy(cw), torch.from_numpy(cb), 1, 1)[0].numpy()
    out["cv_y2"] = F.conv2d(torch.from_numpy(cx)[None], torch.from_numpy(cw), torch.from_numpy(cb), 2, 1)[0].numpy()
    # ConvTranspose2d k4 s4 (dpt.py:60-64)
    tx = rng.standard_normal((8, 5, 6)).astype(np.float32)
    tw = rng.standard_normal((8, 6, 4, 4)).astype(np.float32) * 0.2
    tb = rng.standard_normal(6).astype(np.float32)
    out["ct_x"], out["ct_w"], out["ct_b"] = tx, tw, tb
    out["ct_y"] = F.conv_transpose2d(torch.from_numpy(tx)[None], torch.from_numpy(tw), torch.from_numpy(tb),
                                     stride=4)[0].numpy()
    # positional-embedding interpolation (dinov2.py:184-213) for a 5x7 patch grid
    m = DepthAnythingV2(encoder="vits", features=64, out_channels=[48, 96, 192, 384]).eval()
    # the input grid is regenerated from its seed by the tests (not stored)
    pos = (np.random.default_rng(5).standard_normal((1, 1370, 384)) * 0.02).astype(np.float32)
    with torch.no_grad():
        m.pretrained.pos_embed.copy_(torch.from_numpy(pos))
        tokens = torch.zeros(1, 5 * 7 + 1, 384)
        pe = m.pretrained.interpolate_pos_encoding(tokens, 7 * 14, 5 * 14)  # x is [B, C, w, h] = 98 x 70
    out["pos_out"] = pe.numpy()
    # Attention module (attention.py:49-62), dim 128 / 2 heads, on a seeded qkv
    att = Attention(128, num_heads=2, qkv_bias=True).eval()
    ax = rng.standard_normal((1, 9, 128)).astype(np.float32)
    with torch.no_grad():
        for p in att.parameters():
            p.copy_(torch.from_numpy(rng.standard_normal(p.shape).astype(np.float32) * 0.1))
        qkv = att.qkv(torch.from_numpy(ax))
        # attention output before the projection, by the module's own steps
        B, N, C = 1, 9, 128
        q = qkv.reshape(B, N, 3, 2, 64).permute(2, 0, 3, 1, 4)
        a = ((q[0] * att.scale) @ q[1].transpose(-2, -1)).softmax(-1)
        o = (a @ q[2]).transpose(1, 2).reshape(B, N, C)
    out["att_qkv"], out["att_out"] = qkv[0].numpy(), o[0].numpy()
    np.savez_compressed(HERE / "ops.npz", **out)

    # full model, seeded weights, planar inputs
    sd = dav2file.random_state_dict("vits", seed=0)
    sd_strong = dav2file.random_state_dict("vits", seed=1, std=0.05, bias_std=0.02)
    res = {}
    for tag, state in (("base", sd), ("strong", sd_strong)):
        model = DepthAnythingV2(encoder="vits", features=64, out_channels=[48, 96, 192, 384]).eval()
        model.load_state_dict({k: torch.from_numpy(v) for k, v in state.items()})
        for shape in ((70, 98), (126, 126)):
            img = np.random.default_rng(shape[0]).standard_normal((3, *shape)).astype(np.float32)
            with torch.no_grad():
                d = model(torch.from_numpy(img)[None])[0].numpy()
            res[f"{tag}_{shape[0]}x{shape[1]}_in"] = img
            res[f"{tag}_{shape[0]}x{shape[1]}_out"] = d
    np.savez_compressed(HERE / "model_vits.npz", **res)

    # infer_image: BGR8 -> cv2 bicubic -> model -> bilinear to the source size
    model = DepthAnythingV2(encoder="vits", features=64, out_channels=[48, 96, 192, 384]).eval()
    model.load_state_dict({k: torch.from_numpy(v) for k, v in sd_strong.items()})
    bgr = np.random.default_rng(77).integers(0, 256, (37, 53, 3), dtype=np.uint8)
    tensor, (h, w) = model.image2tensor(bgr, 70)
    depth = model.infer_image(bgr, 70)
    np.savez_compressed(HERE / "image_vits.npz", bgr=bgr, tensor=tensor[0].numpy(), depth=depth.astype(np.float32))

    # metric-depth model: same network, sigmoid head scaled by max_depth
    import subprocess  # the metric package shares the relative package's name: run it in a child
    code = (
        "import sys, numpy as np, torch\n"
        f"sys.path.insert(0, {str(Path(reference) / 'metric_depth')!r})\n"
        "from depth_anything_v2.dpt import DepthAnythingV2\n"
        f"sys.path.insert(0, {str(ROOT / 'depth-anything-v2_b200')!r})\n"
        "from dav2_b200 import dav2file\n"
        "res = {}\n"
        f"fx = np.load({str(HERE / 'model_vits.npz')!r})\n"
        "for tag, kw in (('base', dict(seed=0)), ('strong', dict(seed=1, std=0.05, bias_std=0.02))):\n"
        "    sd = dav2file.random_state_dict('vits', **kw)\n"
        "    m = DepthAnythingV2(encoder='vits', features=64, out_channels=[48, 96, 192, 384], max_depth=20.0).eval()\n"
        "    m.load_state_dict({k: torch.from_numpy(v) for k, v in sd.items()})\n"
        "    for shape in ('70x98', '126x126'):\n"
        "        img = fx[f'{tag}_{shape}_in']\n"
        "        with torch.no_grad():\n"
        "            res[f'{tag}_{shape}_in'] = img\n"
        "            res[f'{tag}_{shape}_out'] = m(torch.from_numpy(img)[None])[0].numpy()\n"
        f"np.savez_compressed({str(HERE / 'model_vits_metric.npz')!r}, **res)\n")
    subprocess.run([sys.executable, "-c", code], check=True)

    # full size: 518x518 source, input size 518 (1370 tokens)
    model = DepthAnythingV2(encoder="vits", features=64, out_channels=[48, 96, 192, 384]).eval()
    model.load_state_dict({k: torch.from_numpy(v) for k, v in sd.items()})
    bgr = np.random.default_rng(0).integers(0, 256, (518, 518, 3), dtype=np.uint8)
    with torch.no_grad():
        depth = model.infer_image(bgr, 518)
    np.savez_compressed(HERE / "image_vits_518.npz", depth=depth.astype(np.float16))
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    # the reference checkout: the first argument, else DAV2_REFERENCE_DIR
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DAV2_REFERENCE_DIR", "")
    if not ref:
        sys.exit(f"usage: python {Path(__file__).name} <reference checkout> (or set DAV2_REFERENCE_DIR)")
    main(ref)
