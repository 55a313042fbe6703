"""PyTorch-CPU restatement of the reference graph — the CPU baseline.

TEST / BASELINE INFRASTRUCTURE ONLY (never part of the product). The
reference's own CPU execution of this path is its Python model run by PyTorch
on the CPU in fp32 (depth_anything_v2/dpt.py:153-221 driving
dinov2.py:184-328, dinov2_layers/{block,attention,mlp}.py and
util/blocks.py); it is the accuracy authority the reference names. That
source cannot ship with this repository, so this module restates the same
forward pass as plain torch functional calls on a state dict — the same
operators (F.linear, F.layer_norm, F.gelu, softmax, F.conv2d,
F.conv_transpose2d, F.interpolate) in the same order — so that it costs what
the reference's CPU run costs. tests/test_torch_graph_cpu.py pins it to the
fixtures produced by the reference model itself.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

ARCH = {
    "vits": (384, 6, 12, (2, 5, 8, 11), 64, (48, 96, 192, 384)),
    "vitb": (768, 12, 12, (2, 5, 8, 11), 128, (96, 192, 384, 768)),
    "vitl": (1024, 16, 24, (4, 11, 17, 23), 256, (256, 512, 1024, 1024)),
}


def to_torch(sd: dict) -> dict:
    return {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in sd.items()}


def _pos_embed(w, pos, ph, pw):
    """dinov2.py:184-213: bicubic resize of the 37x37 grid with
    scale_factor = ((ph + 0.1)/37, (pw + 0.1)/37)."""
    d = pos.shape[-1]
    n = pos.shape[1] - 1
    if n == ph * pw and ph == pw:
        return pos
    g = int(math.sqrt(n))
    grid = pos[:, 1:].reshape(1, g, g, d).permute(0, 3, 1, 2)
    grid = F.interpolate(grid, scale_factor=((ph + 0.1) / g, (pw + 0.1) / g), mode="bicubic", antialias=False)
    return torch.cat((pos[:, :1], grid.permute(0, 2, 3, 1).reshape(1, -1, d)), dim=1)


def encoder(w, x, name):
    d, heads, blocks, taps, _, _ = ARCH[name]
    b, _, h, wd = x.shape
    ph, pw = h // 14, wd // 14
    t = F.conv2d(x, w["pretrained.patch_embed.proj.weight"], w["pretrained.patch_embed.proj.bias"], stride=14)
    t = t.flatten(2).transpose(1, 2)
    t = torch.cat((w["pretrained.cls_token"].expand(b, -1, -1), t), dim=1)
    t = t + _pos_embed(w, w["pretrained.pos_embed"], ph, pw)
    feats = []
    n = t.shape[1]
    for i in range(blocks):
        p = f"pretrained.blocks.{i}"
        y = F.layer_norm(t, (d,), w[p + ".norm1.weight"], w[p + ".norm1.bias"], 1e-6)
        qkv = F.linear(y, w[p + ".attn.qkv.weight"], w[p + ".attn.qkv.bias"])
        qkv = qkv.reshape(b, n, 3, heads, d // heads).permute(2, 0, 3, 1, 4)
        a = ((qkv[0] * (d // heads) ** -0.5) @ qkv[1].transpose(-2, -1)).softmax(-1)
        y = (a @ qkv[2]).transpose(1, 2).reshape(b, n, d)
        y = F.linear(y, w[p + ".attn.proj.weight"], w[p + ".attn.proj.bias"])
        t = t + y * w[p + ".ls1.gamma"]
        y = F.layer_norm(t, (d,), w[p + ".norm2.weight"], w[p + ".norm2.bias"], 1e-6)
        y = F.gelu(F.linear(y, w[p + ".mlp.fc1.weight"], w[p + ".mlp.fc1.bias"]))
        y = F.linear(y, w[p + ".mlp.fc2.weight"], w[p + ".mlp.fc2.bias"])
        t = t + y * w[p + ".ls2.gamma"]
        if i in taps:
            feats.append(F.layer_norm(t, (d,), w["pretrained.norm.weight"], w["pretrained.norm.bias"], 1e-6)[:, 1:])
    return feats, ph, pw


def _rcu(w, x, p):
    y = F.conv2d(F.relu(x), w[p + ".conv1.weight"], w[p + ".conv1.bias"], padding=1)
    y = F.conv2d(F.relu(y), w[p + ".conv2.weight"], w[p + ".conv2.bias"], padding=1)
    return y + x


def _fusion(w, path, skip, p, size):
    if skip is not None:
        path = path + _rcu(w, skip, p + ".resConfUnit1")
    path = _rcu(w, path, p + ".resConfUnit2")
    path = F.interpolate(path, size=size, mode="bilinear", align_corners=True)
    return F.conv2d(path, w[p + ".out_conv.weight"], w[p + ".out_conv.bias"])


def head(w, feats, ph, pw, name, metric_max_depth=0.0):
    h = "depth_head"
    out = []
    for i, f in enumerate(feats):
        x = f.permute(0, 2, 1).reshape(f.shape[0], f.shape[-1], ph, pw)
        x = F.conv2d(x, w[f"{h}.projects.{i}.weight"], w[f"{h}.projects.{i}.bias"])
        if i == 0:
            x = F.conv_transpose2d(x, w[f"{h}.resize_layers.0.weight"], w[f"{h}.resize_layers.0.bias"], stride=4)
        elif i == 1:
            x = F.conv_transpose2d(x, w[f"{h}.resize_layers.1.weight"], w[f"{h}.resize_layers.1.bias"], stride=2)
        elif i == 3:
            x = F.conv2d(x, w[f"{h}.resize_layers.3.weight"], w[f"{h}.resize_layers.3.bias"], stride=2, padding=1)
        out.append(x)
    rn = [F.conv2d(out[i], w[f"{h}.scratch.layer{i + 1}_rn.weight"], None, padding=1) for i in range(4)]
    s = f"{h}.scratch"
    path = _fusion(w, rn[3], None, s + ".refinenet4", rn[2].shape[2:])
    path = _fusion(w, path, rn[2], s + ".refinenet3", rn[1].shape[2:])
    path = _fusion(w, path, rn[1], s + ".refinenet2", rn[0].shape[2:])
    path = _fusion(w, path, rn[0], s + ".refinenet1", (rn[0].shape[2] * 2, rn[0].shape[3] * 2))
    y = F.conv2d(path, w[s + ".output_conv1.weight"], w[s + ".output_conv1.bias"], padding=1)
    y = F.interpolate(y, (ph * 14, pw * 14), mode="bilinear", align_corners=True)
    y = F.relu(F.conv2d(y, w[s + ".output_conv2.0.weight"], w[s + ".output_conv2.0.bias"], padding=1))
    y = F.conv2d(y, w[s + ".output_conv2.2.weight"], w[s + ".output_conv2.2.bias"])
    y = torch.sigmoid(y) * metric_max_depth if metric_max_depth > 0 else F.relu(y)
    return y[:, 0]


@torch.inference_mode()
def forward(w, images, name, out_size=None, metric_max_depth=0.0):
    """images: float32 [B, 3, H, W] (normalized RGB) -> depth [B, H, W]
    (or [B, out_h, out_w] with the align-corners resize of infer_image);
    metric_max_depth > 0 selects the metric head (sigmoid * max depth)."""
    x = images if isinstance(images, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(images))
    feats, ph, pw = encoder(w, x, name)
    d = head(w, feats, ph, pw, name, metric_max_depth)
    if out_size is not None and tuple(out_size) != tuple(d.shape[-2:]):
        d = F.interpolate(d[:, None], out_size, mode="bilinear", align_corners=True)[:, 0]
    return d
