"""The bf16 precision (BASELINE configuration 3's arithmetic: ViT-B, bf16
activations, f32 accumulation), the high-resolution frame path
(configuration 5's: 1920x1080 BGR8 frames resized bilinearly to a square
1036x1036 input, depth back at 1920x1080) and the normalizing device submit
path (the reference's GPU submit sequence without graphics interop).

References: the fp32 reference forward (oracle/torch_graph.py, pinned to the
reference model's own fixtures) and the oracle's restatements of the
preprocessing, min/max normalization and align-corners resize. bf16 has no
counterpart in the reference (fp16 only): a single block and the whole graph
are held to 1e-2 of fp32 (PyTorch's own bf16-autocast distance from fp32 on
the same model is printed beside it). Models: tests/models.py."""
import ctypes

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
import torch_graph
from abi_helpers import create
from dav2_b200 import capi, dav2file
from models import nondegenerate

pytestmark = pytest.mark.gpu


def rel(got, want):
    return float(np.abs(got.astype(np.float64) - want).max() / np.abs(want).max())


@pytest.fixture(scope="module")
def vitb(tmp_path_factory, dav2lib):
    sd = nondegenerate("vitb")
    path = tmp_path_factory.mktemp("vitb") / "vitb.dav2"
    dav2file.write_dav2(path, sd, "vitb")
    return path, sd


@pytest.fixture(scope="module")
def vits(tmp_path_factory, dav2lib):
    sd = nondegenerate("vits")
    path = tmp_path_factory.mktemp("vits") / "vits.dav2"
    dav2file.write_dav2(path, sd, "vits")
    return path, sd


def torch_block(w, x, i, heads):
    """One DINOv2 block in fp32 (the reference's dinov2_layers/block.py order)."""
    d = x.shape[-1]
    p = f"pretrained.blocks.{i}"
    n = x.shape[0]
    y = F.layer_norm(x, (d,), w[p + ".norm1.weight"], w[p + ".norm1.bias"], 1e-6)
    qkv = F.linear(y, w[p + ".attn.qkv.weight"], w[p + ".attn.qkv.bias"]).reshape(n, 3, heads, 64).permute(1, 2, 0, 3)
    a = ((qkv[0] * 0.125) @ qkv[1].transpose(-2, -1)).softmax(-1)
    y = (a @ qkv[2]).transpose(0, 1).reshape(n, d)
    x = x + F.linear(y, w[p + ".attn.proj.weight"], w[p + ".attn.proj.bias"]) * w[p + ".ls1.gamma"]
    y = F.layer_norm(x, (d,), w[p + ".norm2.weight"], w[p + ".norm2.bias"], 1e-6)
    y = F.linear(F.gelu(F.linear(y, w[p + ".mlp.fc1.weight"], w[p + ".mlp.fc1.bias"])), w[p + ".mlp.fc2.weight"],
                 w[p + ".mlp.fc2.bias"])
    return x + y * w[p + ".ls2.gamma"]


def test_vitb_bf16_blocks_vs_fp32(cuda, dav2lib, vitb):
    path, sd = vitb
    rc, ctx = create(dav2lib, path, "vitb", capi.FLAGS["bf16"])
    assert rc == 0, dav2lib.dav2_last_error()
    w = torch_graph.to_torch(sd)
    try:
        imgs = [np.random.default_rng(s).integers(0, 256, (518, 518, 3), dtype=np.uint8) for s in (0, 1)]
        x = np.concatenate([oracle.embed(sd, oracle.preprocess_bgr8(b, 518, 518), "vitb") for b in imgs])
        for i in range(12):
            out = np.empty_like(x)
            assert dav2lib.dav2_probe_encoder_block(ctx, 2, 518, 518, i, x.ctypes.data, out.ctypes.data, None,
                                                    None) == 0, dav2lib.dav2_last_error()
            if i in (0, 5, 11):
                with torch.inference_mode():
                    want = torch.cat([torch_block(w, torch.from_numpy(x[k * 1370:(k + 1) * 1370]), i, 12)
                                      for k in range(2)]).numpy()
                r = rel(out, want)
                print(f"vitb bf16 block {i}: max rel {r:.2e}")
                assert r < 1e-2
            x = out
    finally:
        dav2lib.dav2_destroy(ctx)


def test_vitb_bf16_full_graph(cuda, dav2lib, vitb):
    """Two 518x518 BGR8 images through the batched host entry point."""
    path, sd = vitb
    imgs = np.stack([np.random.default_rng(s).integers(0, 256, (518, 518, 3), dtype=np.uint8) for s in (0, 1)])
    rc, ctx = create(dav2lib, path, "vitb", capi.FLAGS["bf16"])
    assert rc == 0, dav2lib.dav2_last_error()
    try:
        got = np.zeros((2, 518, 518), np.float32)
        assert dav2lib.dav2_infer_bgr8_batch(ctx, imgs.ctypes.data, 2, 518, 518, 518 * 3, 518 * 518 * 3, 518,
                                             got.ctypes.data, got.size) == 0, dav2lib.dav2_last_error()
    finally:
        dav2lib.dav2_destroy(ctx)
    w = torch_graph.to_torch(sd)
    x = np.stack([oracle.preprocess_bgr8(b, 518, 518) for b in imgs])
    fp32 = torch_graph.forward(w, x, "vitb").numpy()
    with torch.autocast("cpu", dtype=torch.bfloat16):
        auto = torch_graph.forward(w, x, "vitb").float().numpy()
    for k in range(2):
        r, floor = rel(got[k], fp32[k]), rel(auto[k], fp32[k])
        print(f"vitb bf16 image {k}: vs fp32 {r:.2e} (PyTorch bf16 autocast vs fp32 {floor:.2e}); "
              f"vs autocast {rel(got[k], auto[k]):.2e}")
        assert fp32[k].min() > 0  # every pixel carries signal in this model
        assert r < 1e-2


@pytest.mark.parametrize("prec", ["fp16", "bf16"])
def test_frames_1920x1080_to_1036(cuda, dav2lib, vits, prec):
    """The configuration-5 frame path on ViT-S (5477 tokens): two 1920x1080
    frames (np.random.default_rng(frame index)) on the device, padded rows."""
    path, sd = vits
    W, H, N = 1920, 1080, 1036
    frames = np.stack([np.random.default_rng(f).integers(0, 256, (H, W, 3), dtype=np.uint8) for f in (0, 1)])
    row = W * 3 + 32
    buf = np.zeros((2, H, row), np.uint8)
    buf[:, :, :W * 3] = frames.reshape(2, H, W * 3)
    rc, ctx = create(dav2lib, path, "vits", capi.FLAGS[prec])
    assert rc == 0, dav2lib.dav2_last_error()
    try:
        dbuf = torch.from_numpy(buf).cuda()
        out = torch.full((2, H, W), -1.0, device="cuda")
        s = torch.cuda.Stream()
        assert dav2lib.dav2_infer_device_frames_bgr8(ctx, dbuf.data_ptr(), 2, W, H, row, row * H, N, out.data_ptr(),
                                                     ctypes.c_void_p(s.cuda_stream)) == 0, dav2lib.dav2_last_error()
        assert dav2lib.dav2_synchronize(ctx) == 0, dav2lib.dav2_last_error()
        assert dav2lib.dav2_infer_device_frames_bgr8(ctx, dbuf.data_ptr(), 2, W, H, row, row * H, 1030, out.data_ptr(),
                                                     None) == 1  # not a multiple of 14
        got = out.cpu().numpy()
    finally:
        dav2lib.dav2_destroy(ctx)
    w = torch_graph.to_torch(sd)
    for k in range(2):
        x = oracle.preprocess_bgr8_bilinear(frames[k], N, N)[None]
        d = torch_graph.forward(w, x, "vits")[0].numpy()
        want = oracle.bilinear_align_true(d[None], W, H)[0]
        r = rel(got[k], want)
        print(f"frames {prec} frame {k}: max rel {r:.2e}")
        assert r < (1e-2 if prec == "fp16" else 2e-2)


@pytest.mark.parametrize("fmt", ["bgra", "rgba"])
@pytest.mark.parametrize("kind", ["relative", "metric"])
def test_submit_device_pixels(cuda, dav2lib, tmp_path, vits, fmt, kind):
    """dav2_submit_device_pixels: packed pixels -> bicubic -> graph -> per-image
    min/max normalization at the network size -> align-corners expansion to
    the image size (src/vulkan_executor.cpp:740-786), against the oracle's
    restatement of that sequence on the fp32 forward. Outputs lie in [0, 1]:
    the bound is absolute."""
    _, sd = vits
    metric = 20.0 if kind == "metric" else 0.0
    path = tmp_path / f"vits_{kind}.dav2"
    dav2file.write_dav2(path, sd, "vits", metric_max_depth=metric)
    W, H, size = 300, 200, 140
    px = np.stack([np.random.default_rng(10 + k).integers(0, 256, (H, W, 4), dtype=np.uint8) for k in range(2)])
    rc, ctx = create(dav2lib, path, "vits", capi.FLAGS["fp16"])
    assert rc == 0, dav2lib.dav2_last_error()
    try:
        dpx = torch.from_numpy(px).cuda()
        out = torch.full((2, H, W), -1.0, device="cuda")
        fmt_id = 1 if fmt == "bgra" else 2
        assert dav2lib.dav2_submit_device_pixels(ctx, dpx.data_ptr(), 2, W, H, W * 4, W * H * 4, fmt_id, size,
                                                 out.data_ptr(), None) == 0, dav2lib.dav2_last_error()
        assert dav2lib.dav2_submit_device_pixels(ctx, dpx.data_ptr(), 2, W, H, W * 4, W * H * 4, 3, size,
                                                 out.data_ptr(), None) == 1  # depth pixels are no input format
        got = out.cpu().numpy()
    finally:
        dav2lib.dav2_destroy(ctx)
    nw, nh = oracle.network_shape(W, H, size)
    w = torch_graph.to_torch(sd)
    for k in range(2):
        words = px[k].view(np.uint32).reshape(H, W)
        x = oracle.preprocess_u32_bicubic(words, nw, nh, rgba=(fmt == "rgba"))[None]
        d = torch_graph.forward(w, x, "vits", metric_max_depth=metric)[0].numpy().reshape(-1)
        rng_ = np.array([d.min(), d.max()], np.float32)
        n = oracle.normalize_metric(d, rng_, 25.0) if metric else oracle.normalize_relative(d, rng_)
        want = oracle.bilinear_align_true(n.reshape(1, nh, nw), W, H)[0]
        err = np.abs(got[k] - want).max()
        print(f"submit {fmt} {kind} image {k}: max abs {err:.2e} (range {want.min():.3f}..{want.max():.3f})")
        assert got[k].min() >= 0.0 and got[k].max() <= 1.0
        assert err < 1e-2
