"""The benchmark's own entry points, dav2_infer_device_bgr8_batch (device
buffers, caller stream) and dav2_infer_bgr8_batch (host buffers), on padded
row and image strides: every image must be bit-identical to the same image
through the single-image public entry point dav2_infer_bgr8, and image 0
(np.random.default_rng(0), 518x518) within 1e-2 of the reference's own
infer_image output (tests/golden/image_vits_518.npz, ViT-S seed 0, fp32).
A source size that is not the network size exercises the resize branch
that writes straight into the caller's buffer."""
import ctypes
from pathlib import Path

import numpy as np
import pytest

from abi_helpers import create
from dav2_b200 import capi, dav2file

pytestmark = pytest.mark.gpu
G = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def vits0(tmp_path_factory, dav2lib):
    path = tmp_path_factory.mktemp("entry") / "vits0.dav2"
    dav2file.write_dav2(path, dav2file.random_state_dict("vits", seed=0), "vits")
    return path


def padded_batch(imgs, row_pad=64, image_pad=4096):
    b, h, w, _ = imgs.shape
    row = w * 3 + row_pad
    image = row * h + image_pad
    buf = np.zeros(b * image, np.uint8)
    for i in range(b):
        v = buf[i * image:i * image + row * h].reshape(h, row)
        v[:, :w * 3] = imgs[i].reshape(h, w * 3)
    return buf, row, image


@pytest.mark.parametrize("prec", ["fp16", "int8"])
@pytest.mark.parametrize("size", [(518, 518), (640, 428)])
def test_batched_entry_points_match_single_image(cuda, dav2lib, vits0, prec, size):
    torch = cuda
    w, h = size
    imgs = np.stack([np.random.default_rng(s).integers(0, 256, (h, w, 3), dtype=np.uint8) for s in range(4)])
    buf, row, image = padded_batch(imgs)
    rc, ctx = create(dav2lib, vits0, "vits", capi.FLAGS[prec])
    assert rc == 0, dav2lib.dav2_last_error()
    try:
        single = np.zeros((4, h, w), np.float32)
        for i in range(4):
            one = np.ascontiguousarray(imgs[i])
            assert dav2lib.dav2_infer_bgr8(ctx, one.ctypes.data, w, h, w * 3, 518, single[i].ctypes.data,
                                           w * h) == 0, dav2lib.dav2_last_error()
        host = np.zeros((4, h, w), np.float32)
        assert dav2lib.dav2_infer_bgr8_batch(ctx, buf.ctypes.data, 4, w, h, row, image, 518, host.ctypes.data,
                                             host.size) == 0, dav2lib.dav2_last_error()
        dbuf = torch.from_numpy(buf).cuda()
        dout = torch.full((4, h, w), -1.0, dtype=torch.float32, device="cuda")
        s = torch.cuda.Stream()
        assert dav2lib.dav2_infer_device_bgr8_batch(ctx, dbuf.data_ptr(), 4, w, h, row, image, 518,
                                                    dout.data_ptr(), ctypes.c_void_p(s.cuda_stream)) == 0
        assert dav2lib.dav2_synchronize(ctx) == 0, dav2lib.dav2_last_error()
        dev = dout.cpu().numpy()
        # the context's own stream (NULL): synchronous
        dout2 = torch.full((4, h, w), -1.0, dtype=torch.float32, device="cuda")
        assert dav2lib.dav2_infer_device_bgr8_batch(ctx, dbuf.data_ptr(), 4, w, h, row, image, 518,
                                                    dout2.data_ptr(), None) == 0
        dev2 = dout2.cpu().numpy()
    finally:
        dav2lib.dav2_destroy(ctx)
    for name, got in (("host batch", host), ("device batch", dev), ("device batch, context stream", dev2)):
        assert np.array_equal(got, single), f"{name} differs from single-image calls"
    if size == (518, 518):
        want = np.load(G / "image_vits_518.npz")["depth"].astype(np.float64)
        r = np.abs(single[0] - want).max() / np.abs(want).max()
        print(f"{prec} 518: image 0 vs the reference's infer_image: max rel {r:.2e}")
        assert r < 1e-2
