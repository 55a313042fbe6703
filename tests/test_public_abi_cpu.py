"""The public C ABI without a GPU: the reference's tests/c_abi_smoke.c checks,
option validation and model-file errors (all answered before any device
work), and the .dav2 writer/reader round trip."""
import ctypes
import struct

import numpy as np

from abi_helpers import create
from dav2_b200 import capi, dav2file


def test_c_abi_smoke(dav2lib):
    # tests/c_abi_smoke.c:6-50
    lib = dav2lib
    assert lib.dav2_abi_version() == 1
    assert len(lib.dav2_version_string()) > 0
    assert lib.dav2_status_string(0) == b"ok"
    assert lib.dav2_status_string(11) == b"cancelled"
    shape = capi.ImageShape()
    assert lib.dav2_get_network_shape(640, 480, 518, ctypes.byref(shape)) == 0
    assert (shape.width, shape.height) == (686, 518)
    assert lib.dav2_get_network_shape(480, 640, 518, ctypes.byref(shape)) == 0
    assert (shape.width, shape.height) == (518, 686)
    assert lib.dav2_get_network_shape(0, 480, 518, ctypes.byref(shape)) == 1
    assert len(lib.dav2_last_error()) > 0
    info = capi.ModelInfo()
    info.struct_size = ctypes.sizeof(info)
    assert lib.dav2_get_model_info(None, ctypes.byref(info)) == 1
    caps = capi.GpuCapabilities()
    caps.struct_size = ctypes.sizeof(caps)
    assert lib.dav2_probe_gpu_capabilities(0, ctypes.byref(caps)) == 0
    assert caps.abi_version == 1
    caps.struct_size = ctypes.sizeof(caps)
    assert lib.dav2_get_gpu_capabilities(None, ctypes.byref(caps)) == 1
    job = ctypes.c_void_p()
    assert lib.dav2_submit_d3d12_texture(None, None, ctypes.byref(job)) == 1


def test_network_shapes(dav2lib):
    # tests/image_tests.cpp:10-17
    shape = capi.ImageShape()
    for (w, h, s), want in {(640, 480, 518): (686, 518), (480, 640, 518): (518, 686), (518, 518, 518): (518, 518),
                            (1920, 1080, 280): (504, 280)}.items():
        assert dav2lib.dav2_get_network_shape(w, h, s, ctypes.byref(shape)) == 0
        assert (shape.width, shape.height) == want
    assert dav2lib.dav2_get_inferbridge_shape(640, 480, 518, ctypes.byref(shape)) == 0
    assert (shape.width, shape.height) == (518, 686)


def test_network_shapes_vs_reference_native(dav2lib):
    """The shape table of tests/golden/preprocess_ref.npz, made by the
    reference's own compiled network_shape (src/image.cpp), through both
    public entry points; sizes the reference rejects answer INVALID_ARGUMENT."""
    from pathlib import Path

    f = np.load(Path(__file__).resolve().parent / "golden" / "preprocess_ref.npz")
    shape = capi.ImageShape()
    for (w, h, s), rc, (ow, oh) in zip(f["shape_in"].tolist(), f["shape_rc"].tolist(), f["shape_out"].tolist()):
        assert dav2lib.dav2_get_network_shape(w, h, s, ctypes.byref(shape)) == rc
        if rc == 0:
            assert (shape.width, shape.height) == (ow, oh)
        assert dav2lib.dav2_get_inferbridge_shape(w, h, s, ctypes.byref(shape)) == rc
        if rc == 0:
            assert (shape.width, shape.height) == (oh, ow)  # src/dav2.cpp:142-155 swaps the axes


def test_create_validation(dav2lib, tmp_path):
    lib = dav2lib
    ctx = ctypes.c_void_p()
    assert lib.dav2_create(b"x.dav2", None, ctypes.byref(ctx)) == 1
    assert lib.dav2_create(b"", None, ctypes.byref(ctx)) == 1
    assert create(lib, tmp_path / "missing.dav2")[0] == 2  # MODEL_IO
    assert create(lib, tmp_path / "m.dav2", flags=capi.FLAGS["fp16"] | capi.FLAGS["int8"])[0] == 1
    assert create(lib, tmp_path / "m.dav2", flags=1 << 9)[0] == 1
    opts = capi.CreateOptions(ctypes.sizeof(capi.CreateOptions), 2, 0, 0, 0, None)
    assert lib.dav2_create(b"m.dav2", ctypes.byref(opts), ctypes.byref(ctx)) == 1


def test_model_format_errors(dav2lib, tmp_path):
    sd = {"pretrained.cls_token": np.zeros((1, 1, 384), np.float32)}
    good = tmp_path / "tiny.dav2"
    dav2file.write_dav2(good, sd, "vits")
    # wrong encoder -> MODEL_FORMAT, before any device work
    assert create(dav2lib, good, encoder="vitl")[0] == 3
    bad = tmp_path / "bad.dav2"
    data = bytearray(good.read_bytes())
    data[0] = ord("X")
    bad.write_bytes(bytes(data))
    assert create(dav2lib, bad)[0] == 3
    trunc = tmp_path / "trunc.dav2"
    trunc.write_bytes(good.read_bytes()[:100])
    assert create(dav2lib, trunc)[0] == 3


def test_dav2_round_trip(tmp_path):
    sd = dav2file.random_state_dict("vits", seed=3)
    path = tmp_path / "s.dav2"
    size = dav2file.write_dav2(path, sd, "vits", metric_max_depth=20.0)
    assert path.stat().st_size == size
    enc, back = dav2file.read_dav2(path)
    assert enc == 0 and set(back) == set(sd)
    for k in sd:
        assert np.array_equal(back[k], sd[k])
    raw = path.read_bytes()
    assert raw[:8] == b"DAV2MOD\0"
    assert struct.unpack_from("<I", raw, 8)[0] == 1
