"""Full-graph parity through the public C ABI (dav2_create ->
dav2_infer_tensor_f32 / dav2_infer_bgr8 / batched extensions) on the B200.

References:
  * the Python reference model's outputs (tests/golden/*.npz, torch CPU fp32);
  * the oracle's restatement of the same-precision path (oracle.infer_tensor
    with precision "int8": int8 linears/projections/resize layers).
Error measures: max|a-b| / max|b| (the 1e-2 bound) and max|a-b| / (max b -
min b) (sensitivity to the spatial signal, reported alongside).

The int8 graph is chaotic under last-bit changes before a quantization (a
code that flips at a rounding tie moves every later block; the oracle's own
int8 ViT-L output moves by several percent under a 1e-7 perturbation of its
first LayerNorm). So the free-running int8 graph is held to 1e-2 where the
network is well conditioned (ViT-S / ViT-B at the BASELINE init), and
everywhere else the int8 chain is checked teacher-forced: every block and the
head, through the stage probes, on the GPU's own input to that stage, each
within 1e-2 of the oracle's same-precision stage (the free-running distance
is printed)."""
from pathlib import Path

import numpy as np
import pytest

import oracle
from abi_helpers import create, infer_bgr8, infer_tensor, infer_tensor_batch
from dav2_b200 import capi, dav2file

pytestmark = pytest.mark.gpu
G = Path(__file__).resolve().parent / "golden"


def errs(got, ref):
    d = np.abs(got.astype(np.float64) - ref)
    return d.max() / np.abs(ref).max(), d.max() / max(ref.max() - ref.min(), 1e-30)


@pytest.fixture(scope="module")
def models(tmp_path_factory, dav2lib):
    d = tmp_path_factory.mktemp("models")
    out = {}
    for tag, kw in (("base", dict(seed=0)), ("strong", dict(seed=1, std=0.05, bias_std=0.02))):
        sd = dav2file.random_state_dict("vits", **kw)
        path = d / f"vits_{tag}.dav2"
        dav2file.write_dav2(path, sd, "vits")
        out[tag] = (path, sd)
    return out


def context(lib, path, encoder="vits", flags=0):
    rc, ctx = create(lib, path, encoder, flags)
    assert rc == 0, lib.dav2_last_error()
    return ctx


@pytest.mark.parametrize("tag", ["base", "strong"])
@pytest.mark.parametrize("shape", ["70x98", "126x126"])
def test_fp16_vs_reference_python(cuda, dav2lib, models, tag, shape):
    fx = np.load(G / "model_vits.npz")
    ctx = context(dav2lib, models[tag][0], flags=capi.FLAGS["fp16"])
    try:
        got = infer_tensor(dav2lib, ctx, fx[f"{tag}_{shape}_in"])
    finally:
        dav2lib.dav2_destroy(ctx)
    rel, rng_rel = errs(got, fx[f"{tag}_{shape}_out"])
    print(f"fp16 {tag} {shape}: rel {rel:.2e} range-rel {rng_rel:.2e}")
    assert rel < 1e-2


def teacher_forced_int8(lib, ctx, sd, encoder, image, metric_max_depth=0.0):
    """Every int8 stage on the GPU's own input to it, against the oracle's
    same-precision stage: returns (max block error, head error), both max
    relative. Block i is fed the GPU's block i-1 output; the head the GPU's
    tapped residual streams."""
    import ctypes

    _, _, blocks, taps, _, _ = oracle.ENCODERS[encoder]
    _, h, w = image.shape
    x = np.ascontiguousarray(oracle.embed(sd, image, encoder, "int8"), np.float32)
    worst, tapped = 0.0, []
    for i in range(blocks):
        out = np.empty_like(x)
        rc = lib.dav2_probe_encoder_block(ctx, 1, w, h, i, x.ctypes.data, out.ctypes.data, None, None)
        assert rc == 0, lib.dav2_last_error()
        want = oracle.encoder_block(sd, x, i, encoder, "int8")
        worst = max(worst, errs(out, want)[0])
        x = out
        if i in taps:
            tapped.append(x)
    depth = np.empty((h, w), np.float32)
    tap_x = np.ascontiguousarray(np.stack(tapped), np.float32)
    assert lib.dav2_probe_head(ctx, 1, w, h, tap_x.ctypes.data, depth.ctypes.data) == 0, lib.dav2_last_error()
    feats = [oracle.layer_norm(t, sd["pretrained.norm.weight"], sd["pretrained.norm.bias"]) for t in tapped]
    want = oracle.dpt_forward(sd, feats, w // 14, h // 14, encoder, "int8", metric_max_depth)
    return worst, errs(depth, want)[0]


@pytest.mark.parametrize("tag", ["base", "strong"])
def test_int8_vs_oracle_same_precision(cuda, dav2lib, models, tag):
    fx = np.load(G / "model_vits.npz")
    img = fx[f"{tag}_126x126_in"]
    ctx = context(dav2lib, models[tag][0], flags=capi.FLAGS["int8"])
    try:
        got = infer_tensor(dav2lib, ctx, img)
        stages = teacher_forced_int8(dav2lib, ctx, models[tag][1], "vits", img)
    finally:
        dav2lib.dav2_destroy(ctx)
    want = oracle.infer_tensor(models[tag][1], img, "vits", precision="int8")
    rel, rng_rel = errs(got, want)
    print(f"int8 {tag}: free-running rel {rel:.2e} range-rel {rng_rel:.2e}; teacher-forced blocks {stages[0]:.2e} "
          f"head {stages[1]:.2e}")
    assert stages[0] < 1e-2 and stages[1] < 1e-2
    if tag == "base":
        assert rel < 1e-2


def test_infer_bgr8_vs_reference_python(cuda, dav2lib, models):
    fx = np.load(G / "image_vits.npz")
    ctx = context(dav2lib, models["strong"][0], flags=capi.FLAGS["fp16"])
    try:
        got = infer_bgr8(dav2lib, ctx, fx["bgr"], input_size=70)
    finally:
        dav2lib.dav2_destroy(ctx)
    assert got.shape == fx["depth"].shape
    rel, rng_rel = errs(got, fx["depth"])
    print(f"bgr8: rel {rel:.2e} range-rel {rng_rel:.2e}")
    assert rel < 1e-2


@pytest.mark.parametrize("prec", ["fp16", "int8"])
def test_full_size_bgr8_vs_reference_python(cuda, dav2lib, models, prec):
    """The benchmark's full size through the public BGR8 entry point: a 518x518
    BGR8 image (np.random.default_rng(0), the BASELINE CPU configuration's
    image), input size 518 (1370 tokens), ViT-S with random_state_dict(seed=0),
    against the reference's own infer_image (torch fp32, tests/golden). The
    int8 path is held to the same bound: at this init the oracle's int8
    restatement is within 5e-4 of the fp32 reference."""
    fx = np.load(G / "image_vits_518.npz")
    bgr = np.random.default_rng(0).integers(0, 256, (518, 518, 3), dtype=np.uint8)
    ctx = context(dav2lib, models["base"][0], flags=capi.FLAGS[prec])
    try:
        got = infer_bgr8(dav2lib, ctx, bgr, input_size=518)
    finally:
        dav2lib.dav2_destroy(ctx)
    want = fx["depth"].astype(np.float64)
    assert got.shape == want.shape
    rel, rng_rel = errs(got, want)
    print(f"518x518 {prec}: rel {rel:.2e} range-rel {rng_rel:.2e}")
    assert rel < 1e-2


def test_batch_matches_single(cuda, dav2lib, models):
    ctx = context(dav2lib, models["strong"][0], flags=capi.FLAGS["int8"])
    try:
        imgs = np.random.default_rng(4).standard_normal((3, 3, 56, 84)).astype(np.float32)
        batch = infer_tensor_batch(dav2lib, ctx, imgs)
        for i in range(3):
            assert np.array_equal(batch[i], infer_tensor(dav2lib, ctx, imgs[i]))
    finally:
        dav2lib.dav2_destroy(ctx)


@pytest.mark.parametrize("encoder", ["vitb", "vitl"])
def test_larger_encoders_vs_oracle(cuda, dav2lib, tmp_path, encoder):
    sd = dav2file.random_state_dict(encoder, seed=2)  # BASELINE init: N(0, 0.02)
    path = tmp_path / f"{encoder}.dav2"
    dav2file.write_dav2(path, sd, encoder)
    img = np.random.default_rng(5).standard_normal((3, 70, 84)).astype(np.float32)
    got = {}
    for prec in ("fp16", "int8"):
        ctx = context(dav2lib, path, encoder, flags=capi.FLAGS[prec])
        try:
            got[prec] = infer_tensor(dav2lib, ctx, img)
        finally:
            dav2lib.dav2_destroy(ctx)
    fp32 = oracle.infer_tensor(sd, img, encoder, precision="fp32")
    int8 = oracle.infer_tensor(sd, img, encoder, precision="int8")
    rel16, _ = errs(got["fp16"], fp32)
    rel8, rr8 = errs(got["int8"], int8)
    ctx = context(dav2lib, path, encoder, flags=capi.FLAGS["int8"])
    try:
        stages = teacher_forced_int8(dav2lib, ctx, sd, encoder, img)
    finally:
        dav2lib.dav2_destroy(ctx)
    print(f"{encoder}: fp16 vs fp32 {rel16:.2e}; int8 free-running {rel8:.2e} range-rel {rr8:.2e}; teacher-forced "
          f"blocks {stages[0]:.2e} head {stages[1]:.2e}")
    assert rel16 < 1e-2
    assert stages[0] < 1e-2 and stages[1] < 1e-2
    if encoder == "vitb":
        assert rel8 < 1e-2


def test_errors_and_counters(cuda, dav2lib, models):
    import ctypes

    ctx = context(dav2lib, models["base"][0])
    try:
        img = np.zeros((3, 28, 28), np.float32)
        out = np.zeros(28 * 28, np.float32)
        assert dav2lib.dav2_infer_tensor_f32(ctx, img.ctypes.data, 27, 28, out.ctypes.data, out.size) == 1
        assert dav2lib.dav2_infer_tensor_f32(ctx, img.ctypes.data, 28, 28, out.ctypes.data, 10) == 7
        assert dav2lib.dav2_infer_tensor_f32(ctx, img.ctypes.data, 28, 28, out.ctypes.data, out.size) == 0
        c = capi.TransferCounters()
        c.struct_size = ctypes.sizeof(c)
        assert dav2lib.dav2_get_transfer_counters(ctx, ctypes.byref(c)) == 0
        assert c.tensor_upload_bytes >= img.nbytes and c.tensor_download_bytes >= out.nbytes
        info = capi.ModelInfo()
        info.struct_size = ctypes.sizeof(info)
        assert dav2lib.dav2_get_model_info(ctx, ctypes.byref(info)) == 0
        assert info.encoder == 0 and info.is_metric == 0
        job = ctypes.c_void_p()
        req = ctypes.create_string_buffer(256)
        assert dav2lib.dav2_submit_d3d12(ctx, req, ctypes.byref(job)) == 8
    finally:
        dav2lib.dav2_destroy(ctx)


@pytest.fixture(scope="module")
def metric_models(tmp_path_factory, dav2lib):
    d = tmp_path_factory.mktemp("metric")
    out = {}
    for tag, kw in (("base", dict(seed=0)), ("strong", dict(seed=1, std=0.05, bias_std=0.02))):
        sd = dav2file.random_state_dict("vits", **kw)
        path = d / f"vits_metric_{tag}.dav2"
        dav2file.write_dav2(path, sd, "vits", metric_max_depth=20.0)
        out[tag] = (path, sd)
    return out


@pytest.mark.parametrize("tag", ["base", "strong"])
@pytest.mark.parametrize("shape", ["70x98", "126x126"])
def test_metric_fp16_vs_reference_python(cuda, dav2lib, metric_models, tag, shape):
    """A metric-depth .dav2 (is_metric, max depth 20: sigmoid head) through
    dav2_infer_tensor_f32 against the reference's metric model."""
    import ctypes

    fx = np.load(G / "model_vits_metric.npz")
    ctx = context(dav2lib, metric_models[tag][0], flags=capi.FLAGS["fp16"])
    try:
        info = capi.ModelInfo()
        info.struct_size = ctypes.sizeof(info)
        assert dav2lib.dav2_get_model_info(ctx, ctypes.byref(info)) == 0
        assert info.is_metric == 1 and info.metric_max_depth == 20.0
        got = infer_tensor(dav2lib, ctx, fx[f"{tag}_{shape}_in"])
    finally:
        dav2lib.dav2_destroy(ctx)
    ref = fx[f"{tag}_{shape}_out"]
    rel, rng_rel = errs(got, ref)
    print(f"metric fp16 {tag} {shape}: rel {rel:.2e} range-rel {rng_rel:.2e}")
    assert rel < 1e-2
    if tag == "strong":
        assert rng_rel < 1e-2  # measured 1.2e-3


def test_metric_int8_vs_oracle_same_precision(cuda, dav2lib, metric_models):
    fx = np.load(G / "model_vits_metric.npz")
    img = fx["strong_126x126_in"]
    ctx = context(dav2lib, metric_models["strong"][0], flags=capi.FLAGS["int8"])
    try:
        got = infer_tensor(dav2lib, ctx, img)
    finally:
        dav2lib.dav2_destroy(ctx)
    want = oracle.infer_tensor(metric_models["strong"][1], img, "vits", precision="int8", metric_max_depth=20.0)
    rel, rng_rel = errs(got, want)
    ctx = context(dav2lib, metric_models["strong"][0], flags=capi.FLAGS["int8"])
    try:
        stages = teacher_forced_int8(dav2lib, ctx, metric_models["strong"][1], "vits", img, metric_max_depth=20.0)
    finally:
        dav2lib.dav2_destroy(ctx)
    print(f"metric int8: free-running rel {rel:.2e} range-rel {rng_rel:.2e}; teacher-forced blocks {stages[0]:.2e} "
          f"head {stages[1]:.2e}")
    assert rel < 1e-2
    assert stages[0] < 1e-2 and stages[1] < 1e-2


@pytest.mark.parametrize("kind", ["relative", "metric"])
@pytest.mark.parametrize("case", [0, 1, 3])
def test_inferbridge_bgra8_vs_oracle(cuda, dav2lib, models, metric_models, kind, case):
    """dav2_inferbridge_bgra8_f32 (src/dav2.cpp:754-803) on the padded-stride
    BGRA8 sources of tests/golden/preprocess_ref.npz: the preprocessed tensor
    is pinned to the reference's compiled code there; here the whole call
    (nearest resize to the transposed shape, graph, host min/max normalization)
    is compared with the oracle's fp32 restatement. The output lies in [0, 1];
    the bound is absolute."""
    import ctypes

    f = np.load(G / "preprocess_ref.npz")
    w, h, stride, dw, dh = f[f"bgra{case}_meta"].tolist()
    src = np.ascontiguousarray(f[f"bgra{case}_src"])
    size = {0: 70, 1: 140, 3: 70}[case]
    path, sd = (models if kind == "relative" else metric_models)["strong"]
    ctx = context(dav2lib, path, flags=capi.FLAGS["fp16"])
    try:
        out = np.full(dw * dh, -1.0, np.float32)
        assert dav2lib.dav2_inferbridge_bgra8_f32(ctx, src.ctypes.data, w, h, stride, size, out.ctypes.data,
                                                  out.size - 1) == 7  # BUFFER_TOO_SMALL
        assert dav2lib.dav2_inferbridge_bgra8_f32(ctx, src.ctypes.data, w, h, w * 4 - 1, size, out.ctypes.data,
                                                  out.size) == 1  # stride below width * 4
        assert dav2lib.dav2_inferbridge_bgra8_f32(ctx, None, w, h, stride, size, out.ctypes.data, out.size) == 1
        rc = dav2lib.dav2_inferbridge_bgra8_f32(ctx, src.ctypes.data, w, h, stride, size, out.ctypes.data, out.size)
        assert rc == 0, dav2lib.dav2_last_error()
    finally:
        dav2lib.dav2_destroy(ctx)
    metric = 20.0 if kind == "metric" else 0.0
    tensor = f[f"bgra{case}_out"]
    depth = oracle.infer_tensor(sd, tensor, "vits", metric_max_depth=metric)
    lo = np.float32(depth.min())
    span = (np.float32(25.0) if metric else np.float32(depth.max())) - lo
    want = ((depth - lo) / span).reshape(-1)
    bgra = src[:, :w * 4].reshape(h, w, 4)
    assert np.array_equal(oracle.inferbridge_bgra8(sd, bgra, "vits", size, metric_max_depth=metric).reshape(-1), want)
    err = np.abs(out - want).max()
    print(f"inferbridge {kind} case {case} ({dw}x{dh}): max abs {err:.2e} (output range {want.min():.3f}..{want.max():.3f})")
    assert out.min() >= 0.0 and (metric or out.max() == 1.0)
    assert err < (1e-2 if kind == "relative" else 1e-3)  # measured 2.0e-3 / 1.4e-4


@pytest.mark.parametrize("prec", ["fp16", "int8"])
def test_batch_matches_single_images(cuda, dav2lib, models, prec):
    """Six 518x518 images in one batched call (8220 token rows) against the
    same images one at a time: every operator of the graph is row- or
    image-independent, so batching must not change a single value."""
    imgs = np.random.default_rng(5).standard_normal((6, 3, 518, 518)).astype(np.float32)
    ctx = context(dav2lib, models["strong"][0], flags=capi.FLAGS[prec])
    try:
        batched = infer_tensor_batch(dav2lib, ctx, imgs)
        single = np.stack([infer_tensor(dav2lib, ctx, im) for im in imgs])
    finally:
        dav2lib.dav2_destroy(ctx)
    rel, rng_rel = errs(batched, single.astype(np.float64))
    print(f"batch vs single ({prec}): rel {rel:.2e} range-rel {rng_rel:.2e}")
    assert rel < 1e-5

