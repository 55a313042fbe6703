"""ViT-L parity at the benchmark's size (518x518, 1370 tokens): the encoder
and weights of BASELINE configuration 4 (random_state_dict("vitl", seed=0),
N(0, 0.02)), checked stage by stage against the oracle's same-precision
restatement, and the fp16 full graph against the fp32 reference forward
(the final bias is zeroed so that the depth map is not identically zero; see
the `vitl` fixture).

A full int8 graph cannot be compared end to end at 1e-2: a code that flips
at a rounding tie (LayerNorm or attention reduction order) moves every later
block, and 24 such blocks amplify it (the oracle's own int8 output moves by
several percent under a 1e-7 perturbation of its first LayerNorm). So the
int8 chain is pinned stage by stage, each stage fed the same input on both
sides:
  * blocks 0, 11 and 23 (batch 2) through dav2_probe_encoder_block, fed the
    residual stream that the GPU's own preceding blocks produced: the first
    LayerNorm's int8 codes must equal the oracle's except at rounding ties
    (|x/scale - (k + 1/2)| < 1e-3; their count is printed and bounded), and
    the block output must be within 1e-2 (max relative) of the oracle's;
  * the DPT head (tap LayerNorms, int8 projections / resize layers, f16
    refinement) through dav2_probe_head from the GPU's tapped residual
    streams, within 1e-2 of the oracle's int8 head.
"""
import numpy as np
import pytest

import oracle
import torch_graph
from abi_helpers import create
from dav2_b200 import capi, dav2file

pytestmark = pytest.mark.gpu
S, T, D = 518, 1370, 1024
TAPS = (4, 11, 17, 23)


@pytest.fixture(scope="module")
def vitl(tmp_path_factory, dav2lib):
    """BASELINE configuration 4's weights with one change: the last
    convolution's bias (depth_head.scratch.output_conv2.2.bias, -0.029 in
    this draw) is set to 0. With the drawn bias the ReLU'd depth of every
    pixel is 0 for any image — a degenerate output that no comparison can
    check — while with 0 about 43% of the pixels are positive. Nothing else
    changes, so every kernel does the benchmark's work."""
    sd = dav2file.random_state_dict("vitl", seed=0)
    sd["depth_head.scratch.output_conv2.2.bias"] = np.zeros_like(sd["depth_head.scratch.output_conv2.2.bias"])
    path = tmp_path_factory.mktemp("vitl") / "vitl_seed0.dav2"
    dav2file.write_dav2(path, sd, "vitl")
    return path, sd


@pytest.fixture(scope="module")
def int8_ctx(vitl, dav2lib):
    rc, ctx = create(dav2lib, vitl[0], "vitl", capi.FLAGS["int8"])
    assert rc == 0, dav2lib.dav2_last_error()
    yield ctx
    dav2lib.dav2_destroy(ctx)


def rel(got, want):
    return float(np.abs(got.astype(np.float64) - want).max() / np.abs(want).max())


def probe_block(lib, ctx, batch, block, x, codes=False):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    c = np.empty(x.shape, np.int8) if codes else None
    s = np.empty(x.shape[0], np.float32) if codes else None
    rc = lib.dav2_probe_encoder_block(ctx, batch, S, S, block, x.ctypes.data, out.ctypes.data,
                                      None if c is None else c.ctypes.data, None if s is None else s.ctypes.data)
    assert rc == 0, lib.dav2_last_error()
    return out, c, s


@pytest.fixture(scope="module")
def gpu_stream(int8_ctx, vitl, dav2lib):
    """Residual rows entering every block for two 518x518 BGR8 images
    (np.random.default_rng(0) and (1), the BASELINE image rule): block 0's
    input is the oracle's int8 embedding of the oracle-preprocessed images;
    block i+1's input is the GPU's block-i output."""
    sd = vitl[1]
    xs = []
    for seed in (0, 1):
        bgr = np.random.default_rng(seed).integers(0, 256, (S, S, 3), dtype=np.uint8)
        xs.append(oracle.embed(sd, oracle.preprocess_bgr8(bgr, S, S), "vitl", "int8"))
    x = np.concatenate(xs)
    stream = [x]
    for i in range(24):
        x, _, _ = probe_block(dav2lib, int8_ctx, 2, i, x)
        stream.append(x)
    return stream


@pytest.mark.parametrize("block", [0, 11, 23])
def test_int8_block_vs_oracle(cuda, dav2lib, int8_ctx, vitl, gpu_stream, block):
    sd = vitl[1]
    xin = gpu_stream[block]
    got, codes, scales = probe_block(dav2lib, int8_ctx, 2, block, xin, codes=True)
    n, px, sx = oracle.ln1_codes(sd, xin, block)
    want_codes = px.view(np.int8).reshape(n.shape)
    assert np.abs(scales.astype(np.float64) - sx).max() <= 1e-6 * np.abs(sx).max()
    flips = np.argwhere(codes != want_codes)
    t = n[flips[:, 0], flips[:, 1]] / sx[flips[:, 0]] if len(flips) else np.zeros(0)
    tie = np.abs(np.abs(t - np.floor(t)) - 0.5) if len(flips) else np.zeros(0)
    print(f"block {block}: LN1 code flips {len(flips)} of {codes.size} (all within {tie.max() if len(tie) else 0:.1e} "
          f"of a tie)")
    assert len(flips) <= codes.size * 1e-5
    assert (tie < 1e-3).all(), "a code differs away from a rounding tie"
    assert (np.abs(codes.astype(np.int32) - want_codes) <= 1).all()
    want = oracle.encoder_block(sd, xin, block, "vitl", "int8", tokens=T)
    r = rel(got, want)
    print(f"block {block}: output max rel {r:.2e} (max |x| {np.abs(want).max():.1f})")
    assert r < 1e-2


def test_int8_head_vs_oracle(cuda, dav2lib, int8_ctx, vitl, gpu_stream):
    """Image 0 of the stream: its four tapped residual streams (the GPU's block
    outputs 4, 11, 17, 23) through the GPU head and the oracle's int8 head."""
    sd = vitl[1]
    taps = [gpu_stream[i + 1][:T] for i in TAPS]
    depth = np.empty((S, S), np.float32)
    tap_x = np.ascontiguousarray(np.stack(taps), np.float32)
    rc = dav2lib.dav2_probe_head(int8_ctx, 1, S, S, tap_x.ctypes.data, depth.ctypes.data)
    assert rc == 0, dav2lib.dav2_last_error()
    feats = [oracle.layer_norm(x, sd["pretrained.norm.weight"], sd["pretrained.norm.bias"]) for x in taps]
    want = oracle.dpt_forward(sd, feats, S // 14, S // 14, "vitl", "int8")
    r = rel(depth, want)
    print(f"head: depth max rel {r:.2e} (positive pixels {np.mean(want > 0):.2f}, max {want.max():.2e})")
    assert want.max() > 0 and np.mean(want > 0) > 0.1  # a non-degenerate depth map
    assert r < 1e-2


def test_fp16_full_graph_vs_fp32_reference_forward(cuda, dav2lib, vitl):
    """The fp16 path end to end through dav2_infer_bgr8 at 518x518 against
    the fp32 reference forward (oracle/torch_graph.py, pinned to the
    reference model's own fixtures) on the same BGR8 image."""
    import torch

    path, sd = vitl
    bgr = np.random.default_rng(0).integers(0, 256, (S, S, 3), dtype=np.uint8)
    rc, ctx = create(dav2lib, path, "vitl", capi.FLAGS["fp16"])
    assert rc == 0, dav2lib.dav2_last_error()
    try:
        got = np.zeros((S, S), np.float32)
        assert dav2lib.dav2_infer_bgr8(ctx, bgr.ctypes.data, S, S, S * 3, S, got.ctypes.data, got.size) == 0, \
            dav2lib.dav2_last_error()
    finally:
        dav2lib.dav2_destroy(ctx)
    torch.set_num_threads(max(1, torch.get_num_threads()))
    x = oracle.preprocess_bgr8(bgr, S, S)[None]
    want = torch_graph.forward(torch_graph.to_torch(sd), x, "vitl")[0].numpy()
    r = rel(got, want)
    print(f"vitl fp16 518: max rel {r:.2e} vs fp32 (positive pixels {np.mean(want > 0):.2f})")
    assert want.max() > 0 and np.mean(want > 0) > 0.1
    assert r < 1e-2
