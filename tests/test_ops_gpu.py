"""Operator parity on the B200: each dav2cuda_* entry point (called through
the C ABI) against the CPU oracle on the same seeded inputs.

Tolerances: int8 codes, scales and im2col indexing bit-exact; int8 GEMMs
bit-exact (integer accumulation, dequant rounded in the oracle's order);
fp32 operators 1e-4 max relative error; tensor-core ops with half operands
(attention, *_half) against the fp32 oracle at the half-precision bound
stated per test.
"""
import numpy as np
import pytest

import oracle
from conftest import max_rel
from devbuf import call, dev, empty, finish, host, ptr

pytestmark = pytest.mark.gpu


def rng(seed=0):
    return np.random.default_rng(seed)


# ---------------------------------------------------------------- row ops
@pytest.mark.parametrize("rows,cols", [(4, 17), (37, 384), (129, 768), (300, 1024), (5, 1000),
                                       (8200, 1024), (9001, 768), (10960, 1024), (1, 1024), (7, 1024),
                                       (301, 1024)])
def test_layer_norm(cuda, dav2lib, rows, cols):
    """Row counts from a handful to above the ViT-S batch-6 token count, and
    BASELINE configuration 2's [10960, 1024]; odd row counts at ViT-L's width."""
    r = rng(rows)
    x = r.standard_normal((rows, cols)).astype(np.float32) * 3 + 0.5
    w = r.standard_normal(cols).astype(np.float32)
    b = r.standard_normal(cols).astype(np.float32)
    want = oracle.layer_norm(x, w, b, 1e-6)
    dx, dw, db, out = dev(cuda, x), dev(cuda, w), dev(cuda, b), empty(cuda, (rows, cols))
    call(dav2lib, "dav2cuda_layer_norm", ptr(out), ptr(dx), ptr(dw), ptr(db), rows, cols, 1e-6, None)
    finish(cuda, dav2lib)
    assert max_rel(host(out), want) < 1e-4


def test_layer_norm_reference_kat(cuda, dav2lib):
    # tests/vulkan_smoke.cpp:436-494: (i%23-10)*0.125, 4x17, gamma 1, beta 0, +-1e-5
    x = ((np.arange(4 * 17) % 23) - 10).astype(np.float32).reshape(4, 17) * 0.125
    w, b = np.ones(17, np.float32), np.zeros(17, np.float32)
    out = empty(cuda, (4, 17))
    call(dav2lib, "dav2cuda_layer_norm", ptr(out), ptr(dev(cuda, x)), ptr(dev(cuda, w)), ptr(dev(cuda, b)), 4, 17,
         1e-6, None)
    finish(cuda, dav2lib)
    mean = x.mean(1, keepdims=True)
    var = np.maximum((x * x).mean(1, keepdims=True) - mean * mean, 0)
    assert np.abs(host(out) - (x - mean) / np.sqrt(var + 1e-6)).max() <= 1e-5


@pytest.mark.parametrize("n", [1, 7, 4096, 10960 * 4, 10960 * 4096])  # the last: configuration 2's shape
def test_gelu(cuda, dav2lib, n):
    x = rng(n).standard_normal(n).astype(np.float32) * 4
    out = empty(cuda, (n,))
    call(dav2lib, "dav2cuda_gelu", ptr(out), ptr(dev(cuda, x)), n, None)
    finish(cuda, dav2lib)
    want = oracle.gelu(x)
    assert np.abs(host(out) - want).max() <= 1e-4 * max(1.0, np.abs(want).max())


@pytest.mark.parametrize("rows,cols,scale", [(16, 1370, 0.125), (8, 5, 1.0), (3, 3001, 1.0), (2, 4000, 0.125),
                                              (5, 7, 0.5),
                                              (8 * 16 * 1370, 1370, 0.125)])  # configuration 2's [8,16,1370,1370]
def test_softmax(cuda, dav2lib, rows, cols, scale):
    x = rng(cols).standard_normal((rows, cols)).astype(np.float32) * 4
    out = empty(cuda, (rows, cols))
    call(dav2lib, "dav2cuda_softmax_rows", ptr(out), ptr(dev(cuda, x)), rows, cols, scale, None)
    finish(cuda, dav2lib)
    assert max_rel(host(out), oracle.softmax_rows(x, scale)) < 1e-4


def test_add_scaled_exact(cuda, dav2lib):
    # tests/vulkan_smoke.cpp:496-538: exact (precise) result
    res = np.arange(15, dtype=np.float32) * 0.125
    add = (np.arange(15, dtype=np.float32) + 2) * -0.0625
    sc = (np.arange(5, dtype=np.float32) + 1) * 0.25
    out = empty(cuda, (15,))
    call(dav2lib, "dav2cuda_add_scaled", ptr(out), ptr(dev(cuda, res)), ptr(dev(cuda, add)), ptr(dev(cuda, sc)), 15, 5,
         None)
    finish(cuda, dav2lib)
    assert np.array_equal(host(out), oracle.add_scaled(res, add, sc))
    r = rng(3)
    res = r.standard_normal(1024 * 33).astype(np.float32)
    add = r.standard_normal(1024 * 33).astype(np.float32)
    sc = r.standard_normal(1024).astype(np.float32)
    out = empty(cuda, res.shape)
    call(dav2lib, "dav2cuda_add_scaled", ptr(out), ptr(dev(cuda, res)), ptr(dev(cuda, add)), ptr(dev(cuda, sc)),
         res.size, 1024, None)
    finish(cuda, dav2lib)
    assert np.array_equal(host(out), oracle.add_scaled(res, add, sc))


def test_elementwise(cuda, dav2lib):
    x = rng(4).standard_normal(1001).astype(np.float32)
    y = rng(5).standard_normal(1001).astype(np.float32)
    out = empty(cuda, x.shape)
    call(dav2lib, "dav2cuda_relu", ptr(out), ptr(dev(cuda, x)), x.size, None)
    finish(cuda, dav2lib)
    assert np.array_equal(host(out), oracle.relu(x))
    call(dav2lib, "dav2cuda_add", ptr(out), ptr(dev(cuda, x)), ptr(dev(cuda, y)), x.size, None)
    finish(cuda, dav2lib)
    assert np.array_equal(host(out), oracle.add(x, y))
    call(dav2lib, "dav2cuda_sigmoid_scale", ptr(out), ptr(dev(cuda, x)), x.size, 20.0, None)
    finish(cuda, dav2lib)
    assert max_rel(host(out), oracle.sigmoid_scale(x, 20.0)) < 1e-6


# ------------------------------------------------------------- resampling
@pytest.mark.parametrize("c,ih,iw,oh,ow", [(3, 19, 23, 37, 45), (2, 37, 37, 74, 74), (1, 5, 7, 5, 7),
                                           (4, 1, 9, 3, 17), (1, 518, 518, 1080, 1920)])
def test_bilinear_align_true(cuda, dav2lib, c, ih, iw, oh, ow):
    x = rng(ih * iw).standard_normal((c, ih, iw)).astype(np.float32)
    out = empty(cuda, (c, oh, ow))
    call(dav2lib, "dav2cuda_bilinear_align_true", ptr(out), ptr(dev(cuda, x)), iw, ih, ow, oh, c, None)
    finish(cuda, dav2lib)
    want = oracle.bilinear_align_true(x, ow, oh)
    assert np.array_equal(host(out), want)


@pytest.mark.parametrize("bf16", [0, 1])
@pytest.mark.parametrize("b,c,ih,iw,oh,ow", [(2, 256, 37, 37, 74, 74),   # fusion resize (ViT-L, 37 -> 74)
                                             (1, 128, 74, 74, 148, 148),
                                             (3, 64, 19, 21, 37, 45),
                                             (1, 8, 1, 5, 3, 9),           # one source row
                                             (1, 2048, 3, 3, 7, 5)])       # widest channel count
def test_bilinear_nhwc_16_bit_exact(cuda, dav2lib, bf16, b, c, ih, iw, oh, ow):
    """The graph's channels-last 16-bit resize against the oracle's f32
    align-corners bilinear of the same 16-bit inputs, rounded to the 16-bit
    type: bit-exact."""
    torch = cuda
    dt = torch.bfloat16 if bf16 else torch.float16
    x = torch.from_numpy(rng(c + ih).standard_normal((b, ih, iw, c)).astype(np.float32)).to(dt)
    xd, out = x.cuda(), torch.empty((b, oh, ow, c), dtype=dt, device="cuda")
    call(dav2lib, "dav2cuda_bilinear_align_nhwc_16", out.data_ptr(), xd.data_ptr(), b, iw, ih, ow, oh, c, bf16, None)
    finish(cuda, dav2lib)
    xf = x.float().numpy()
    for i in range(b):
        want = oracle.bilinear_align_true(np.ascontiguousarray(xf[i].transpose(2, 0, 1)), ow, oh)
        want16 = torch.from_numpy(np.ascontiguousarray(want.transpose(1, 2, 0))).to(dt)
        assert torch.equal(out[i].cpu().view(torch.int16), want16.view(torch.int16))


def test_minmax_normalize_kat(cuda, dav2lib):
    # tests/vulkan_smoke.cpp:121-142: {2,3,5,10} -> {0,.125,.375,1} +-1e-6
    d = dev(cuda, np.array([2, 3, 5, 10], np.float32))
    rg = empty(cuda, (2,))
    call(dav2lib, "dav2cuda_reduce_minmax", ptr(d), ptr(rg), 4, None)
    call(dav2lib, "dav2cuda_normalize_relative", ptr(d), ptr(rg), 4, None)
    finish(cuda, dav2lib)
    assert np.abs(host(d) - [0, 0.125, 0.375, 1]).max() <= 1e-6


@pytest.mark.parametrize("n", [1, 255, 268324, 1920 * 1080])
def test_minmax_normalize(cuda, dav2lib, n):
    x = rng(n).standard_normal(n).astype(np.float32) * 5 + 2
    d, rg = dev(cuda, x), empty(cuda, (2,))
    call(dav2lib, "dav2cuda_reduce_minmax", ptr(d), ptr(rg), n, None)
    finish(cuda, dav2lib)
    want_rg = oracle.reduce_minmax(x)
    assert np.array_equal(host(rg), want_rg)
    call(dav2lib, "dav2cuda_normalize_relative", ptr(d), ptr(rg), n, None)
    finish(cuda, dav2lib)
    assert np.abs(host(d) - oracle.normalize_relative(x, want_rg)).max() <= 1e-6
    d = dev(cuda, x)
    call(dav2lib, "dav2cuda_normalize_metric", ptr(d), ptr(rg), n, 20.0, None)
    finish(cuda, dav2lib)
    assert np.abs(host(d) - oracle.normalize_metric(x, want_rg, 20.0)).max() <= 1e-6


@pytest.mark.parametrize("sw,sh,dw,dh,rgba", [(73, 51, 98, 70, 0), (640, 480, 686, 518, 1), (37, 53, 14, 28, 0)])
def test_preprocess_u32(cuda, dav2lib, sw, sh, dw, dh, rgba):
    px = rng(sw).integers(0, 2**32, (sh, sw), dtype=np.uint64).astype(np.uint32)
    out = empty(cuda, (3, dh, dw))
    call(dav2lib, "dav2cuda_preprocess_u32", ptr(out), ptr(dev(cuda, px.view(np.int32))), sw, sh, sw, rgba, dw, dh,
         None)
    finish(cuda, dav2lib)
    assert max_rel(host(out), oracle.preprocess_u32_bicubic(px, dw, dh, bool(rgba))) < 1e-5


@pytest.mark.parametrize("sw,sh,dw,dh", [(53, 37, 98, 70), (518, 518, 518, 518), (640, 480, 686, 518),
                                         (1920, 1080, 504, 280)])
def test_preprocess_bgr8(cuda, dav2lib, sw, sh, dw, dh):
    bgr = rng(sw + sh).integers(0, 256, (2, sh, sw, 3), dtype=np.uint8)
    out = empty(cuda, (2, 3, dh, dw))
    call(dav2lib, "dav2cuda_preprocess_bgr8", ptr(out), ptr(dev(cuda, bgr)), 2, sw, sh, sw * 3, sw * sh * 3, dw, dh,
         None)
    finish(cuda, dav2lib)
    got = host(out)
    for i in range(2):
        want = oracle.preprocess_bgr8(bgr[i], dw, dh)
        assert np.abs(got[i] - want).max() <= 1e-4 * np.abs(want).max()


@pytest.mark.parametrize("case", range(5))
def test_preprocess_bgr8_vs_reference_native(cuda, dav2lib, case):
    """The device preprocess_bgr8 against the reference's own compiled
    src/image.cpp (tests/golden/preprocess_ref.npz: padded row strides,
    upscaling, a one-pixel-wide source)."""
    from pathlib import Path

    f = np.load(Path(__file__).resolve().parent / "golden" / "preprocess_ref.npz")
    w, h, stride, dw, dh = f[f"bgr{case}_meta"].tolist()
    src = np.ascontiguousarray(f[f"bgr{case}_src"])
    want = f[f"bgr{case}_out"]
    out = empty(cuda, (1, 3, dh, dw))
    call(dav2lib, "dav2cuda_preprocess_bgr8", ptr(out), ptr(dev(cuda, src)), 1, w, h, stride, stride * h, dw, dh,
         None)
    finish(cuda, dav2lib)
    assert np.abs(host(out)[0] - want).max() <= 1e-4 * np.abs(want).max()


def test_preprocess_bgr8_bilinear(cuda, dav2lib):
    bgr = rng(9).integers(0, 256, (2, 108, 192, 3), dtype=np.uint8)
    out = empty(cuda, (2, 3, 98, 98))
    call(dav2lib, "dav2cuda_preprocess_bgr8_bilinear", ptr(out), ptr(dev(cuda, bgr)), 2, 192, 108, 192 * 3,
         192 * 108 * 3, 98, 98, None)
    finish(cuda, dav2lib)
    for i in range(2):
        want = oracle.preprocess_bgr8_bilinear(bgr[i], 98, 98)
        assert np.abs(host(out)[i] - want).max() <= 1e-4 * np.abs(want).max()


# ------------------------------------------------------------------ int8
@pytest.mark.parametrize("rows,cols,offset", [(1369, 384, 384), (5, 4, 0), (300, 4096, 0), (7, 1028, 8),
                                             (8221, 1024, 0), (2741, 4096, 0), (513, 768, 0), (1370, 2048, 0)])
def test_quantize_rows_bit_exact(cuda, dav2lib, rows, cols, offset):
    """Generic, warp-per-row (<= 2048 columns) and register-resident (4096)
    f32 quantizers — the latter two are the graph's attention-output and
    GELU-hidden quantizers."""
    x = rng(cols).standard_normal(rows * cols + offset).astype(np.float32)
    x[offset + 3 * cols: offset + 4 * cols] = 0 if rows > 3 else x[offset + 3 * cols: offset + 4 * cols]  # zero row
    pk, sc = empty(cuda, (rows, cols // 4), np.uint32), empty(cuda, (rows,))
    call(dav2lib, "dav2cuda_quantize_rows_s8", ptr(pk), ptr(sc), ptr(dev(cuda, x)), rows, cols, offset, None)
    finish(cuda, dav2lib)
    want_pk, want_sc = oracle.quantize_rows_s8(x, rows, cols, offset)
    assert np.array_equal(host(sc), want_sc)
    assert np.array_equal(host(pk, np.uint32), want_pk)


@pytest.mark.parametrize("c,h,w,k,s,p", [(4, 4, 5, 3, 1, 1), (3, 28, 42, 14, 14, 0), (256, 19, 23, 3, 1, 1),
                                         (5, 9, 11, 3, 2, 1), (32, 6, 6, 1, 1, 0)])
def test_im2col_quantize_bit_exact(cuda, dav2lib, c, h, w, k, s, p):
    x = rng(c * h).standard_normal((c, h, w)).astype(np.float32)
    ow, oh = (w + 2 * p - k) // s + 1, (h + 2 * p - k) // s + 1
    words = (c * k * k + 3) // 4
    pk, sc = empty(cuda, (ow * oh, words), np.uint32), empty(cuda, (ow * oh,))
    call(dav2lib, "dav2cuda_im2col_quantize_s8", ptr(pk), ptr(sc), ptr(dev(cuda, x)), w, h, c, ow, oh, k, s, p, None)
    finish(cuda, dav2lib)
    want_pk, want_sc = oracle.im2col_quantize_s8(x, k, s, p)
    assert np.array_equal(host(sc), want_sc)
    assert np.array_equal(host(pk, np.uint32), want_pk)


@pytest.mark.parametrize("b,c,h,w,k,s,p", [(2, 64, 9, 7, 3, 2, 1), (1, 1024, 37, 37, 3, 2, 1), (2, 12, 5, 6, 3, 1, 1),
                                           (3, 256, 37, 37, 1, 1, 0), (1, 8, 1, 1, 3, 1, 1)])
def test_im2col_quantize_nhwc_bit_exact(cuda, dav2lib, b, c, h, w, k, s, p):
    """The graph's channels-last im2col-quantize (ViT-L's resize-3 convolution:
    1024 channels 3x3 stride 2 on 37x37; the conv-transpose inputs: 1x1 rows;
    a channel count off the 8-channel vector path; a one-pixel map) against the
    oracle's planar im2col of each image: equal row scales, and equal codes once
    the reference's (c, ky, kx) columns are put in (ky, kx, c) order; the row
    padding is zero."""
    x = rng(b * c + h).standard_normal((b, c, h, w)).astype(np.float32)
    ow, oh = (w + 2 * p - k) // s + 1, (h + 2 * p - k) // s + 1
    cols = c * k * k
    row_bytes = (cols + 15) // 16 * 16
    codes, sc = empty(cuda, (b * oh * ow, row_bytes), np.uint8), empty(cuda, (b * oh * ow,))
    nhwc = np.ascontiguousarray(x.transpose(0, 2, 3, 1))
    call(dav2lib, "dav2cuda_im2col_quantize_nhwc", ptr(codes), ptr(sc), ptr(dev(cuda, nhwc)), b, h, w, c, k, s, p,
         row_bytes, None)
    finish(cuda, dav2lib)
    got = host(codes, np.uint8).reshape(b, oh * ow, row_bytes)
    got_sc = host(sc).reshape(b, oh * ow)
    for i in range(b):
        want_pk, want_sc = oracle.im2col_quantize_s8(x[i], k, s, p)
        want = want_pk.view(np.uint8)[:, :cols].reshape(oh * ow, c, k, k).transpose(0, 2, 3, 1).reshape(oh * ow, cols)
        assert np.array_equal(got_sc[i], want_sc)
        assert np.array_equal(got[i, :, :cols], want)
        assert not got[i, :, cols:].any()


def _s8_problem(seed, rows, k, n):
    r = rng(seed)
    x = r.standard_normal((rows, k)).astype(np.float32)
    w = (r.standard_normal((n, k)) * 0.02).astype(np.float32)
    b = r.standard_normal(n).astype(np.float32) * 0.1
    px, sx = oracle.quantize_rows_s8(x, rows, k)
    pw, sw = oracle.pack_weight_s8(w)
    return x, w, b, px, sx, pw, sw


@pytest.mark.parametrize("rows,k,n", [(1, 16, 8), (130, 384, 1152), (1369, 1024, 256), (257, 4096, 1024),
                                      (200, 768, 3072), (77, 128, 48)])
def test_linear_s8_packed_bit_exact(cuda, dav2lib, rows, k, n):
    _, _, b, px, sx, pw, sw = _s8_problem(rows + k, rows, k, n)
    out = empty(cuda, (rows, n))
    call(dav2lib, "dav2cuda_linear_s8_packed", ptr(out), ptr(dev(cuda, px.view(np.int32))),
         ptr(dev(cuda, pw.view(np.int32))), ptr(dev(cuda, sx)), ptr(dev(cuda, sw)), ptr(dev(cuda, b)), rows, k, n, 0,
         rows, 0, 1, None)
    finish(cuda, dav2lib)
    want = oracle.linear_s8(px, pw, sx, sw, b, rows, k, n).reshape(rows, n)
    assert np.array_equal(host(out), want)


def test_linear_s8_packed_transposed_offset(cuda, dav2lib):
    rows, k, n = 300, 256, 96
    _, _, b, px, sx, pw, sw = _s8_problem(11, rows, k, n)
    stride = rows + 1
    out = empty(cuda, (n * stride,))
    call(dav2lib, "dav2cuda_linear_s8_packed", ptr(out), ptr(dev(cuda, px.view(np.int32))),
         ptr(dev(cuda, pw.view(np.int32))), ptr(dev(cuda, sx)), ptr(dev(cuda, sw)), ptr(dev(cuda, b)), rows, k, n, 1,
         stride, 1, 1, None)
    finish(cuda, dav2lib)
    want = oracle.linear_s8(px, pw, sx, sw, b, rows, k, n, row_offset=1, row_stride=stride, transposed=True)
    got = host(out)
    mask = np.ones(n * stride, bool)
    mask[::stride] = False  # row 0 of each column is not written
    assert np.array_equal(got[mask], want[mask])


@pytest.mark.parametrize("rows,k,n,gelu", [(1370, 384, 1536, 1), (64, 20, 9, 0), (500, 1024, 1024, 0)])
def test_linear_int8(cuda, dav2lib, rows, k, n, gelu):
    x, w, b, px, sx, pw, sw = _s8_problem(k, rows, k, n)
    ws = dav2lib.dav2cuda_linear_int8_workspace_size(rows, k, n)
    wsb = empty(cuda, (ws,), np.uint8)
    out = empty(cuda, (rows, n))
    call(dav2lib, "dav2cuda_linear_int8", ptr(out), ptr(dev(cuda, x)), ptr(dev(cuda, pw.view(np.int32))),
         ptr(dev(cuda, sw)), ptr(dev(cuda, b)), rows, k, n, gelu, ptr(wsb), ws, None)
    finish(cuda, dav2lib)
    want = oracle.linear_s8(px, pw, sx, sw, b, rows, k, n).reshape(rows, n)
    if gelu:
        want = oracle.gelu(want)
        assert np.abs(host(out) - want).max() <= 1e-4 * max(1.0, np.abs(want).max())
    else:
        assert np.array_equal(host(out), want)


@pytest.mark.parametrize("rows,k,n", [(1370, 1024, 1024), (300, 4096, 1024), (129, 384, 384), (64, 20, 9),
                                      (77, 128, 48)])
def test_linear_int8_residual_bit_exact(cuda, dav2lib, rows, k, n):
    """The encoder's fused int8 residual update (proj: K = D; fc2: K = 4D, which
    runs the 8-warp epilogue; narrow and unaligned outputs take the generic row
    program; K = 20 pads the weight rows) against the oracle's linear_s8 then
    add_scaled, bit for bit."""
    x, _, b, px, sx, pw, sw = _s8_problem(rows * 7 + k, rows, k, n)
    r = rng(rows + n)
    res = r.standard_normal((rows, n)).astype(np.float32)
    gamma = (r.standard_normal(n) * 0.1).astype(np.float32)
    ws = dav2lib.dav2cuda_linear_int8_workspace_size(rows, k, n)
    wsb = empty(cuda, (ws,), np.uint8)
    dres = dev(cuda, res)
    call(dav2lib, "dav2cuda_linear_int8_residual", ptr(dres), ptr(dev(cuda, x)), ptr(dev(cuda, pw.view(np.int32))),
         ptr(dev(cuda, sw)), ptr(dev(cuda, b)), ptr(dev(cuda, gamma)), rows, k, n, ptr(wsb), ws, None)
    finish(cuda, dav2lib)
    lin = oracle.linear_s8(px, pw, sx, sw, b, rows, k, n).reshape(rows, n)
    want = oracle.add_scaled(res, lin, gamma)
    assert np.array_equal(host(dres), want)


def test_conv2d_int8_reference_kat(cuda, dav2lib):
    # tests/vulkan_smoke.cpp:143-186: int8 conv 3x3 pad 1 within 0.006 of fp32 conv
    W, H, C, O, K = 5, 4, 4, 5, 3
    x = (((np.arange(W * H * C) % 23) - 11) * 0.03125).astype(np.float32).reshape(C, H, W)
    w = (((np.arange(O * C * K * K) % 19) - 9) * 0.015625).astype(np.float32).reshape(O, C, K, K)
    b = (np.arange(O) * 0.01).astype(np.float32)
    pw, sw = oracle.pack_weight_s8(w)
    ws = dav2lib.dav2cuda_conv2d_int8_workspace_size(W, H, C, O, K, 1, 1)
    out, wsb = empty(cuda, (O, H, W)), empty(cuda, (ws,), np.uint8)
    call(dav2lib, "dav2cuda_conv2d_int8", ptr(out), ptr(dev(cuda, x)), ptr(dev(cuda, pw.view(np.int32))),
         ptr(dev(cuda, sw)), ptr(dev(cuda, b)), W, H, C, O, K, 1, 1, 1, ptr(wsb), ws, None)
    finish(cuda, dav2lib)
    got = host(out)
    assert np.abs(got - oracle.conv2d_f32(x, w, b, 1, 1)).max() <= 0.006
    pk, sc = oracle.im2col_quantize_s8(x, 3, 1, 1)
    want = oracle.linear_s8(pk, pw, sc, sw, b, W * H, C * 9, O, transposed=True).reshape(O, H, W)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("c,h,w,o,k,s", [(256, 19, 23, 256, 3, 1), (64, 37, 37, 128, 3, 2), (32, 10, 12, 16, 1, 1)])
def test_conv2d_int8_bit_exact(cuda, dav2lib, c, h, w, o, k, s):
    p = k // 2
    x = rng(c).standard_normal((c, h, w)).astype(np.float32)
    wt = (rng(o).standard_normal((o, c, k, k)) * 0.02).astype(np.float32)
    b = rng(1).standard_normal(o).astype(np.float32)
    pw, sw = oracle.pack_weight_s8(wt)
    ow, oh = (w + 2 * p - k) // s + 1, (h + 2 * p - k) // s + 1
    ws = dav2lib.dav2cuda_conv2d_int8_workspace_size(w, h, c, o, k, s, p)
    out, wsb = empty(cuda, (o, oh, ow)), empty(cuda, (ws,), np.uint8)
    call(dav2lib, "dav2cuda_conv2d_int8", ptr(out), ptr(dev(cuda, x)), ptr(dev(cuda, pw.view(np.int32))),
         ptr(dev(cuda, sw)), ptr(dev(cuda, b)), w, h, c, o, k, s, p, 1, ptr(wsb), ws, None)
    finish(cuda, dav2lib)
    pk, sc = oracle.im2col_quantize_s8(x, k, s, p)
    want = oracle.linear_s8(pk, pw, sc, sw, b, ow * oh, c * k * k, o, transposed=True).reshape(o, oh, ow)
    assert np.array_equal(host(out), want)


def test_conv_transpose_int8_reference_kat(cuda, dav2lib):
    # tests/vulkan_smoke.cpp:187-240: int8 ConvT within 0.004 of fp32 ConvT
    W, H, I, O, K = 3, 2, 4, 3, 2
    x = (((np.arange(W * H * I) % 17) - 8) * 0.03125).astype(np.float32).reshape(I, H, W)
    w = (((np.arange(I * O * K * K) % 13) - 6) * 0.02).astype(np.float32).reshape(I, O, K, K)
    b = (np.arange(O) * 0.01).astype(np.float32)
    pw, sw = oracle.pack_weight_s8(w, transposed_conv=True)
    ws = dav2lib.dav2cuda_conv_transpose_int8_workspace_size(W, H, I, O, K)
    out, wsb = empty(cuda, (O, H * K, W * K)), empty(cuda, (ws,), np.uint8)
    call(dav2lib, "dav2cuda_conv_transpose_int8", ptr(out), ptr(dev(cuda, x)), ptr(dev(cuda, pw.view(np.int32))),
         ptr(dev(cuda, sw)), ptr(dev(cuda, b)), W, H, I, O, K, ptr(wsb), ws, None)
    finish(cuda, dav2lib)
    got = host(out)
    assert np.abs(got - oracle.conv_transpose_f32(x, w, b)).max() <= 0.004
    pk, sc = oracle.im2col_quantize_s8(x, 1, 1, 0)
    assert np.array_equal(got, oracle.conv_transpose_s8(pk, pw, sc, sw, b, W, H, I, O, K))


@pytest.mark.parametrize("c,h,w,k", [(256, 37, 37, 4), (512, 19, 21, 2), (48, 5, 7, 4)])
def test_conv_transpose_int8_bit_exact(cuda, dav2lib, c, h, w, k):
    x = rng(c).standard_normal((c, h, w)).astype(np.float32)
    wt = (rng(k).standard_normal((c, c, k, k)) * 0.02).astype(np.float32)
    b = rng(2).standard_normal(c).astype(np.float32)
    pw, sw = oracle.pack_weight_s8(wt, transposed_conv=True)
    ws = dav2lib.dav2cuda_conv_transpose_int8_workspace_size(w, h, c, c, k)
    out, wsb = empty(cuda, (c, h * k, w * k)), empty(cuda, (ws,), np.uint8)
    call(dav2lib, "dav2cuda_conv_transpose_int8", ptr(out), ptr(dev(cuda, x)), ptr(dev(cuda, pw.view(np.int32))),
         ptr(dev(cuda, sw)), ptr(dev(cuda, b)), w, h, c, c, k, ptr(wsb), ws, None)
    finish(cuda, dav2lib)
    pk, sc = oracle.im2col_quantize_s8(x, 1, 1, 0)
    assert np.array_equal(host(out), oracle.conv_transpose_s8(pk, pw, sc, sw, b, w, h, c, c, k))


@pytest.mark.parametrize("B,C,H,W,O", [(2, 256, 20, 18, 256),
                                       # ragged pixel tiles, a partial channel chunk, zero pad columns (kp > 9C)
                                       (1, 36, 9, 70, 32),
                                       # two channel chunks (128 + 4), planar conv output (O % 32 != 0)
                                       (1, 132, 5, 33, 48),
                                       # 1x1 maps: every tap but the centre is padding
                                       (3, 8, 1, 1, 64)])
def test_conv3x3_int8_up2(cuda, dav2lib, B, C, H, W, O):
    x = rng(7).standard_normal((B, C, H, W)).astype(np.float32)
    wt = rng(8).uniform(-127, 127, (O, C, 3, 3)).astype(np.float32)
    b = rng(9).standard_normal(O).astype(np.float32)
    pw, sw = oracle.pack_weight_s8(wt)
    ws = dav2lib.dav2cuda_conv3x3_int8_up2_workspace_size(B, W, H, C, O)
    out, wsb = empty(cuda, (B, O, 2 * H, 2 * W)), empty(cuda, (ws,), np.uint8)
    call(dav2lib, "dav2cuda_conv3x3_int8_up2", ptr(out), ptr(dev(cuda, x)), ptr(dev(cuda, pw.view(np.int32))),
         ptr(dev(cuda, sw)), ptr(dev(cuda, b)), B, W, H, C, O, ptr(wsb), ws, None)
    finish(cuda, dav2lib)
    got = host(out)
    for i in range(B):
        pk, sc = oracle.im2col_quantize_s8(x[i], 3, 1, 1)
        conv = oracle.linear_s8(pk, pw, sc, sw, b, H * W, C * 9, O, transposed=True).reshape(O, H, W)
        assert np.array_equal(got[i], oracle.bilinear_align_true(conv, 2 * W, 2 * H))


def test_conv3x3_int8_up2_bench_shape(cuda, dav2lib):
    """BASELINE configuration 2's full shape [8,256,148,148]: the last image's
    codes and scales (read back from the workspace) bit-exact against the
    oracle, and its upsampled output bit-exact against the oracle's order of
    operations. The conv sums are an exact float64 BLAS product of the integer
    codes (|acc| < 2^24), dequantized in f32 as (acc*s_in)*s_w + b."""
    B, C, H, W, O = 8, 256, 148, 148, 256
    x = rng(11).standard_normal((B, C, H, W)).astype(np.float32)
    wt = rng(12).uniform(-127, 127, (O, C, 3, 3)).astype(np.float32)
    b = rng(13).standard_normal(O).astype(np.float32)
    pw, sw = oracle.pack_weight_s8(wt)
    ws = dav2lib.dav2cuda_conv3x3_int8_up2_workspace_size(B, W, H, C, O)
    out, wsb = empty(cuda, (B, O, 2 * H, 2 * W)), empty(cuda, (ws,), np.uint8)
    call(dav2lib, "dav2cuda_conv3x3_int8_up2", ptr(out), ptr(dev(cuda, x)), ptr(dev(cuda, pw.view(np.int32))),
         ptr(dev(cuda, sw)), ptr(dev(cuda, b)), B, W, H, C, O, ptr(wsb), ws, None)
    finish(cuda, dav2lib)
    i, hw, K = B - 1, H * W, 9 * C
    kp = (K + 15) // 16 * 16
    a256 = lambda n: (n + 255) // 256 * 256
    codes_off = a256(B * hw * 4)
    scales_off = codes_off + a256(B * hw * kp)
    got_codes = wsb[codes_off + i * hw * kp: codes_off + (i + 1) * hw * kp].cpu().numpy().view(np.int8)
    got_scales = wsb[scales_off + i * hw * 4: scales_off + (i + 1) * hw * 4].cpu().numpy().view(np.float32)
    pk, sc = oracle.im2col_quantize_s8(x[i], 3, 1, 1)
    codes = pk.view(np.int8).reshape(hw, -1)[:, :K]  # columns (c, ky, kx)
    assert np.array_equal(got_scales, sc)
    # the device rows hold the same codes in (ky, kx, c) column order
    assert np.array_equal(got_codes.reshape(hw, kp)[:, :K].reshape(hw, 9, C),
                          codes.reshape(hw, C, 9).transpose(0, 2, 1))
    wc = pw.view(np.int8).reshape(O, -1)[:, :K].astype(np.float64)
    conv = np.empty((hw, O), np.float32)
    for r0 in range(0, hw, 4096):
        acc = codes[r0:r0 + 4096].astype(np.float64) @ wc.T
        conv[r0:r0 + 4096] = (acc.astype(np.float32) * sc[r0:r0 + 4096, None]) * sw[None, :] + b[None, :]
    want = oracle.bilinear_align_true(np.ascontiguousarray(conv.T.reshape(O, H, W)), 2 * W, 2 * H)
    assert np.array_equal(host(out[i]), want)


@pytest.mark.parametrize("bf16,b,c,h,w,max_depth", [(0, 2, 128, 20, 150, 0.0),   # ViT-L head width, ragged tile
                                                   (1, 2, 128, 9, 300, 0.0),
                                                   (0, 1, 64, 1, 37, 0.0),      # one row: halo rows are padding
                                                   (1, 1, 64, 3, 518, 0.0),
                                                   (0, 1, 128, 5, 128, 20.0)])  # metric head
def test_conv3x3_head_16(cuda, dav2lib, bf16, b, c, h, w, max_depth):
    """The output head kernel (3x3 conv to 32 channels, ReLU, 1x1 to one
    channel, ReLU or sigmoid * max_depth) against a float64 evaluation of the
    same 16-bit inputs; the kernel accumulates in f32, bound 2e-4 of the
    largest |depth|."""
    torch = cuda
    dt = torch.bfloat16 if bf16 else torch.float16
    r = rng(c + h + w)
    x = torch.from_numpy(r.standard_normal((b, h, w, c)).astype(np.float32)).to(dt)
    wt = torch.from_numpy((r.standard_normal((32, 9 * c)) * 0.03).astype(np.float32)).to(dt)
    bias = (r.standard_normal(32) * 0.1).astype(np.float32)
    hw = (r.standard_normal(32) * 0.2).astype(np.float32)
    hb = 0.05
    xd, wd = x.cuda(), wt.cuda()
    out = empty(cuda, (b, h, w))
    call(dav2lib, "dav2cuda_conv3x3_head_16", ptr(out), xd.data_ptr(), wd.data_ptr(), ptr(dev(cuda, bias)),
         ptr(dev(cuda, hw)), hb, max_depth, b, w, h, c, bf16, None)
    finish(cuda, dav2lib)
    xf = np.pad(x.float().numpy().astype(np.float64), ((0, 0), (1, 1), (1, 1), (0, 0)))
    wf = wt.float().numpy().astype(np.float64)
    acc = np.zeros((b, h, w, 32))
    for t in range(9):
        ky, kx = divmod(t, 3)
        acc += xf[:, ky:ky + h, kx:kx + w, :] @ wf[:, t * c:(t + 1) * c].T
    d = np.maximum(acc + bias, 0.0) @ hw.astype(np.float64) + hb
    want = max_depth / (1.0 + np.exp(-d)) if max_depth > 0 else np.maximum(d, 0.0)
    got = host(out)
    assert np.abs(got - want).max() <= 2e-4 * max(np.abs(want).max(), 1e-6)


@pytest.mark.parametrize("bf16,b,c,h,w", [(0, 2, 256, 7, 150),    # odd height: the last tile's second row is padding
                                          (1, 1, 256, 4, 296),
                                          (0, 1, 64, 1, 37),      # one row
                                          (1, 2, 128, 6, 128)])
def test_conv3x3_c128_16(cuda, dav2lib, bf16, b, c, h, w):
    """output_conv1's kernel (3x3 to 128 channels + bias, 16-bit channels-last)
    against a float64 evaluation of the same 16-bit inputs, compared after
    rounding the reference to the 16-bit type: within one 16-bit step plus the
    f32 accumulation error (bound 8e-3 of the largest |output|)."""
    torch = cuda
    dt = torch.bfloat16 if bf16 else torch.float16
    r = rng(c + h + w + 1)
    x = torch.from_numpy(r.standard_normal((b, h, w, c)).astype(np.float32)).to(dt)
    wt = torch.from_numpy((r.standard_normal((128, 9 * c)) * 0.03).astype(np.float32)).to(dt)
    bias = (r.standard_normal(128) * 0.1).astype(np.float32)
    xd, wd = x.cuda(), wt.cuda()
    out = torch.empty((b, h, w, 128), dtype=dt, device="cuda")
    call(dav2lib, "dav2cuda_conv3x3_c128_16", out.data_ptr(), xd.data_ptr(), wd.data_ptr(), ptr(dev(cuda, bias)),
         b, w, h, c, bf16, None)
    finish(cuda, dav2lib)
    xf = np.pad(x.float().numpy().astype(np.float64), ((0, 0), (1, 1), (1, 1), (0, 0)))
    wf = wt.float().numpy().astype(np.float64)
    acc = np.zeros((b, h, w, 128))
    for t in range(9):
        ky, kx = divmod(t, 3)
        acc += xf[:, ky:ky + h, kx:kx + w, :] @ wf[:, t * c:(t + 1) * c].T
    want = acc + bias
    got = out.float().cpu().numpy().astype(np.float64)
    assert np.abs(got - want).max() <= 8e-3 * np.abs(want).max()


# ------------------------------------------------------------- attention
def test_attention_reference_kat(cuda, dav2lib):
    # tests/vulkan_smoke.cpp:540-628: 5 tokens, 2 heads; fp16 within 3e-4 of fp32
    T, Hh = 5, 2
    qkv = (((np.arange(T * Hh * 64 * 3) % 29) - 14) * 0.0078125).astype(np.float32)
    ws = dav2lib.dav2cuda_attention_head64_workspace_size(1, T, Hh)
    out, wsb = empty(cuda, (T, Hh * 64)), empty(cuda, (ws,), np.uint8)
    call(dav2lib, "dav2cuda_attention_head64", ptr(out), ptr(dev(cuda, qkv)), 1, T, Hh, ptr(wsb), ws, None)
    finish(cuda, dav2lib)
    assert np.abs(host(out) - oracle.attention_head64(qkv, T, Hh)).max() <= 3e-4


@pytest.mark.parametrize("batch,tokens,heads", [(1, 1370, 6), (2, 130, 16), (1, 63, 2), (1, 5477, 1),
                                                 (1, 1300, 2), (3, 384, 3),
                                                 # more work units than SMs: each persistent CTA walks
                                                 # several units (two-tile units, then single-tile tails)
                                                 (4, 1370, 16), (3, 256, 64), (5, 100, 40), (2, 513, 50)])
def test_attention(cuda, dav2lib, batch, tokens, heads):
    qkv = (rng(tokens).standard_normal((batch, tokens, 3 * heads * 64)) * 0.5).astype(np.float32)
    ws = dav2lib.dav2cuda_attention_head64_workspace_size(batch, tokens, heads)
    out, wsb = empty(cuda, (batch, tokens, heads * 64)), empty(cuda, (ws,), np.uint8)
    call(dav2lib, "dav2cuda_attention_head64", ptr(out), ptr(dev(cuda, qkv)), batch, tokens, heads, ptr(wsb), ws,
         None)
    finish(cuda, dav2lib)
    got = host(out)
    for i in range(batch):
        want = oracle.attention_head64(qkv[i], tokens, heads)
        assert np.abs(got[i] - want).max() <= 5e-3 * np.abs(want).max()


# -------------------------------------------------------- half tensor cores
@pytest.mark.parametrize("rows,k,n,precision", [(3, 19, 7, 2), (1370, 384, 1152, 1), (257, 1024, 4096, 2)])
def test_linear_half(cuda, dav2lib, rows, k, n, precision):
    # tests/vulkan_smoke.cpp:338-402 pattern for the small case
    if rows == 3:
        x = (((np.arange(rows * k) % 13) - 6) * 0.03125).astype(np.float32).reshape(rows, k)
        w = (((np.arange(n * k) % 11) - 5) * 0.015625).astype(np.float32).reshape(n, k)
        b = (np.arange(n) * 0.0625).astype(np.float32)
    else:
        x = rng(k).standard_normal((rows, k)).astype(np.float32)
        w = (rng(n).standard_normal((n, k)) * 0.02).astype(np.float32)
        b = rng(1).standard_normal(n).astype(np.float32)
    ws = dav2lib.dav2cuda_linear_half_workspace_size(rows, k, n)
    out, wsb = empty(cuda, (rows, n)), empty(cuda, (ws,), np.uint8)
    call(dav2lib, "dav2cuda_linear_half", ptr(out), ptr(dev(cuda, x)), ptr(dev(cuda, w)), ptr(dev(cuda, b)), rows, k,
         n, 0, precision, ptr(wsb), ws, None)
    finish(cuda, dav2lib)
    want = oracle.linear_f32(x, w, b)
    tol = 4e-3 if precision == 2 else 2e-2
    assert max_rel(host(out), want) < tol


@pytest.mark.parametrize("c,h,w,o,k,s,p", [(5, 9, 11, 9, 3, 2, 1), (64, 20, 24, 64, 3, 1, 1), (256, 37, 37, 256, 3, 1, 1),
                                           (128, 30, 17, 32, 3, 1, 1), (32, 7, 9, 1, 1, 1, 0), (96, 8, 8, 64, 1, 1, 0)])
def test_conv2d_half(cuda, dav2lib, c, h, w, o, k, s, p):
    if c == 5:  # tests/vulkan_smoke.cpp:241-337 pattern (conv 3x3 stride 2)
        x = (((np.arange(c * h * w) % 17) - 8) * 0.03125).astype(np.float32).reshape(c, h, w)
        wt = (((np.arange(o * c * 9) % 13) - 6) * 0.015625).astype(np.float32).reshape(o, c, 3, 3)
        b = ((np.arange(o) - 4) * 0.0078125).astype(np.float32)
    else:
        x = rng(c + h).standard_normal((c, h, w)).astype(np.float32)
        wt = (rng(o).standard_normal((o, c, k, k)) * 0.05).astype(np.float32)
        b = rng(3).standard_normal(o).astype(np.float32)
    ow, oh = (w + 2 * p - k) // s + 1, (h + 2 * p - k) // s + 1
    ws = dav2lib.dav2cuda_conv2d_half_workspace_size(w, h, c, o, k, s, p)
    out, wsb = empty(cuda, (o, oh, ow)), empty(cuda, (ws,), np.uint8)
    call(dav2lib, "dav2cuda_conv2d_half", ptr(out), ptr(dev(cuda, x)), ptr(dev(cuda, wt)), ptr(dev(cuda, b)), w, h,
         c, o, k, s, p, ptr(wsb), ws, None)
    finish(cuda, dav2lib)
    want = oracle.conv2d_f32(x, wt, b, s, p)
    assert max_rel(host(out), want) < 4e-3


# ------------------------------------------------------ error behaviour
def test_invalid_arguments_do_not_launch(cuda, dav2lib):
    before = dav2lib.dav2cuda_launch_count(0)
    assert dav2lib.dav2cuda_layer_norm(None, None, None, None, 0, 4, 1e-6, None) == 1
    assert b"layer norm" in dav2lib.dav2cuda_last_error()
    assert dav2lib.dav2cuda_add_scaled(None, None, None, None, 10, 3, None) == 1
    assert dav2lib.dav2cuda_quantize_rows_s8(None, None, None, 2, 6, 0, None) == 1
    assert dav2lib.dav2cuda_linear_s8_packed(None, None, None, None, None, None, 4, 20, 4, 0, 4, 0, 0, None) == 1
    assert dav2lib.dav2cuda_launch_count(0) == before


@pytest.mark.parametrize("kind,shape", [(0, (1152, 384)), (0, (96, 1020)), (1, (256, 256, 4, 4)), (1, (48, 48, 4, 4)),
                                        (2, (64, 96, 3, 3)), (2, (256, 1024, 3, 3))])
def test_device_weight_packing_bit_exact(cuda, dav2lib, kind, shape):
    """The executor's on-device int8 weight packer (per-output-row symmetric
    codes, src/gpu_model.cpp:207-284) against the oracle's packer: kind 0 a
    linear [N][K]; kind 1 a conv-transpose [Ci][Co][k][k] read as rows
    (ky*k+kx)*Co+co over Ci; kind 2 a conv [Co][Ci][k][k] whose columns the
    device orders (ky, kx, ci) — the oracle's (ci, ky, kx) codes permuted."""
    w = (rng(sum(shape)).standard_normal(shape) * 0.02).astype(np.float32)
    w.reshape(shape[0], -1)[1] = 0.0  # an all-zero row (scale floor 1e-8)
    if kind == 0:
        rows, K, co, k, ci = shape[0], shape[1], 0, 0, 0
    elif kind == 1:
        ci, co, k = shape[0], shape[1], shape[2]
        rows, K = k * k * co, ci
    else:
        co, ci, k = shape[0], shape[1], shape[2]
        rows, K = co, ci * k * k
    kp = (K + 15) // 16 * 16
    out, sc = empty(cuda, (rows, kp), np.uint8), empty(cuda, (rows,))
    call(dav2lib, "dav2cuda_pack_weight_s8", ptr(out), ptr(sc), ptr(dev(cuda, w)), kind, rows, K, kp, co, k, ci, None)
    finish(cuda, dav2lib)
    codes = host(out).view(np.int8)[:, :K]
    want_pk, want_sc = oracle.pack_weight_s8(w, transposed_conv=(kind == 1))
    want = want_pk.view(np.int8).reshape(rows, -1)[:, :K]
    if kind == 2:  # oracle columns (ci, ky, kx) -> device columns (ky, kx, ci)
        want = want.reshape(rows, ci, k, k).transpose(0, 2, 3, 1).reshape(rows, K)
    assert np.array_equal(host(sc), want_sc)
    assert np.array_equal(codes, want)
    assert not host(out)[:, K:].any()  # padding columns are zero


# ------------------------------------------------------------- token ops
def _prepare_tokens(cuda, dav2lib, image, w_patch, bias, cls, pos, e, mode):
    _, h, w = image.shape
    t = 1 + (w // 14) * (h // 14)
    ws = dav2lib.dav2cuda_prepare_tokens_workspace_size(w, h, e)
    out, wsb = empty(cuda, (t, e)), empty(cuda, (ws,), np.uint8)
    if mode == "int8":
        pw, sw = oracle.pack_weight_s8(w_patch.reshape(e, -1))
        call(dav2lib, "dav2cuda_prepare_tokens_int8", ptr(out), ptr(dev(cuda, image)), ptr(dev(cuda, pw)),
             ptr(dev(cuda, sw)), ptr(dev(cuda, bias)), ptr(dev(cuda, cls)), ptr(dev(cuda, pos)), w, h, e, ptr(wsb), ws,
             None)
    else:
        call(dav2lib, "dav2cuda_prepare_tokens_half", ptr(out), ptr(dev(cuda, image)), ptr(dev(cuda, w_patch)),
             ptr(dev(cuda, bias)), ptr(dev(cuda, cls)), ptr(dev(cuda, pos)), w, h, e, {"bf16": 1, "f16": 2}[mode],
             ptr(wsb), ws, None)
    finish(cuda, dav2lib)
    return host(out)


@pytest.mark.parametrize("mode", ["f16", "bf16", "int8"])
def test_prepare_tokens_reference_kat(cuda, dav2lib, mode):
    """tests/vulkan_smoke.cpp:630-754: a 42x28 zero image (3x2 patch grid, not
    37x37), zero patch weights, embedding 3: every token is its bias plus the
    bicubic-resized position (class row: class token + position row 0),
    within 2e-6 (exact zeros through the tensor-core GEMM)."""
    e, w, h = 3, 42, 28
    image = np.zeros((3, h, w), np.float32)
    w_patch = np.zeros((e, 3, 14, 14), np.float32)
    bias = np.array([0.25, -0.5, 0.75], np.float32)
    cls = np.array([1.0, 2.0, 3.0], np.float32)
    pos = ((np.arange(1370 * e) % 31 - 15) * 0.015625).astype(np.float32).reshape(1370, e)
    got = _prepare_tokens(cuda, dav2lib, image, w_patch, bias, cls, pos, e, mode)
    assert np.array_equal(got[0], cls + pos[0])
    planar = oracle.position_bicubic(pos, w // 14, h // 14)  # [e][ph][pw], pinned to the same KAT on the CPU
    want = bias[None, :] + planar.reshape(e, -1).T
    assert np.abs(got[1:] - want).max() <= 2e-6


@pytest.mark.parametrize("mode", ["f16", "int8"])
@pytest.mark.parametrize("w,h", [(84, 70), (518, 518)])
def test_prepare_tokens_vs_oracle(cuda, dav2lib, mode, w, h):
    """Seeded image and ViT-S-sized weights; 518x518 is the 37x37 identity
    grid, 84x70 a resized one. int8: codes, integer GEMM and dequant are
    exact, so only the bicubic position sum can differ in the last bit."""
    r = rng(w + h)
    e = 384
    image = r.standard_normal((3, h, w)).astype(np.float32)
    w_patch = (r.standard_normal((e, 3, 14, 14)) * 0.02).astype(np.float32)
    bias = (r.standard_normal(e) * 0.02).astype(np.float32)
    cls = (r.standard_normal(e) * 0.02).astype(np.float32)
    pos = (r.standard_normal((1370, e)) * 0.02).astype(np.float32)
    got = _prepare_tokens(cuda, dav2lib, image, w_patch, bias, cls, pos, e, mode)
    pw, ph = w // 14, h // 14
    sd = {"pretrained.patch_embed.proj.weight": w_patch, "pretrained.patch_embed.proj.bias": bias,
          "pretrained.cls_token": cls, "pretrained.pos_embed": pos}
    want = oracle.embed(sd, image, "vits", "int8" if mode == "int8" else "fp32")
    err = max_rel(got, want)
    print(f"prepare_tokens {mode} {w}x{h}: max rel {err:.2e}")
    assert err < (1e-5 if mode == "int8" else 4e-3)


@pytest.mark.parametrize("mode", ["f16", "bf16", "int8"])
@pytest.mark.parametrize("pw,ph,e,co", [(37, 37, 1024, 256), (6, 5, 384, 48), (37, 37, 768, 768)])
def test_project_tokens_vs_oracle(cuda, dav2lib, mode, pw, ph, e, co):
    r = rng(e + co)
    tokens = r.standard_normal((1 + pw * ph, e)).astype(np.float32)
    wt = (r.standard_normal((co, e)) * 0.02).astype(np.float32)
    b = (r.standard_normal(co) * 0.02).astype(np.float32)
    ws = dav2lib.dav2cuda_project_tokens_workspace_size(pw, ph, e, co)
    out, wsb = empty(cuda, (co, ph, pw)), empty(cuda, (ws,), np.uint8)
    if mode == "int8":
        pk, sw = oracle.pack_weight_s8(wt)
        call(dav2lib, "dav2cuda_project_tokens_int8", ptr(out), ptr(dev(cuda, tokens)), ptr(dev(cuda, pk)),
             ptr(dev(cuda, sw)), ptr(dev(cuda, b)), pw, ph, e, co, ptr(wsb), ws, None)
        finish(cuda, dav2lib)
        px, sx = oracle.quantize_rows_s8(tokens, pw * ph, e, input_offset=e)
        want = oracle.linear_s8(px, pk, sx, sw, b, pw * ph, e, co, transposed=True).reshape(co, ph, pw)
        assert np.array_equal(host(out), want)  # bit-exact: codes, integer GEMM, dequant order
    else:
        call(dav2lib, "dav2cuda_project_tokens_half", ptr(out), ptr(dev(cuda, tokens)), ptr(dev(cuda, wt)),
             ptr(dev(cuda, b)), pw, ph, e, co, {"bf16": 1, "f16": 2}[mode], ptr(wsb), ws, None)
        finish(cuda, dav2lib)
        want = oracle.project_tokens_f32(tokens, wt, b, pw, ph)
        assert max_rel(host(out), want) < (4e-3 if mode == "f16" else 2e-2)


@pytest.mark.parametrize("mode", ["f16", "bf16"])
@pytest.mark.parametrize("c,h,w,o,k", [(256, 37, 37, 256, 4), (512, 37, 37, 512, 2), (48, 5, 7, 48, 4), (20, 3, 4, 12, 2)])
def test_conv_transpose_half_vs_oracle(cuda, dav2lib, mode, c, h, w, o, k):
    r = rng(c + k)
    x = r.standard_normal((c, h, w)).astype(np.float32)
    wt = (r.standard_normal((c, o, k, k)) * 0.05).astype(np.float32)
    b = r.standard_normal(o).astype(np.float32)
    ws = dav2lib.dav2cuda_conv_transpose_half_workspace_size(w, h, c, o, k)
    out, wsb = empty(cuda, (o, h * k, w * k)), empty(cuda, (ws,), np.uint8)
    call(dav2lib, "dav2cuda_conv_transpose_half", ptr(out), ptr(dev(cuda, x)), ptr(dev(cuda, wt)), ptr(dev(cuda, b)),
         w, h, c, o, k, {"bf16": 1, "f16": 2}[mode], ptr(wsb), ws, None)
    finish(cuda, dav2lib)
    want = oracle.conv_transpose_f32(x, wt, b)
    assert max_rel(host(out), want) < (4e-3 if mode == "f16" else 2e-2)
