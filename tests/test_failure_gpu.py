"""Failure detection without a GPU fault.

Every pipeline wait of the kernels (TMA ring, TMEM accumulators, softmax
phases) is bounded: when it gives up it sets the device error word to 1 and
the kernel drains and returns, so the context stays usable. Here a wait is
made to run out on purpose through dav2cuda_wait_probe — the same bounded
wait, with a limit of one millisecond, on an mbarrier phase that nothing
completes — and the tests check that the word reaches the host: through the
operator ABI (dav2cuda_device_error) and through the public ABI as
DAV2_STATUS_INFERENCE_FAILED (6) with a message, for a synchronous call and
for the asynchronous caller-stream path. Nothing here faults, traps or hangs
the GPU: the probe kernel touches only its own shared memory and the error
word, and returns after its limit."""
import ctypes

import numpy as np
import pytest

from abi_helpers import create
from dav2_b200 import capi, dav2file

pytestmark = pytest.mark.gpu
LIMIT_NS = 1_000_000  # 1 ms


@pytest.fixture(scope="module")
def vits_model(tmp_path_factory, dav2lib):
    path = tmp_path_factory.mktemp("failure") / "vits.dav2"
    dav2file.write_dav2(path, dav2file.random_state_dict("vits", seed=0), "vits")
    return path


def test_wait_probe_reports_through_the_error_word(cuda, dav2lib):
    assert dav2lib.dav2cuda_device_error() == 0
    assert dav2lib.dav2cuda_wait_probe(LIMIT_NS, 1, None) == 0  # completed phase: no error
    assert dav2lib.dav2cuda_device_error() == 0
    assert dav2lib.dav2cuda_wait_probe(LIMIT_NS, 0, None) == 0  # nothing completes it: gives up
    assert dav2lib.dav2cuda_device_error() == 1
    assert dav2lib.dav2cuda_device_error() == 0  # reading clears the word
    # the limit is validated before any launch
    assert dav2lib.dav2cuda_wait_probe(0, 0, None) == 1
    assert dav2lib.dav2cuda_wait_probe(2_000_000_000, 0, None) == 1


def test_timeout_is_inference_failed_on_a_synchronous_call(cuda, dav2lib, vits_model):
    rc, ctx = create(dav2lib, vits_model, "vits", capi.FLAGS["fp16"])
    assert rc == 0, dav2lib.dav2_last_error()
    try:
        img = np.random.default_rng(0).standard_normal((3, 28, 28)).astype(np.float32)
        out = np.zeros(28 * 28, np.float32)
        assert dav2lib.dav2_infer_tensor_f32(ctx, img.ctypes.data, 28, 28, out.ctypes.data, out.size) == 0
        assert dav2lib.dav2cuda_wait_probe(LIMIT_NS, 0, None) == 0
        cuda.cuda.synchronize()
        assert dav2lib.dav2_synchronize(ctx) == 6
        assert b"timed out" in dav2lib.dav2_last_error()
        assert dav2lib.dav2_synchronize(ctx) == 0  # reported once, then cleared
        again = np.zeros_like(out)
        assert dav2lib.dav2_infer_tensor_f32(ctx, img.ctypes.data, 28, 28, again.ctypes.data, again.size) == 0
        assert np.array_equal(out, again)  # the context is still usable
        # a timeout before a synchronous inference fails that inference
        assert dav2lib.dav2cuda_wait_probe(LIMIT_NS, 0, None) == 0
        cuda.cuda.synchronize()
        assert dav2lib.dav2_infer_tensor_f32(ctx, img.ctypes.data, 28, 28, again.ctypes.data, again.size) == 6
        assert dav2lib.dav2_infer_tensor_f32(ctx, img.ctypes.data, 28, 28, again.ctypes.data, again.size) == 0
    finally:
        dav2lib.dav2_destroy(ctx)


def test_timeout_on_the_caller_stream_path(cuda, dav2lib, vits_model):
    """dav2_infer_device_bgr8_batch on a caller stream returns once the work
    is queued; a device-side failure of that work is reported by
    dav2_synchronize (or the context's next call)."""
    torch = cuda
    rc, ctx = create(dav2lib, vits_model, "vits", capi.FLAGS["fp16"])
    assert rc == 0, dav2lib.dav2_last_error()
    try:
        bgr = torch.randint(0, 256, (2, 42, 56, 3), dtype=torch.uint8, device="cuda")
        out = torch.zeros((2, 42, 56), dtype=torch.float32, device="cuda")
        s = torch.cuda.Stream()
        args = (ctx, bgr.data_ptr(), 2, 56, 42, 56 * 3, 42 * 56 * 3, 56, out.data_ptr(), ctypes.c_void_p(s.cuda_stream))
        assert dav2lib.dav2_infer_device_bgr8_batch(*args) == 0
        assert dav2lib.dav2_synchronize(ctx) == 0
        assert dav2lib.dav2cuda_wait_probe(LIMIT_NS, 0, ctypes.c_void_p(s.cuda_stream)) == 0
        assert dav2lib.dav2_infer_device_bgr8_batch(*args) == 0  # queued behind the probe
        assert dav2lib.dav2_synchronize(ctx) == 6
        assert b"timed out" in dav2lib.dav2_last_error()
        assert dav2lib.dav2_infer_device_bgr8_batch(*args) == 0
        assert dav2lib.dav2_synchronize(ctx) == 0
        assert torch.isfinite(out).all()
    finally:
        dav2lib.dav2_destroy(ctx)
