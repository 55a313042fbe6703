"""CPU checks of the shipped library: it loads without a GPU, exports every
function that include/*.h declares, and its argument validation answers
before any launch (no compute calls are made here)."""
import ctypes
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def declared_functions():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = "\n".join(l for l in header.read_text().splitlines() if not l.lstrip().startswith("#"))
        for m in re.finditer(r"(?:DAV2CUDA_API|DAV2_API)\s+[^;(]*?\b(\w+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_headers_declare_entry_points():
    names = declared_functions()
    assert "dav2cuda_layer_norm" in names and "dav2cuda_linear_s8_packed" in names


def test_library_exports_every_declared_symbol(dav2lib):
    missing = [n for n in sorted(declared_functions()) if not hasattr(dav2lib, n)]
    assert not missing, f"missing exports: {missing}"


def test_validation_without_gpu(dav2lib):
    # size / null checks return DAV2CUDA_INVALID_ARGUMENT before touching CUDA
    assert dav2lib.dav2cuda_layer_norm(None, None, None, None, 0, 16, 1e-6, None) == 1
    assert b"invalid layer norm" in dav2lib.dav2cuda_last_error()
    assert dav2lib.dav2cuda_add_scaled(None, None, None, None, 10, 3, None) == 1
    assert dav2lib.dav2cuda_quantize_rows_s8(None, None, None, 4, 6, 0, None) == 1
    assert dav2lib.dav2cuda_linear_s8_packed(None, None, None, None, None, None, 4, 20, 4, 0, 4, 0, 0, None) == 1
    assert dav2lib.dav2cuda_conv2d_int8(None, None, None, None, None, 0, 4, 4, 4, 3, 1, 1, 1, None, 0, None) == 1
    assert dav2lib.dav2cuda_linear_int8_workspace_size(1370, 1024, 1024) >= 1370 * 1024
    assert dav2lib.dav2cuda_attention_head64_workspace_size(1, 1370, 16) >= 1370 * 1024 * 2 * 4


def test_validation_of_graph_form_entries(dav2lib):
    # the operator forms of the executor's fused kernels reject bad shapes and
    # buffers before any launch (null pointers only: nothing can be touched)
    f = dav2lib.dav2cuda_linear_int8_residual
    assert f(None, None, None, None, None, None, 0, 1024, 1024, None, 0, None) == 1
    assert b"invalid INT8 residual dimensions" in dav2lib.dav2cuda_last_error()
    assert f(None, None, None, None, None, None, 4, 0xFFFFFFF4, 8, None, 0, None) == 1
    assert b"too large" in dav2lib.dav2cuda_last_error()
    assert f(None, None, None, None, None, None, 4, 1024, 1024, None, 1 << 20, None) == 1
    assert b"null buffer" in dav2lib.dav2cuda_last_error()
    g = dav2lib.dav2cuda_im2col_quantize_nhwc
    assert g(None, None, None, 1, 4, 4, 8, 0, 1, 0, 16, None) == 1
    assert b"invalid channels-last im2col dimensions" in dav2lib.dav2cuda_last_error()
    assert g(None, None, None, 1, 2, 2, 8, 5, 1, 1, 256, None) == 1  # 5x5 kernel on a 2x2 map, pad 1
    assert g(None, None, None, 1, 4, 4, 8, 3, 1, 1, 71, None) == 1  # 72 columns need 72 bytes
    assert b"row_bytes below" in dav2lib.dav2cuda_last_error()
    assert g(None, None, None, 1, 64, 64, 1 << 28, 3, 1, 1, 0xFFFFFFFF, None) == 1
    assert b"too large" in dav2lib.dav2cuda_last_error()
    assert g(None, None, None, 1, 4, 4, 8, 3, 1, 1, 80, None) == 1
    assert b"null buffer" in dav2lib.dav2cuda_last_error()


def test_oracle_library_builds():
    import oracle

    assert oracle.threads() >= 1
