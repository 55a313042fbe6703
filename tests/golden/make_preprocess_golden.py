"""Generate tests/golden/preprocess_ref.npz from the reference's OWN native
image preprocessing (src/image.cpp: network_shape, preprocess_bgr8,
preprocess_inferbridge_bgra8), compiled from the reference sources into
oracle/_ref/ by `make -C oracle ref REF=<checkout>`.

Run where the reference checkout exists:
    python tests/golden/make_preprocess_golden.py /path/to/Depth-Anything-V2
The GPU box never needs the reference: the fixture travels instead.

Contents:
  shape_in / shape_out / shape_rc   network_shape on a table of sizes
                                     (rc 1 where the reference throws);
  bgr{i}_src, bgr{i}_meta, bgr{i}_out        preprocess_bgr8 cases;
  bgra{i}_src, bgra{i}_meta, bgra{i}_out     preprocess_inferbridge_bgra8
                                     cases. meta = [width, height, stride
                                     bytes, dst_w, dst_h]; src is the padded
                                     buffer [height, stride].
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE = HERE.parent.parent / "oracle"

SHAPES = [(640, 480, 518), (480, 640, 518), (1920, 1080, 518), (518, 518, 518), (53, 37, 70), (37, 53, 70),
          (1, 1000, 70), (1000, 1, 70), (7, 7, 14), (13, 29, 14), (255, 1, 518), (0, 10, 70), (10, 10, 0)]
# (width, height, extra stride bytes, input size)
BGR_CASES = [(53, 37, 0, 70), (97, 61, 5, 140), (20, 15, 0, 70), (123, 77, 3, 140), (1, 9, 0, 28)]
BGRA_CASES = [(53, 37, 0, 70), (160, 90, 12, 140), (20, 15, 0, 70), (31, 200, 4, 70), (9, 1, 0, 28)]


def main(reference: str) -> None:
    subprocess.run(["make", "-s", "-C", str(ORACLE), "ref", f"REF={reference}"], check=True)
    lib = ctypes.CDLL(str(ORACLE / "_ref" / "libref_image.so"))
    i32p = ctypes.POINTER(ctypes.c_int)
    lib.dav2r_network_shape.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, i32p, i32p]
    for fn in (lib.dav2r_preprocess_bgr8, lib.dav2r_preprocess_inferbridge_bgra8):
        fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_ssize_t, ctypes.c_int, ctypes.c_int,
                       ctypes.c_void_p]
    for fn in (lib.dav2r_network_shape, lib.dav2r_preprocess_bgr8, lib.dav2r_preprocess_inferbridge_bgra8):
        fn.restype = ctypes.c_int

    def shape(w, h, s):
        ow, oh = ctypes.c_int(), ctypes.c_int()
        rc = lib.dav2r_network_shape(w, h, s, ctypes.byref(ow), ctypes.byref(oh))
        return rc, ow.value, oh.value

    out = {}
    res = [shape(*s) for s in SHAPES]
    out["shape_in"] = np.array(SHAPES, np.int32)
    out["shape_rc"] = np.array([r[0] for r in res], np.int32)
    out["shape_out"] = np.array([r[1:] for r in res], np.int32)

    rng = np.random.default_rng(7)
    for tag, cases, ch, fn, swap in (("bgr", BGR_CASES, 3, lib.dav2r_preprocess_bgr8, False),
                                     ("bgra", BGRA_CASES, 4, lib.dav2r_preprocess_inferbridge_bgra8, True)):
        for i, (w, h, pad, size) in enumerate(cases):
            stride = w * ch + pad
            src = rng.integers(0, 256, (h, stride), dtype=np.uint8)
            rc, nw, nh = shape(w, h, size)
            assert rc == 0
            dw, dh = (nh, nw) if swap else (nw, nh)  # InferBridge swaps (src/dav2.cpp:773-776)
            dst = np.empty((3, dh, dw), np.float32)
            assert fn(src.ctypes.data, w, h, stride, dw, dh, dst.ctypes.data) == 0
            out[f"{tag}{i}_src"] = src
            out[f"{tag}{i}_meta"] = np.array([w, h, stride, dw, dh], np.int64)
            out[f"{tag}{i}_out"] = dst
    np.savez_compressed(HERE / "preprocess_ref.npz", **out)
    print("wrote preprocess_ref.npz:", len(out), "arrays")


if __name__ == "__main__":
    # the reference checkout: the first argument, else DAV2_REFERENCE_DIR
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DAV2_REFERENCE_DIR", "")
    if not ref:
        sys.exit(f"usage: python {Path(__file__).name} <reference checkout> (or set DAV2_REFERENCE_DIR)")
    main(ref)
