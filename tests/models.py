"""Seeded test models whose depth output is not degenerate.

With the BASELINE init (every weight and bias N(0, 0.02)), the last
convolution's drawn bias often dominates its input: for ViT-L seed 0 every
pixel's ReLU'd depth is 0, for ViT-S seed 0 the map is 0.022 plus a signal a
hundred times smaller. Comparisons on such maps check little, so the parity
tests use these draws with the last bias (depth_head.scratch.
output_conv2.2.bias) set to 0, picked so that the depth keeps a spatial
signal comparable to its maximum at 518x518 (found with the fp32 reference
forward): ViT-S seed 3, ViT-B seed 3 (every pixel positive), ViT-L seed 0
(about 43% positive). Every other weight is the plain draw, so every kernel
does the same work as with the BASELINE init."""
import numpy as np

from dav2_b200 import dav2file

SEEDS = {"vits": 3, "vitb": 3, "vitl": 0}


def nondegenerate(encoder: str) -> dict:
    sd = dav2file.random_state_dict(encoder, seed=SEEDS[encoder])
    name = "depth_head.scratch.output_conv2.2.bias"
    sd[name] = np.zeros_like(sd[name])
    return sd
