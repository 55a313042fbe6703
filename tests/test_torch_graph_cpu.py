"""Pins the PyTorch-CPU restatement used as the CPU baseline
(oracle/torch_graph.py) to the reference model's own outputs."""
from pathlib import Path

import numpy as np
import pytest

import torch_graph
from conftest import max_rel
from dav2_b200 import dav2file

G = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("tag", ["base", "strong"])
@pytest.mark.parametrize("shape", ["70x98", "126x126"])
def test_torch_graph_vs_reference(tag, shape):
    fx = np.load(G / "model_vits.npz")
    sd = dav2file.random_state_dict("vits", seed=0) if tag == "base" else \
        dav2file.random_state_dict("vits", seed=1, std=0.05, bias_std=0.02)
    got = torch_graph.forward(torch_graph.to_torch(sd), fx[f"{tag}_{shape}_in"][None], "vits")[0].numpy()
    assert max_rel(got, fx[f"{tag}_{shape}_out"]) < 1e-5


def test_torch_graph_infer_image():
    import oracle

    fx = np.load(G / "image_vits.npz")
    sd = dav2file.random_state_dict("vits", seed=1, std=0.05, bias_std=0.02)
    nw, nh = oracle.network_shape(53, 37, 70)
    x = oracle.preprocess_bgr8(fx["bgr"], nw, nh)[None]
    got = torch_graph.forward(torch_graph.to_torch(sd), x, "vits", out_size=(37, 53))[0].numpy()
    assert max_rel(got, fx["depth"]) < 1e-5
