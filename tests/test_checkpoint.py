"""The checkpoint reader parses the reference's own core_indexer.pt layout
(written by the reference's save_indexer_stack in tests/golden/make_golden.py)."""

import os

import numpy as np
import torch

from core_b200 import checkpoint as C
from helpers import GOLDEN, TWO_STEP_CASE, load_case

CKPT = os.path.join(GOLDEN, "core_indexer_two_step.pt")


def test_reads_reference_checkpoint():
    parts = C.load_checkpoint(CKPT)
    d, m = load_case(TWO_STEP_CASE)
    layer = m["layer"]
    w1, b1, w2, b2, w3, b3 = parts["indexer"].params(layer)
    for got, key in zip((w1, b1, w2, b2, w3, b3),
                        ("mlp_w1", "mlp_b1", "mlp_w2", "mlp_b2", "mlp_w3", "mlp_b3")):
        np.testing.assert_array_equal(got.numpy(), d[key])
    geo = parts["geometry"]
    np.testing.assert_array_equal(geo.weight[layer].numpy(), d["geometry"])
    np.testing.assert_allclose(geo.prototypes.numpy(), d["prototypes"], rtol=1e-6, atol=1e-7)
    np.testing.assert_array_equal(geo.hadamard.numpy(), d["hadamard"])
    th, gw1, gb1, gw2, gb2 = parts["memory"].params(layer)
    np.testing.assert_array_equal(th.numpy(), d["theta"])
    np.testing.assert_array_equal(gw1.numpy(), d["gate_w1"])
    np.testing.assert_array_equal(gw2.numpy(), d["gate_w2"].reshape(-1))
    cfg = parts["config"]
    assert cfg.n_q_heads == 8 and cfg.n_kv_heads == 2 and cfg.memory_dim == 64
    assert parts["use_stack"] is True


def test_fixed_geometry_constructions_match_reference_bank():
    d, m = load_case(TWO_STEP_CASE)
    np.testing.assert_allclose(C.unit_prototypes(64, 64, 42).numpy(), d["prototypes"], rtol=1e-6,
                               atol=1e-7)
    np.testing.assert_allclose(C.hadamard_rotation(64, 42).numpy(), d["hadamard"], rtol=1e-6,
                               atol=1e-7)
    geo = C.gaussian_geometry(2, 2, 128, 64, 42)
    np.testing.assert_allclose(geo[m["layer"]].numpy(), d["geometry"], rtol=1e-6, atol=1e-7)


def test_round_trip(tmp_path):
    parts = C.random_checkpoint_parts(seed=3, n_layers=3, n_kv_heads=2, n_q_heads=8, d_mem=128)
    path = str(tmp_path / "core_indexer.pt")
    C.save_checkpoint(path, config=parts["config"], indexer=parts["indexer"],
                      geometry=parts["geometry"], memory=parts["memory"])
    back = C.load_checkpoint(path)
    for a, b in zip(parts["indexer"].modules[2], back["indexer"].modules[2]):
        assert torch.equal(a, b)
    for a, b in zip(parts["memory"].modules[1], back["memory"].modules[1]):
        assert torch.equal(a.reshape(-1), b.reshape(-1))
    assert torch.equal(back["geometry"].weight, parts["geometry"].weight)


def test_interface_is_validated(tmp_path):
    parts = C.random_checkpoint_parts(seed=1, n_layers=1, n_kv_heads=2, n_q_heads=8, d_mem=128)
    cfg = dict(parts["config"])
    cfg["memory_value_space"] = "post_o_proj"
    path = str(tmp_path / "bad.pt")
    C.save_checkpoint(path, config=cfg, indexer=parts["indexer"], geometry=parts["geometry"])
    try:
        C.load_checkpoint(path)
    except ValueError as e:
        assert "memory_value_space" in str(e)
    else:
        raise AssertionError("interface mismatch not rejected")
