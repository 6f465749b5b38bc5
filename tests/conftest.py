"""Shared test setup: import paths, the ``gpu`` marker and golden fixtures."""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "flash-head_b200")
GOLDEN = os.path.join(REPO, "tests", "golden")
for p in (PKG, REPO):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def load_golden(name: str):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


def load_golden_meta(name: str) -> dict:
    with open(os.path.join(GOLDEN, name + ".json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def golden_small():
    return load_golden("small_greedy")


@pytest.fixture(scope="session")
def small_head_np(golden_small):
    """The small golden head as numpy arrays (weight as float32 bf16 values)."""
    from oracle import flashhead_oracle as O
    g = golden_small
    W = O.bf16_bits_to_f32(g["weight_bits"])
    C = g["centroids"].astype(np.float32)
    A = g["assignments"].astype(np.int64)
    K = C.shape[1]
    vm = O.vocab_maps_from_assignments(A, K)
    cw = O.bf16_round(O.normalized_cluster_weight(C))
    return {"W": W, "C": C, "A": A, "K": K, "vm": vm, "cw": cw,
            "w_perm": O.permute_weight(W, vm), "p": int(g["n_probes"]),
            "H": O.bf16_bits_to_f32(g["hidden_bits"])}


@pytest.fixture(scope="session")
def config_a_head():
    """Config A head regenerated from its seed (CPU, bit-identical to the fixture's)."""
    from flash_head.synthetic import HeadShape, head_checksum, make_head
    meta = load_golden_meta("config_a")
    shape = HeadShape(**meta["shape"])
    head = make_head(shape, seed=meta["head_seed"])
    assert np.allclose(head_checksum(head), meta["checksum"], rtol=0, atol=0), \
        "regenerated config-A head differs from the one the fixture was made with"
    return head, meta
