"""Offline balanced clustering (flash_head/clustering.py) and the clustering
cache it writes, on CPU.

The reference reads a balanced clustering from clustering_cache.safetensors
(flash_head.py:41-118) but ships no tool that makes one, so there is no
reference output to match: the tests check the properties the reader
requires (every cluster exactly cap tokens, the cache layout), recovery of
the planted clusters of the seeded synthetic heads, the quality of the
FlashHead step built on a learned clustering against the oracle's dense
argmax, and that the reference's own reader accepts the file.
"""

from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle import flashhead_oracle as O

# The reference's source tree (directory holding its flash_head package), when
# present on this machine; the test that runs the reference's reader skips
# without it.
REFERENCE_SRC = os.environ.get("FLASHHEAD_REFERENCE_SRC", "")


def _head(D, V, K, seed, noise_std=0.005):
    from flash_head.synthetic import HeadShape, make_head
    return make_head(HeadShape(hidden=D, vocab=V, n_clusters=K, n_probes=16), seed=seed,
                     noise_std=noise_std)


@pytest.mark.parametrize("D,V,K", [(64, 4096, 256), (128, 16384, 1024)])
def test_recovers_planted_clusters(D, V, K):
    """Centre + noise heads (centres N(0, 0.02^2), noise N(0, 0.005^2)): every
    learned cluster is exactly one planted cluster, and its centroid is that
    cluster's mean row."""
    from flash_head.clustering import balanced_clusters
    head = _head(D, V, K, seed=3)
    assign, cent = balanced_clusters(head.weight, cap=16)
    a, planted = assign.numpy(), head.assignments.numpy()
    assert assign.dtype == torch.int64 and cent.shape == (D, K) and cent.dtype == torch.float32
    assert np.all(np.bincount(a, minlength=K) == 16)
    label = np.empty(K, dtype=np.int64)
    for k in range(K):
        members = set(planted[a == k].tolist())
        assert len(members) == 1, k
        label[k] = members.pop()
    assert len(set(label.tolist())) == K
    np.testing.assert_allclose(cent.numpy(), head.centroids.numpy()[:, label], rtol=0, atol=1e-6)


def test_deterministic_and_input_checks():
    from flash_head.clustering import balanced_clusters
    head = _head(32, 1024, 64, seed=8, noise_std=0.02)
    a1, c1 = balanced_clusters(head.weight, cap=16, seed=4)
    a2, c2 = balanced_clusters(head.weight.clone(), cap=16, seed=4)
    assert torch.equal(a1, a2) and torch.equal(c1, c2)
    a8, _ = balanced_clusters(head.weight, cap=8)
    assert np.all(np.bincount(a8.numpy(), minlength=128) == 8)
    with pytest.raises(ValueError, match="not a multiple"):
        balanced_clusters(head.weight[:1000], cap=16)
    with pytest.raises(ValueError, match=r"\[V, D\]"):
        balanced_clusters(head.weight[0], cap=16)


def test_degenerate_heads_stay_balanced():
    """One cluster, clusters of one token, identical and all-zero rows (ties
    everywhere), and a bf16 weight: every cluster still gets exactly cap
    tokens and the centroids are the member means."""
    from flash_head.clustering import balanced_clusters
    a, c = balanced_clusters(torch.randn(16, 8), cap=16)
    assert a.tolist() == [0] * 16 and c.shape == (8, 1)
    w = torch.randn(10, 4)
    a, c = balanced_clusters(w, cap=1)
    assert sorted(a.tolist()) == list(range(10))
    np.testing.assert_allclose(c.numpy(), w.numpy()[np.argsort(a.numpy())].T, atol=1e-7)
    w = torch.zeros(64, 8)
    w[:32] = torch.randn(1, 8)
    a, c = balanced_clusters(w, cap=16)
    assert np.all(np.bincount(a.numpy(), minlength=4) == 16)
    a, c = balanced_clusters(torch.randn(256, 32).to(torch.bfloat16), cap=16)
    assert np.all(np.bincount(a.numpy(), minlength=16) == 16) and c.dtype == torch.float32


def test_learned_clusters_beat_random_ones_on_a_noisy_head():
    """Noise larger than the centre spread (0.03 vs 0.02): the FlashHead step
    (oracle, p = 16 of 256 clusters) on the learned clustering agrees with the
    dense argmax on far more rows than on a random balanced clustering, and
    nearly as often as on the planted one."""
    from flash_head.clustering import balanced_clusters
    from flash_head.synthetic import make_hidden
    D, V, K, p = 64, 4096, 256, 16
    head = _head(D, V, K, seed=5, noise_std=0.03)
    W = head.weight.float().numpy()
    H = make_hidden(64, D, seed=9).float().numpy()
    dense = [O.dense_argmax(h, W) for h in H]

    def agreement(assign, cent_dk):
        vm = O.vocab_maps_from_assignments(assign, K)
        cw = O.normalized_cluster_weight(cent_dk)
        wp = O.permute_weight(W, vm)
        return np.mean([O.greedy_token(h, wp, vm, cw, p)[0] == d for h, d in zip(H, dense)])

    a, c = balanced_clusters(head.weight, cap=16)
    rnd = np.random.default_rng(0).permutation(np.arange(V) % K)
    rnd_c = np.stack([W[rnd == k].mean(0) for k in range(K)], 1)
    learned, random_ = agreement(a.numpy(), c.numpy()), agreement(rnd, rnd_c)
    planted = agreement(head.assignments.numpy(), head.centroids.numpy())
    assert learned >= random_ + 0.15, (learned, random_)
    assert learned >= planted - 0.1, (learned, planted)


def test_cache_round_trip_through_the_loader(tmp_path):
    """The written cache is read back by get_flash_head_parameters: the same
    centroids and the vocab maps of the assignments."""
    from torch import nn

    from flash_head.clustering import CACHE_FILE, balanced_clusters, save_clustering_cache
    from flash_head.flash_head import get_flash_head_parameters, vocab_maps_from_assignments
    head = _head(64, 4096, 256, seed=3)
    assign, cent = balanced_clusters(head.weight, cap=16)
    path = save_clustering_cache(str(tmp_path / "assets"), cent, assign)
    assert path == str(tmp_path / "assets" / CACHE_FILE)
    lm = nn.Linear(64, 4096, bias=False)
    lm.weight = nn.Parameter(head.weight.float(), requires_grad=False)
    params = get_flash_head_parameters(lm, cache_dir="assets", model_or_dir=str(tmp_path))
    assert torch.equal(params["centroids"], cent)
    assert torch.equal(params["vocab_maps_tensor"], vocab_maps_from_assignments(assign, 256))
    bad = assign.clone()
    bad[0] = (bad[0] + 1) % 256
    with pytest.raises(ValueError, match="not balanced"):
        save_clustering_cache(str(tmp_path / "bad"), cent, bad)
    with pytest.raises(ValueError, match="outside"):
        save_clustering_cache(str(tmp_path / "bad"), cent, assign + 256)


def test_build_cache_from_a_checkpoint(tmp_path):
    """build_clustering_cache reads the LM head of a checkpoint directory (the
    reference's layout, written by synthetic.save_assets) and writes a cache
    that recovers the planted clusters."""
    from safetensors.torch import load_file

    from flash_head.clustering import build_clustering_cache
    from flash_head.synthetic import save_assets
    head = _head(64, 2048, 128, seed=12)
    model = str(tmp_path / "model")
    save_assets(head, model)
    path = build_clustering_cache(model, str(tmp_path / "learned"))
    t = load_file(path)
    a = t["cluster_assignments"].numpy()
    assert t["centroids"].shape == (64, 128) and np.all(np.bincount(a, minlength=128) == 16)
    planted = head.assignments.numpy()
    assert all(len(set(planted[a == k].tolist())) == 1 for k in range(128))


@pytest.mark.skipif(not REFERENCE_SRC or not os.path.isdir(REFERENCE_SRC),
                    reason="FLASHHEAD_REFERENCE_SRC not set to the reference sources")
def test_reference_reader_accepts_the_cache(tmp_path):
    """The reference's own get_flash_head_parameters (run in a separate
    process, its package shadows this one) reads the written cache and
    builds the same vocab maps."""
    from flash_head.clustering import balanced_clusters, save_clustering_cache
    from flash_head.flash_head import vocab_maps_from_assignments
    head = _head(32, 1024, 64, seed=21)
    assign, cent = balanced_clusters(head.weight, cap=16)
    save_clustering_cache(str(tmp_path / "assets"), cent, assign)
    torch.save(head.weight.float(), str(tmp_path / "w.pt"))
    script = (
        "import sys, torch\n"
        f"sys.path.insert(0, {REFERENCE_SRC!r})\n"
        "from torch import nn\n"
        "from flash_head.flash_head import get_flash_head_parameters\n"
        f"w = torch.load({str(tmp_path / 'w.pt')!r})\n"
        "lm = nn.Linear(w.shape[1], w.shape[0], bias=False)\n"
        "lm.weight = nn.Parameter(w, requires_grad=False)\n"
        f"p = get_flash_head_parameters(lm, 'assets', {str(tmp_path)!r})\n"
        f"torch.save({{k: v for k, v in p.items()}}, {str(tmp_path / 'ref.pt')!r})\n")
    env = dict(os.environ, PYTHONDONTWRITEBYTECODE="1", CUDA_VISIBLE_DEVICES="")
    res = subprocess.run([sys.executable, "-c", script], cwd=str(tmp_path), env=env,
                         capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    ref = torch.load(str(tmp_path / "ref.pt"))
    vm_key = next(k for k in ref if "vocab" in k)
    assert torch.equal(ref[vm_key].to(torch.int64), vocab_maps_from_assignments(assign, 64))
    c_key = next(k for k in ref if "centroid" in k)
    assert torch.equal(ref[c_key].float().squeeze(), cent)
