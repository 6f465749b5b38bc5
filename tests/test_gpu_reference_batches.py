"""Kernel outputs against the reference's own outputs on 256 decode rows.

The fixtures (tests/golden/config_b_batch.*, config_c_batch.*) hold what the
reference FlashHead computed on CPU for 256 N(0, 0.25) hidden states of the
Llama-3.2-1B-shaped head (configs A/B) and of the Llama-3.1-8B-shaped head
(config C): its probe sets (flash_head.py:213-214), its largest p + 64 bf16
stage-1 scores with their cluster ids, and its greedy tokens. Heads and
hidden states are regenerated here from their seeds and checksummed.

Rules (the reference's tolerance for bf16 logits, 1e-2 relative):
  * greedy ids identical unless the two tokens' logits are within 1e-2;
  * bf16 stage 1 (the reference's format): probe sets identical except for
    clusters whose reference score is within 1e-2 of the p-th score;
  * fp8 stage 1: the fp8 score error (~2 % of the boundary score on these
    heads) is larger than that band, so the probe-set rule is not expected to
    hold; the test bounds the recall of the reference's probes instead and
    keeps the greedy-token rule.
The same rows also go through the kernels' own oracle check (scores, probes
and tokens on the kernels' own matrices) at 1, 4, 32 and 256 rows.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden, load_golden_meta
from headutil import RTOL, OracleView, build_head, check_greedy_rows, to_np_f32
from oracle import flashhead_oracle as O

pytestmark = pytest.mark.gpu


def _regenerate(name):
    from flash_head.synthetic import HeadShape, head_checksum, make_head, make_hidden
    meta = load_golden_meta(name)
    shape = HeadShape(**meta["shape"])
    head = make_head(shape, seed=meta["head_seed"])
    assert np.allclose(head_checksum(head), meta["checksum"], rtol=0, atol=0), name
    H = make_hidden(meta["rows"], shape.hidden, seed=meta["hidden_seed"])
    b = H.view(torch.int16).to(torch.int64)  # exact: integer sums of the bf16 bits
    idx = torch.arange(b.numel(), dtype=torch.int64).view_as(b)
    assert [int(b.sum()), int((b * (idx % 65521)).sum())] == meta["hidden_checksum"], name
    return head, H, meta


def _reference_rows(fh, g, H_t, stage1):
    """Check every row against the reference; returns the mean probe recall."""
    p = fh.n_probes
    probes = fh.top_clusters_batched(H_t).cpu().numpy()
    toks = fh.get_next_token_batched(H_t).cpu().numpy()
    W = fh.w_perm.view(-1, fh._D)
    vm = fh.vocab_maps.view(-1).cpu().numpy()
    slot = np.empty(vm.size, dtype=np.int64)
    slot[vm] = np.arange(vm.size)
    Hn = to_np_f32(H_t)
    recalls, bad_rows = [], []

    def logit_of(r):
        def f(v):
            return float(W[int(slot[v])].double().cpu() @ torch.from_numpy(Hn[r]).double())
        return f

    for r in range(H_t.shape[0]):
        vals = O.bf16_bits_to_f32(g["ref_top_bits"][r]).astype(np.float64)
        ok, rec, _ = O.probe_rule_vs_reference_list(probes[r], g["ref_probes"][r], vals,
                                                    g["ref_top_ids"][r].astype(np.int64), RTOL)
        recalls.append(rec)
        if stage1 == "model" and not ok:
            bad_rows.append(r)
        assert O.token_within_tolerance(toks[r], int(g["ref_tok_greedy"][r]), logit_of(r),
                                        RTOL), (r, int(toks[r]), int(g["ref_tok_greedy"][r]))
    assert not bad_rows, f"probe-set rule broken on rows {bad_rows[:10]}"
    return float(np.mean(recalls)), float(np.min(recalls)), probes, toks


@pytest.fixture(scope="module")
def config_b():
    head, H, meta = _regenerate("config_b_batch")
    heads = {s: build_head(head.weight, head.centroids, head.assignments,
                           meta["shape"]["n_probes"], stage1=s) for s in ("model", "fp8")}
    return heads, H.cuda(), load_golden("config_b_batch")


@pytest.mark.parametrize("stage1", ["model", "fp8"])
def test_config_b_256_rows_vs_reference(config_b, stage1):
    heads, H, g = config_b
    fh = heads[stage1]
    mean_rec, min_rec, probes, toks = _reference_rows(fh, g, H, stage1)
    print(f"config B {stage1} stage 1: reference probe recall mean {mean_rec:.4f} "
          f"min {min_rec:.4f} over {H.shape[0]} rows")
    if stage1 == "model":
        assert mean_rec >= 0.99
    else:
        assert mean_rec >= 0.95 and min_rec >= 0.90
    # the batched call (256 rows) against the kernels' own oracle
    check_greedy_rows(fh, H, toks, probes)
    assert fh.native().workspace_error() == 0  # no bounded wait ran out


@pytest.mark.parametrize("stage1", ["model", "fp8"])
@pytest.mark.parametrize("rows", [1, 4, 32])
def test_config_b_small_batches_vs_reference(config_b, stage1, rows):
    """The one-kernel (1, 4 rows) and GEMM (32 rows) steps on the same rows."""
    heads, H, g = config_b
    fh = heads[stage1]
    for start in range(0, 64, max(rows, 16)):
        Hs = H[start:start + rows]
        gs = {k: g[k][start:start + rows] for k in g.files}
        _reference_rows(fh, gs, Hs, stage1)
        check_greedy_rows(fh, Hs, fh.get_next_token_batched(Hs).cpu().numpy(),
                          fh.top_clusters_batched(Hs).cpu().numpy())


@pytest.mark.parametrize("stage1", ["model", "fp8"])
def test_config_c_256_rows_vs_reference(stage1):
    """Llama-3.1-8B-shaped head (D=4096): 256 rows against the reference,
    and 1 / 32 / 256 rows against the oracle on the kernels' own data."""
    head, H, meta = _regenerate("config_c_batch")
    g = load_golden("config_c_batch")
    fh = build_head(head.weight, head.centroids, head.assignments, meta["shape"]["n_probes"],
                    stage1=stage1)
    del head
    H = H.cuda()
    mean_rec, min_rec, probes, toks = _reference_rows(fh, g, H, stage1)
    print(f"config C {stage1} stage 1: reference probe recall mean {mean_rec:.4f} "
          f"min {min_rec:.4f}")
    assert mean_rec >= (0.99 if stage1 == "model" else 0.95)
    check_greedy_rows(fh, H, toks, probes)
    for rows in (1, 32):
        Hs = H[:rows]
        check_greedy_rows(fh, Hs, fh.get_next_token_batched(Hs).cpu().numpy(),
                          fh.top_clusters_batched(Hs).cpu().numpy())


def _assert_same_ids(ids, want, H, W, slot, sampled, what):
    """Shards and the unsharded head sum the stage-1 partials of different
    hidden-dimension splits, so fp32 scores may differ in the last bits: ids
    must agree on at least 99 % of the rows, and a differing greedy token must
    be a logit near-tie (1e-3 relative, float64 logits of both tokens)."""
    diff = torch.nonzero(ids != want).view(-1).tolist()
    assert len(diff) <= max(1, ids.numel() // 100), (what, diff)
    if not sampled:
        for r in diff:
            a, b = (float(W[slot[int(t[r])]].double() @ H[r].double()) for t in (ids, want))
            assert abs(a - b) <= 1e-3 * max(abs(a), abs(b)), (what, r, a, b)


@pytest.mark.parametrize("stage1", ["model", "fp8"])
def test_config_e_shards_reproduce_unsharded(stage1):
    """Llama-3.1-70B-shaped head (D=8192, K=8016, p=256), 256 rows: the
    cluster-partitioned shards of R = 2, 4, 8 ranks (run one after another on
    this GPU, the exchange done with torch ops) give the unsharded head's ids,
    greedy and sampled (up to fp32 near-ties, see _assert_same_ids), and the
    unsharded ids pass the oracle."""
    from flash_head.native import NativeHead, derive_buffers, shard_buffers
    from flash_head.synthetic import LLAMA31_70B, make_head, make_hidden
    from flash_head.tp import cluster_range
    head = make_head(LLAMA31_70B, seed=7, device="cuda")
    fh = build_head(head.weight, head.centroids, head.assignments, LLAMA31_70B.n_probes,
                    stage1=stage1)
    del head
    torch.cuda.empty_cache()
    H = make_hidden(256, fh._D, seed=33, device="cuda")
    whole = fh.get_next_token_batched(H)
    whole_s = fh.get_next_token_batched(H, do_sample=True, temperature=0.8, seed=5, offset=1)
    full = derive_buffers(fh.w_perm, fh.vocab_maps, fh.cluster_linear.weight, fh.centroids,
                          fh.special_token_ids_tensor, stage1)
    W = fh.w_perm.view(-1, fh._D)
    vm = fh.vocab_maps.view(-1)
    slot = torch.empty_like(vm)
    slot[vm] = torch.arange(vm.numel(), device=vm.device)
    for world in (2, 4, 8):
        shards = []
        for r in range(world):
            lo, hi = cluster_range(fh._K, world, r)
            shards.append(NativeHead(shard_buffers(full, fh._cap, lo, hi), fh._D, fh._cap,
                                     fh.n_probes, cluster_base=lo))
        for kw, want in ((dict(do_sample=False), whole),
                         (dict(do_sample=True, temperature=0.8, seed=5, offset=1), whole_s)):
            cands = torch.stack([sh.tp_local_candidates(H, **kw) for sh in shards])
            bests = torch.stack([sh.tp_select_and_score(H, cands, world, **kw) for sh in shards])
            ids = NativeHead.tp_finalize(bests.max(dim=0).values)
            _assert_same_ids(ids, want, H, W, slot, kw["do_sample"], (world, kw))
        del shards
    del full
    torch.cuda.empty_cache()
    rows = torch.arange(0, 256, 8, device="cuda")
    check_greedy_rows(fh, H[rows], whole[rows].cpu().numpy(),
                      fh.top_clusters_batched(H[rows]).cpu().numpy())
