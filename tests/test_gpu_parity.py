"""Parity of the sm_100a kernels (through the C ABI) with the oracle and with
the reference's golden outputs.

Tolerance rule (the reference's, stated for bf16 logits): greedy ids must be
identical unless the competing logits are within 1e-2 relative; probe sets
identical unless the differing clusters' scores are within 1e-2 of the p-th
score; sampling distribution-equivalent (chi-squared). Against the oracle run
on the kernels' own data (same fp8 / bf16 stage-1 matrix), the bar is much
tighter: scores within 1e-4 relative, probe sets identical up to
1e-4-relative near-ties, and the token the exact argmax of the kernel's own
candidates up to 1e-5-relative logit ties.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden, load_golden_meta
from headutil import RTOL, OracleView, build_head, check_greedy_rows, to_np_f32
from oracle import flashhead_oracle as O

pytestmark = pytest.mark.gpu


def _small(golden_small, stage1, specials=None, dtype=torch.bfloat16):
    g = golden_small
    W = torch.from_numpy(g["weight_bits"].view(np.int16)).view(torch.bfloat16)
    fh = build_head(W, torch.from_numpy(g["centroids"]), torch.from_numpy(g["assignments"]),
                    int(g["n_probes"]), specials=specials, stage1=stage1, dtype=dtype)
    H = torch.from_numpy(g["hidden_bits"].view(np.int16)).view(torch.bfloat16).cuda().to(dtype)
    return fh, H


# ---------------------------------------------------------------------------
# Small golden head (D=64, V=2048, K=128, p=8)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("stage1", ["model", "fp8"])
def test_small_scores_probes_tokens(golden_small, stage1):
    fh, H = _small(golden_small, stage1)
    probes, scores = fh.top_clusters_batched(H, return_scores=True)
    ov = OracleView(fh)
    S = ov.scores(to_np_f32(H))
    got = scores.double().cpu().numpy()
    assert np.all(np.abs(got - S) <= 1e-4 * np.abs(S).max(axis=1, keepdims=True) + 1e-7)
    toks = fh.get_next_token_batched(H).cpu().numpy()
    check_greedy_rows(fh, H, toks, probes.cpu().numpy())
    # probes come back sorted, unique, in range
    pr = probes.cpu().numpy()
    assert np.all(np.diff(pr, axis=1) > 0) and pr.min() >= 0 and pr.max() < fh._K


def test_small_matches_reference_greedy(golden_small):
    """bf16 stage 1 (the reference's format): tokens and probes vs the reference."""
    g = golden_small
    fh, H = _small(g, "model")
    ov = OracleView(fh)
    Hn = to_np_f32(H)
    S = ov.scores(Hn)
    probes = fh.top_clusters_batched(H).cpu().numpy()
    toks = fh.get_next_token_batched(H).cpu().numpy()
    for r in range(H.shape[0]):
        assert O.probe_set_within_tolerance(probes[r], g["ref_probes"][r], S[r], RTOL), r
        assert O.token_within_tolerance(toks[r], g["ref_tok_greedy"][r],
                                        lambda v: ov.logit(Hn[r], v), RTOL), r
    # reference-shaped API: [1, T, D] -> [T, 1]; [B>10, 1, D] -> dense [B, 1]
    out = fh.get_next_token(H.view(1, -1, H.shape[1]))
    assert out.shape == (H.shape[0], 1) and np.array_equal(out.view(-1).cpu().numpy(), toks)
    dense = fh.get_next_token(H.view(H.shape[0], 1, -1)).view(-1).cpu().numpy()
    for r in range(H.shape[0]):
        assert O.token_within_tolerance(dense[r], g["ref_tok_dense"][r],
                                        lambda v: ov.logit(Hn[r], v), RTOL), r
        assert dense[r] == O.dense_argmax(Hn[r], ov.W) or abs(
            ov.logit(Hn[r], dense[r]) - ov.logit(Hn[r], O.dense_argmax(Hn[r], ov.W))) < 1e-6


def test_small_special_tokens(golden_small):
    g = golden_small
    fh, H = _small(g, "model", specials=g["specials"].tolist())
    ov = OracleView(fh)
    Hn = to_np_f32(H)
    toks = fh.get_next_token_batched(H).cpu().numpy()
    probes = fh.top_clusters_batched(H).cpu().numpy()
    for r in range(H.shape[0]):
        want = ov.greedy_given_probes(Hn[r], probes[r])
        assert O.token_within_tolerance(toks[r], want, lambda v: ov.logit(Hn[r], v), 1e-5)
        assert O.token_within_tolerance(toks[r], g["ref_tok_special"][r],
                                        lambda v: ov.logit(Hn[r], v), RTOL), r
    # special tokens are scored even when their cluster is not probed: with
    # probe lists that exclude its cluster, h = 50 * W[sp] must still pick sp
    sp = int(g["specials"][1])
    cl = int(np.nonzero(ov.vm == sp)[0][0])
    others = [c for c in range(fh._K) if c != cl][:fh.n_probes]
    pr = torch.tensor([others], dtype=torch.int32, device="cuda")
    h = torch.from_numpy(ov.W[sp] * 50).to("cuda", torch.bfloat16).view(1, -1)
    assert int(fh.native().stage2_next_token(h, pr)[0]) == sp
    plain, _ = _small(g, "model")
    assert int(plain.native().stage2_next_token(h, pr)[0]) != sp


def test_fp16_head(golden_small):
    fh, H = _small(golden_small, "model", dtype=torch.float16)
    toks = fh.get_next_token_batched(H).cpu().numpy()
    check_greedy_rows(fh, H, toks, fh.top_clusters_batched(H).cpu().numpy())
    fh8, _ = _small(golden_small, "fp8", dtype=torch.float16)
    toks8 = fh8.get_next_token_batched(H).cpu().numpy()
    check_greedy_rows(fh8, H, toks8, fh8.top_clusters_batched(H).cpu().numpy())


# ---------------------------------------------------------------------------
# Full-size heads
# ---------------------------------------------------------------------------

@pytest.fixture(scope="module")
def llama1b_heads(config_a_head):
    head, meta = config_a_head
    p = meta["shape"]["n_probes"]
    return {s: build_head(head.weight, head.centroids, head.assignments, p, stage1=s)
            for s in ("model", "fp8")}


@pytest.mark.parametrize("stage1", ["model", "fp8"])
def test_config_a_matches_reference(llama1b_heads, stage1):
    """Llama-3.2-1B-shaped head: kernel tokens vs the reference's greedy tokens."""
    g = load_golden("config_a")
    fh = llama1b_heads[stage1]
    H = torch.from_numpy(g["hidden_bits"].view(np.int16)).view(torch.bfloat16).cuda()
    toks = fh.get_next_token_batched(H).cpu().numpy()
    probes = fh.top_clusters_batched(H).cpu().numpy()
    ov = check_greedy_rows(fh, H, toks, probes)
    Hn = to_np_f32(H)
    ref_scores = O.cluster_scores(Hn, O.bf16_bits_to_f32(
        O.f32_to_bf16_bits(O.normalized_cluster_weight(to_np_f32(fh.centroids)))))
    for r in range(H.shape[0]):
        assert O.token_within_tolerance(toks[r], g["ref_tok_greedy"][r],
                                        lambda v: ov.logit(Hn[r], v), RTOL), r
        if stage1 == "model":
            assert O.probe_set_within_tolerance(probes[r], g["ref_probes"][r], ref_scores[r], RTOL)


@pytest.mark.parametrize("rows", [1, 8, 64, 256])
def test_config_b_batch_sweep(llama1b_heads, rows):
    """fp8 stage 1, batch 1/8/64/256 of N(0, 0.25) hidden states."""
    from flash_head.synthetic import make_hidden
    fh = llama1b_heads["fp8"]
    H = make_hidden(rows, fh._D, seed=100 + rows, device="cuda")
    toks = fh.get_next_token_batched(H).cpu().numpy()
    probes = fh.top_clusters_batched(H).cpu().numpy()
    check_greedy_rows(fh, H, toks, probes)


@pytest.mark.parametrize("stage1", ["model", "fp8"])
def test_config_c_llama8b(stage1):
    from flash_head.synthetic import LLAMA31_8B, make_head, make_hidden
    head = make_head(LLAMA31_8B, seed=5, device="cuda")
    fh = build_head(head.weight, head.centroids, head.assignments, 256, stage1=stage1)
    del head
    for rows in (1, 32):
        H = make_hidden(rows, fh._D, seed=200 + rows, device="cuda")
        toks = fh.get_next_token_batched(H).cpu().numpy()
        check_greedy_rows(fh, H, toks, fh.top_clusters_batched(H).cpu().numpy())


# ---------------------------------------------------------------------------
# Stateless kernels with the reference's signatures (fused.py)
# ---------------------------------------------------------------------------

def test_fused_mirrors(golden_small):
    from flash_head import fused
    fh, H = _small(golden_small, "model")
    ov = OracleView(fh)
    Hn = to_np_f32(H)
    T, K, cap = H.shape[0], fh._K, fh._cap
    gen = torch.Generator().manual_seed(3)
    ci = torch.randint(0, K, (T, 12), generator=gen).cuda()
    ci[:, 3] = ci[:, 2]  # duplicate probes are allowed
    w_flat = fh.w_perm.view(-1)
    vm_flat = fh.vocab_maps.view(-1)
    logits = fused.block_sparse_logits(H, w_flat, ci, K, cap)
    assert logits.shape == (T, 12 * cap) and logits.dtype == H.dtype
    want = np.einsum("tpcd,td->tpc", ov.w_perm[ci.cpu().numpy()], Hn.astype(np.float64))
    got = logits.float().view(T, 12, cap).cpu().numpy()
    assert np.all(np.abs(got - want) <= 2.0 ** -8 * np.abs(want) + 1e-6)
    mx, vid = fused.block_sparse_logits_argmax(H, w_flat, ci, vm_flat, K, cap)
    assert mx.shape == (T, 12) and vid.dtype == torch.int64
    best_slot = want.argmax(axis=2)
    assert np.array_equal(vid.cpu().numpy(), np.take_along_axis(
        ov.vm[ci.cpu().numpy()], best_slot[..., None], axis=2)[..., 0])
    out = fused.block_sparse_argmax_atomic(H, w_flat, ci, vm_flat, K, cap)
    assert out.shape == (T, 1)
    for t in range(T):
        vids, lg = O.candidate_logits(Hn[t], ov.w_perm, ov.vm, ci[t].cpu().numpy())
        assert int(out[t, 0]) == O.argmax_smallest_id(vids, lg)[0]
    # out-of-range cluster ids are skipped; a row with none left gets the
    # reference's unpacked sentinel
    bad = ci.clone()
    bad[0, :] = K + 5
    bad[1, 0] = -1
    out2 = fused.block_sparse_argmax_atomic(H, w_flat, bad, vm_flat, K, cap)
    assert int(out2[0, 0]) == 0xFFFFFFFF
    vids, lg = O.candidate_logits(Hn[1], ov.w_perm, ov.vm, ci[1, 1:].cpu().numpy())
    assert int(out2[1, 0]) == O.argmax_smallest_id(vids, lg)[0]
    with pytest.raises(AssertionError):
        fused.block_sparse_argmax_atomic(H, w_flat, ci.int(), vm_flat, K, cap)


# ---------------------------------------------------------------------------
# Edge cases
# ---------------------------------------------------------------------------

def _tiny_head(K, cap, D, seed=0, dup_centroids=False):
    from flash_head.synthetic import HeadShape, make_head
    head = make_head(HeadShape(hidden=D, vocab=K * cap, n_clusters=K, cluster_size=cap), seed=seed)
    if dup_centroids:
        head.centroids[:, 1::2] = head.centroids[:, 0::2][:, :head.centroids[:, 1::2].shape[1]]
    return head


@pytest.mark.parametrize("K,cap,D,p", [(100, 16, 16, 1), (100, 16, 16, 100), (37, 4, 48, 5),
                                       (513, 32, 272, 40), (4096, 2, 64, 4096),
                                       (16384, 16, 32, 256)])
@pytest.mark.parametrize("stage1", ["model", "fp8"])
def test_shapes(K, cap, D, p, stage1):
    from flash_head.synthetic import make_hidden
    head = _tiny_head(K, cap, D)
    fh = build_head(head.weight, head.centroids, head.assignments, p, stage1=stage1)
    H = make_hidden(5, D, seed=9, device="cuda")
    toks = fh.get_next_token_batched(H).cpu().numpy()
    check_greedy_rows(fh, H, toks, fh.top_clusters_batched(H).cpu().numpy())
    assert fh.get_next_token_batched(H[:0]).numel() == 0


def test_tied_scores_pick_smaller_cluster_ids():
    """Clusters 2k and 2k+1 share a centroid, so every score is tied with its
    neighbour's; the selection must keep the smaller id of each tied pair."""
    from flash_head.synthetic import make_hidden
    head = _tiny_head(64, 16, 64, dup_centroids=True)
    fh = build_head(head.weight, head.centroids, head.assignments, 5, stage1="model")
    H = make_hidden(16, 64, seed=4, device="cuda")
    probes, scores = fh.top_clusters_batched(H, return_scores=True)
    s = scores.cpu().numpy()
    for r in range(16):
        assert np.array_equal(probes[r].cpu().numpy(), O.top_probes(s[r], 5))
        assert (probes[r] % 2 == 0).sum() >= 3


def test_cuda_graph_replay(llama1b_heads):
    from flash_head.synthetic import make_hidden
    fh = llama1b_heads["fp8"]
    fh.prepare(8)
    H = make_hidden(8, fh._D, seed=77, device="cuda")
    out = torch.empty(8, dtype=torch.int64, device="cuda")
    eager = fh.get_next_token_batched(H).clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fh.get_next_token_batched(H, out=out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fh.get_next_token_batched(H, out=out)
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    H2 = make_hidden(8, fh._D, seed=78, device="cuda")
    H.copy_(H2)
    g.replay()
    assert torch.equal(out, fh.get_next_token_batched(H2))


# ---------------------------------------------------------------------------
# Sampling
# ---------------------------------------------------------------------------

def test_sampling_matches_oracle_draw_for_draw(golden_small):
    """Same Philox stream as the oracle: identical draws except near-ties."""
    fh, H = _small(golden_small, "model")
    ov = OracleView(fh)
    h = O.bf16_round(to_np_f32(H[:1]) * 20)
    n = 400
    Ht = torch.from_numpy(np.repeat(h, n, axis=0)).to("cuda", torch.bfloat16)
    toks = fh.get_next_token_batched(Ht, do_sample=True, temperature=0.8, seed=1234,
                                     offset=7).cpu().numpy()
    cd = ov.sw * (ov.sscale[:, None] if ov.sscale is not None else 1.0)
    agree = sum(O.sample_token(h[0], ov.w_perm, ov.vm, cd, ov.p, 0.8, 1234, 7, r)[0] == toks[r]
                for r in range(n))
    assert agree >= 0.98 * n
    again = fh.get_next_token_batched(Ht, do_sample=True, temperature=0.8, seed=1234, offset=7)
    assert np.array_equal(again.cpu().numpy(), toks)
    other = fh.get_next_token_batched(Ht, do_sample=True, temperature=0.8, seed=1234, offset=8)
    assert not np.array_equal(other.cpu().numpy(), toks)


def _draws(fh, h_row: torch.Tensor, n: int, temperature: float, seed: int, chunk: int = 8192):
    counts = np.zeros(fh._K * fh._cap, dtype=np.int64)
    done = 0
    while done < n:
        m = min(chunk, n - done)
        toks = fh.get_next_token_batched(h_row.view(1, -1).expand(m, -1).contiguous(),
                                         do_sample=True, temperature=temperature, seed=seed,
                                         offset=done)
        counts += np.bincount(toks.cpu().numpy(), minlength=counts.size)
        done += m
    return counts


@pytest.mark.parametrize("stage1", ["model", "fp8"])
def test_sampling_distribution_small(golden_small, stage1):
    g = load_golden("small_sample")
    fh, _ = _small(golden_small, stage1)
    H = torch.from_numpy(g["hidden_bits"].view(np.int16)).view(torch.bfloat16).cuda()
    for r in range(2):
        ours = _draws(fh, H[r], 40000, float(g["temperature"]), seed=11 + r)
        stat, dof, pval = O.chi2_homogeneity(g["counts"][r], ours)
        assert pval > 1e-4, (r, stat, dof, pval)


@pytest.mark.parametrize("stage1", ["model", "fp8"])
def test_sampling_distribution_qwen_1e5(stage1):
    """Qwen2.5-1.5B-shaped head, T=0.8: 1e5 reference draws vs 1e5 of ours."""
    from flash_head.synthetic import HeadShape, head_checksum, make_head
    meta = load_golden_meta("config_d_sample")
    g = load_golden("config_d_sample")
    shape = HeadShape(**meta["shape"])
    head = make_head(shape, seed=meta["head_seed"])
    assert np.allclose(head_checksum(head), meta["checksum"], rtol=0, atol=0)
    fh = build_head(head.weight, head.centroids, head.assignments, shape.n_probes, stage1=stage1)
    H = torch.from_numpy(g["hidden_bits"].view(np.int16)).view(torch.bfloat16).cuda()
    n = int(g["draws_per_row"])
    for r in range(2):
        ref = np.zeros(shape.vocab, dtype=np.int64)
        ref[g[f"ids{r}"]] = g[f"counts{r}"]
        ours = _draws(fh, H[r], n, float(g["temperature"]), seed=500 + r)
        stat, dof, pval = O.chi2_homogeneity(ref, ours)
        assert dof > 50 and pval > 1e-4, (r, stat, dof, pval)
        # marginal cluster-inclusion frequencies agree too (coarser bins)
        assign = head.assignments.numpy()
        cr = np.bincount(assign, weights=ref, minlength=shape.n_clusters)
        co = np.bincount(assign, weights=ours, minlength=shape.n_clusters)
        assert O.chi2_homogeneity(cr, co)[2] > 1e-4


# ---------------------------------------------------------------------------
# Tensor-parallel steps, emulated on one GPU (ranks run one after another;
# no kernel waits on another)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("do_sample", [False, True])
@pytest.mark.parametrize("rows", [6, 16])
def test_tp_shards_reproduce_unsharded(llama1b_heads, world, do_sample, rows):
    """6 rows score the owned probes with the streamed few-row stage 2, 16
    rows with the cluster-major tensor-core stage 2."""
    from flash_head.native import NativeHead, derive_buffers, shard_buffers
    from flash_head.synthetic import make_hidden
    from flash_head.tp import cluster_range
    fh = llama1b_heads["fp8"]
    full = derive_buffers(fh.w_perm, fh.vocab_maps, fh.cluster_linear.weight, fh.centroids,
                          fh.special_token_ids_tensor, "fp8")
    shards = []
    for r in range(world):
        lo, hi = cluster_range(fh._K, world, r)
        shards.append(NativeHead(shard_buffers(full, fh._cap, lo, hi), fh._D, fh._cap,
                                 fh.n_probes, cluster_base=lo))
    H = make_hidden(rows, fh._D, seed=31, device="cuda")
    kw = dict(do_sample=do_sample, temperature=0.8, seed=99, offset=3)
    cands = torch.stack([sh.tp_local_candidates(H, **kw) for sh in shards])
    bests = torch.stack([sh.tp_select_and_score(H, cands, world, **kw) for sh in shards])
    ids = NativeHead.tp_finalize(bests.max(dim=0).values)
    whole = fh.get_next_token_batched(H, do_sample=do_sample, temperature=0.8, seed=99, offset=3)
    # shards split the hidden dimension of stage 1 differently from the whole
    # head (fp32 sums in another order): at most one near-tie row may differ
    assert int((ids != whole).sum()) <= 1, (ids, whole)


def test_host_buffer_entry_point(llama1b_heads):
    """fh_get_next_token_host (pinned host in, host ids out, synchronised on
    return) gives the ids of fh_get_next_token on the same rows."""
    from flash_head.synthetic import make_hidden
    nh = llama1b_heads["fp8"].native()
    for rows in (1, 3, 7, 20):
        H = make_hidden(rows, nh.D, seed=800 + rows)
        want = nh.next_token(H.to("cuda")).cpu()
        got = nh.next_token_host(H.pin_memory())
        assert got.device.type == "cpu" and torch.equal(got, want), rows
        paged = nh.next_token_host(H.clone(), out_host=torch.empty(rows, dtype=torch.int64))
        assert torch.equal(paged, want), rows  # pageable buffers work too (synchronous copies)
    assert nh.next_token_host(H[:0]).numel() == 0


def test_host_buffer_entry_point_reused_buffers(llama1b_heads):
    """Repeated calls on the same page-locked buffers (read and written by
    the kernels directly) see the buffers' current contents every time, for
    the one-kernel, three-kernel and batched paths; pageable buffers in
    between change nothing."""
    from flash_head.synthetic import make_hidden
    nh = llama1b_heads["fp8"].native()
    for rows in (1, 7, 20):
        hbuf = torch.empty(rows, nh.D, dtype=torch.bfloat16).pin_memory()
        obuf = torch.empty(rows, dtype=torch.int64).pin_memory()
        for i in range(5):
            H = make_hidden(rows, nh.D, seed=950 + 10 * rows + i)
            hbuf.copy_(H)
            got = nh.next_token_host(hbuf, out_host=obuf)
            want = nh.next_token(H.to("cuda")).cpu()
            assert got.data_ptr() == obuf.data_ptr() and torch.equal(got, want), (rows, i)
            if i == 2:
                paged = nh.next_token_host(H.clone(), out_host=torch.empty(rows, dtype=torch.int64))
                assert torch.equal(paged, want), rows
    assert nh.workspace_error() == 0


def _oracle_candidate_logprobs(ov, h, probes, tok):
    """float64 log-softmax over one row's candidates (probed clusters, special
    tokens, and the given token when it is not among them)."""
    vids, logits = O.candidate_logits(h, ov.w_perm, ov.vm, probes, ov.specials)
    if tok not in set(vids.tolist()):
        vids = np.append(vids, tok)
        logits = np.append(logits, ov.logit(h, tok))
    m = logits.max()
    lp = logits - (m + np.log(np.exp(logits - m).sum()))
    return dict(zip(vids.tolist(), lp.tolist()))


@pytest.mark.parametrize("which,rows", [("llama", 1), ("llama", 6), ("specials", 5)])
def test_candidate_logprobs_match_the_oracle(llama1b_heads, which, rows):
    """FlashHead.candidate_logprobs (the sampler hook's logprobs): per row the
    given token's logprob, the top-k ids and values and the token's rank agree
    with the oracle's float64 log-softmax over the same candidate set (the
    kernel's own probes, the special tokens and the token) within 2e-2 (logits
    rounded to bf16). Even rows ask for the greedy token (rank 1), odd rows
    for a token of an unprobed cluster."""
    from flash_head.synthetic import HeadShape, make_head, make_hidden
    if which == "llama":
        fh = llama1b_heads["fp8"]
    else:
        head = make_head(HeadShape(hidden=256, vocab=4800, n_clusters=300, n_probes=24), seed=4)
        fh = build_head(head.weight, head.centroids, head.assignments, 24,
                        specials=[0, 5, 4799], stage1="model")
    nh = fh.native()
    ov = OracleView(fh)
    H = make_hidden(rows, fh._D, seed=1500 + rows, device="cuda")
    Hn = to_np_f32(H)
    probes = nh.top_clusters(H).cpu().numpy()
    greedy = nh.next_token(H).cpu().numpy()
    toks = []
    for r in range(rows):
        if r % 2 == 0:
            toks.append(int(greedy[r]))
        else:
            c = next(c for c in range(ov.K) if c not in set(probes[r].tolist()))
            toks.append(int(ov.vm[c, 0]))
    k, tol = 5, 2e-2
    ids, lps, ranks = fh.candidate_logprobs(H, torch.tensor(toks), k)
    assert ids.shape == (rows, k + 1) and ids.dtype == torch.int32 and lps.dtype == torch.float32
    ids, lps, ranks = ids.cpu().numpy(), lps.cpu().numpy(), ranks.cpu().numpy()
    for r in range(rows):
        want = _oracle_candidate_logprobs(ov, Hn[r], probes[r], toks[r])
        assert ids[r, 0] == toks[r] and abs(lps[r, 0] - want[toks[r]]) <= tol, r
        best = sorted(want.values(), reverse=True)
        assert list(lps[r, 1:]) == sorted(lps[r, 1:], reverse=True), r
        for j in range(1, k + 1):
            assert abs(lps[r, j] - want[int(ids[r, j])]) <= tol, (r, j)
            assert lps[r, j] >= best[j - 1] - tol, (r, j)
        t = want[toks[r]]
        lo = sum(v >= t + tol for v in want.values())
        hi = sum(v >= t - tol for v in want.values())
        assert lo <= ranks[r] <= hi, (r, ranks[r], lo, hi)
        if r % 2 == 0 and hi == 1:
            assert ranks[r] == 1


@pytest.mark.parametrize("batch,max_spec", [(1, 1), (37, 5), (64, 33), (9, 128)])
def test_spec_accept_matches_the_oracle(batch, max_spec):
    """Draft acceptance on the device (fh_spec_accept) equals the oracle's
    restatement of the reference's loop, bit for bit: random draft counts
    0..max (rows without drafts included), drafts matching the target with
    probability 0.9 per position, lengths beyond one warp's 32 lanes."""
    from flash_head.spec import accept_draft_tokens
    rng = np.random.default_rng(batch * 1000 + max_spec)
    num = rng.integers(0, max_spec + 1, size=batch)
    num[0] = max_spec
    T = int(num.sum())
    target = rng.integers(0, 128256, size=T).astype(np.int32)
    draft = np.where(rng.random(T) < 0.9, target, rng.integers(0, 128256, size=T)).astype(np.int32)
    bonus = rng.integers(0, 128256, size=batch).astype(np.int32)
    cu = np.cumsum(num).astype(np.int32)
    out = accept_draft_tokens(torch.from_numpy(draft).cuda(), torch.from_numpy(target).cuda(),
                              torch.from_numpy(bonus).cuda(), torch.from_numpy(cu).cuda(),
                              max_spec)
    want = O.spec_accept(draft, target, bonus, num.tolist(), max_spec)
    assert out.dtype == torch.int32 and np.array_equal(out.cpu().numpy(), want)
    # no drafts at all: every row is its bonus token
    none = accept_draft_tokens(torch.empty(0, dtype=torch.int32, device="cuda"),
                               torch.empty(0, dtype=torch.int32, device="cuda"),
                               torch.from_numpy(bonus).cuda(),
                               torch.zeros(batch, dtype=torch.int32, device="cuda"), 0)
    assert none.view(-1).cpu().tolist() == bonus.tolist()


def test_workspace_reuse_across_row_counts(llama1b_heads):
    """One workspace serves calls with any row count: stage 2 alone (which
    relies on the accumulator left zeroed by earlier calls) matches the full
    step whatever row counts ran before it."""
    from flash_head.synthetic import make_hidden
    nh = llama1b_heads["fp8"].native()
    for i, rows in enumerate((64, 1, 17, 3, 64, 2, 1)):
        H = make_hidden(rows, nh.D, seed=600 + i, device="cuda")
        probes = nh.top_clusters(H)
        a = nh.stage2_next_token(H, probes)
        b = nh.next_token(H)
        assert torch.equal(a, b), rows


# ---------------------------------------------------------------------------
# The one-kernel step (rows <= 4) against the oracle and the three-kernel path
# ---------------------------------------------------------------------------

def _native_pair(fh):
    """The head's NativeHead and a twin that always takes the three-kernel path."""
    from flash_head import _lib
    from flash_head.native import NativeHead
    nh = fh.native()
    twin = NativeHead(nh.bufs, nh.D, nh.cap, nh.p, flags=_lib.FH_FLAG_NO_FUSED)
    return nh, twin


@pytest.mark.parametrize("rows", [1, 2, 3, 4])
@pytest.mark.parametrize("stage1", ["model", "fp8"])
def test_fused_step_matches_oracle(llama1b_heads, rows, stage1):
    from flash_head.synthetic import make_hidden
    fh = llama1b_heads[stage1]
    nh, twin = _native_pair(fh)
    for seed in range(3):
        H = make_hidden(rows, fh._D, seed=700 + 10 * rows + seed, device="cuda")
        fused = nh.next_token(H).cpu().numpy()
        three = twin.next_token(H).cpu().numpy()
        probes = nh.top_clusters(H).cpu().numpy()
        check_greedy_rows(fh, H, fused, probes)
        check_greedy_rows(fh, H, three, probes)
    assert nh.workspace_error() == 0


@pytest.mark.parametrize("K,cap,D,p", [(100, 16, 512, 1), (100, 16, 512, 100), (37, 4, 1024, 5),
                                       (513, 8, 256, 40), (16384, 16, 512, 256),
                                       (300, 16, 4096, 64)])
def test_fused_step_shapes(K, cap, D, p):
    from flash_head.synthetic import make_hidden
    head = _tiny_head(K, cap, D)
    for stage1 in ("model", "fp8"):
        fh = build_head(head.weight, head.centroids, head.assignments, p, stage1=stage1)
        nh, _ = _native_pair(fh)
        for rows in (1, 3):
            H = make_hidden(rows, D, seed=9 + rows, device="cuda")
            toks = nh.next_token(H).cpu().numpy()
            check_greedy_rows(fh, H, toks, nh.top_clusters(H).cpu().numpy())
        assert nh.workspace_error() == 0


def test_fused_step_bucket_larger_than_tie_list(llama1b_heads):
    """A zero hidden row ties all 8016 cluster scores in one bf16 bucket, far
    more keys than the one-kernel step's 1024-entry tie list: the bucket is
    ranked against the scores row instead, so the probes are clusters 0..p-1
    (equal scores, smallest ids first) and the token is the smallest vocab id
    among them, exactly as the oracle and the three-kernel path pick it."""
    from flash_head.synthetic import make_hidden
    fh = llama1b_heads["fp8"]
    nh, twin = _native_pair(fh)
    ov = OracleView(fh)
    H = make_hidden(2, fh._D, seed=123, device="cuda")
    H[0].zero_()
    fused = nh.next_token(H).cpu().numpy()
    three = twin.next_token(H).cpu().numpy()
    want0 = ov.greedy_given_probes(np.zeros(fh._D, np.float32), np.arange(fh.n_probes))
    assert fused[0] == three[0] == want0
    check_greedy_rows(fh, H[1:], fused[1:], nh.top_clusters(H[1:]).cpu().numpy())
    assert nh.workspace_error() == 0


def test_fused_step_special_tokens(golden_small):
    """Fused path (D=64 is below its minimum, so use a D=512 head) with specials."""
    from flash_head.synthetic import make_hidden
    head = _tiny_head(256, 16, 512, seed=3)
    specials = [0, 17, 4095]
    fh = build_head(head.weight, head.centroids, head.assignments, 12, specials=specials,
                    stage1="model")
    nh, twin = _native_pair(fh)
    ov = OracleView(fh)
    for rows in (1, 2, 4):
        H = make_hidden(rows, 512, seed=40 + rows, device="cuda")
        Hn = to_np_f32(H)
        probes = nh.top_clusters(H).cpu().numpy()
        toks = nh.next_token(H).cpu().numpy()
        for r in range(rows):
            want = ov.greedy_given_probes(Hn[r], probes[r])
            assert O.token_within_tolerance(toks[r], want, lambda v: ov.logit(Hn[r], v), 1e-5)
    # a special token far outside the probed clusters still wins
    sp = 4095
    h = torch.from_numpy(ov.W[sp] * 50).to("cuda", torch.bfloat16).view(1, -1)
    assert int(nh.next_token(h)[0]) == int(twin.next_token(h)[0])


@pytest.mark.parametrize("stage1", ["model", "fp8"])
def test_fused_sampling_matches_oracle_draw_for_draw(golden_small, stage1):
    from flash_head.synthetic import make_hidden
    head = _tiny_head(256, 16, 512, seed=8)
    fh = build_head(head.weight, head.centroids, head.assignments, 12, stage1=stage1)
    nh, _ = _native_pair(fh)
    ov = OracleView(fh)
    h = make_hidden(1, 512, seed=5, device="cuda", std=4.0)
    hn = to_np_f32(h)[0]
    cd = ov.sw * (ov.sscale[:, None] if ov.sscale is not None else 1.0)
    n, agree = 300, 0
    for off in range(n):
        tok = int(nh.next_token(h, do_sample=True, temperature=0.7, seed=77, offset=off)[0])
        agree += tok == O.sample_token(hn, ov.w_perm, ov.vm, cd, ov.p, 0.7, 77, off, 0)[0]
    assert agree >= 0.98 * n


def test_fused_barrier_timeout_is_reported_not_hung():
    """The grid barrier of the one-kernel step waits with a poll limit. In the
    test mode it waits for one CTA more than it launched: the wait must run
    out, set error bit 0 in the workspace, and the kernel must still finish,
    leaving the context and the workspace usable."""
    from flash_head import _lib
    from flash_head.native import NativeHead
    from flash_head.synthetic import make_hidden
    head = _tiny_head(300, 16, 512, seed=2)
    fh = build_head(head.weight, head.centroids, head.assignments, 16, stage1="fp8")
    nh = fh.native()
    bad = NativeHead(nh.bufs, nh.D, nh.cap, nh.p, flags=_lib.FH_FLAG_TEST_TIMEOUT)
    H = make_hidden(1, 512, seed=1, device="cuda")
    bad.next_token(H)
    torch.cuda.synchronize()
    assert bad.workspace_error() & 1
    assert bad.workspace_error() == 0  # cleared by the read
    # the timed-out workspace, reused by the normal head: correct results
    nh._ws = dict(bad._ws)
    toks = nh.next_token(H).cpu().numpy()
    check_greedy_rows(fh, H, toks, nh.top_clusters(H).cpu().numpy())
    assert nh.workspace_error() == 0
