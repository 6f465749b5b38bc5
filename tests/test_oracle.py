"""The oracle pinned against the reference's own outputs (golden vectors).

The golden vectors were produced by running the reference FlashHead on CPU
(tests/golden/make_golden.py). Two oracles are checked:
  * oracle.reference_cpu - torch op-for-op port of the reference's CPU path:
    must reproduce the reference BIT-EXACTLY (same ops, same torch);
  * oracle.flashhead_oracle - numpy float64 restatement: must agree with the
    reference under the tolerance rule (ids identical unless the logits are
    within 1e-2 relative; probe sets identical unless scores are within 1e-2
    of the p-th score; sampling distribution-equivalent by chi-squared).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import flashhead_oracle as O
from oracle.reference_cpu import ReferenceHeadCPU

RTOL = 1e-2


def _port_small(golden_small, specials=None):
    g = golden_small
    W = torch.from_numpy(g["weight_bits"].view(np.int16)).view(torch.bfloat16)
    return ReferenceHeadCPU(W, torch.from_numpy(g["centroids"]),
                            torch.from_numpy(g["assignments"]), n_probes=int(g["n_probes"]),
                            special_token_ids=specials)


def _hidden(bits):
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16)


# ---------------------------------------------------------------------------
# Torch port: bit-exact with the reference
# ---------------------------------------------------------------------------

def test_port_layout_matches_reference(golden_small):
    g = golden_small
    port = _port_small(g)
    assert np.array_equal(port.vocab_maps.numpy(), g["ref_vocab_maps"])
    cw_bits = port.cluster_w.contiguous().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(cw_bits, g["ref_cluster_w_bits"])


def test_port_greedy_bit_exact(golden_small):
    g = golden_small
    port = _port_small(g)
    sp_port = _port_small(g, specials=g["specials"].tolist())
    H = _hidden(g["hidden_bits"])
    for r in range(H.shape[0]):
        x = H[r].view(1, 1, -1)
        sims = port.scores(x).view(-1).contiguous().view(torch.int16).numpy().view(np.uint16)
        assert np.array_equal(sims, g["ref_sims_bits"][r])
        assert np.array_equal(np.sort(port.top_clusters(x).view(-1).numpy()), g["ref_probes"][r])
        assert int(port.get_next_token(x, use_identical_tiebreak=True).view(-1)[0]) == \
            int(g["ref_tok_tiebreak"][r])
        assert int(sp_port.get_next_token(x).view(-1)[0]) == int(g["ref_tok_special"][r])
        logits, _, ids = port.gather_logits(x, port.top_clusters(x), False)
        assert int(ids[logits.argmax(dim=-1, keepdim=True)][0].view(-1)[0]) == \
            int(g["ref_tok_greedy"][r])
    dense = port.get_next_token(H.view(H.shape[0], 1, -1)).view(-1).numpy()
    assert np.array_equal(dense, g["ref_tok_dense"])


def test_port_config_a_bit_exact(config_a_head):
    head, meta = config_a_head
    g = load_golden("config_a")
    port = ReferenceHeadCPU(head.weight, head.centroids, head.assignments,
                            n_probes=meta["shape"]["n_probes"])
    H = _hidden(g["hidden_bits"])
    for r in range(3):
        x = H[r].view(1, 1, -1)
        assert np.array_equal(np.sort(port.top_clusters(x).view(-1).numpy()), g["ref_probes"][r])
        assert int(port.get_next_token(x, use_identical_tiebreak=True).view(-1)[0]) == \
            int(g["ref_tok_tiebreak"][r])
        logits, _, ids = port.gather_logits(x, port.top_clusters(x), False)
        assert int(ids[logits.argmax(dim=-1, keepdim=True)][0].view(-1)[0]) == \
            int(g["ref_tok_greedy"][r])


def test_reference_tiebreak_branch_is_not_the_argmax(golden_small, small_head_np):
    """Documents a defect of the reference: get_next_token(...,
    use_identical_tiebreak=True) (flash_head.py:329-333) indexes the sorted
    candidate ids with a position mapped back to the unsorted order, so it
    returns a candidate that is not the argmax. This build returns the argmax
    (ties to the smallest id) for every greedy mode, i.e. the answer of the
    reference's fused greedy kernel, and the tests compare against
    ref_tok_greedy."""
    g, s = golden_small, small_head_np
    W64 = s["W"].astype(np.float64)
    wrong = 0
    for r in range(s["H"].shape[0]):
        h = s["H"][r].astype(np.float64)
        vids, logits = O.candidate_logits(s["H"][r], s["w_perm"], s["vm"], g["ref_probes"][r])
        best = logits.max()
        tb = int(g["ref_tok_tiebreak"][r])
        wrong += (W64[tb] @ h) < best * (1 - RTOL)
        assert abs(W64[int(g["ref_tok_greedy"][r])] @ h - best) <= RTOL * abs(best)
    assert wrong >= s["H"].shape[0] // 2


# ---------------------------------------------------------------------------
# numpy oracle: tolerance rule against the reference
# ---------------------------------------------------------------------------

def test_oracle_layout(golden_small, small_head_np):
    g, s = golden_small, small_head_np
    assert np.array_equal(s["vm"], g["ref_vocab_maps"])
    assert np.array_equal(O.f32_to_bf16_bits(s["cw"]), g["ref_cluster_w_bits"])


def test_oracle_scores_and_probes(golden_small, small_head_np):
    g, s = golden_small, small_head_np
    scores = O.cluster_scores(s["H"], s["cw"])
    ref = O.bf16_bits_to_f32(g["ref_sims_bits"]).astype(np.float64)
    # the reference rounds fp32-accumulated scores to bf16 (half-ulp 2^-9)
    assert np.all(np.abs(scores - ref) <= 2.0 ** -8 * np.abs(scores) + 1e-6)
    for r in range(scores.shape[0]):
        mine = O.top_probes(scores[r], s["p"])
        assert O.probe_set_within_tolerance(mine, g["ref_probes"][r], scores[r], RTOL)


def test_oracle_greedy_tokens(golden_small, small_head_np):
    g, s = golden_small, small_head_np
    W64 = s["W"].astype(np.float64)
    for r in range(s["H"].shape[0]):
        h = s["H"][r]
        tok, _, _ = O.greedy_token(h, s["w_perm"], s["vm"], s["cw"], s["p"])
        logit = lambda v, h=h: W64[v] @ h.astype(np.float64)
        assert O.token_within_tolerance(tok, g["ref_tok_greedy"][r], logit, RTOL)
        tok_sp, _, _ = O.greedy_token(h, s["w_perm"], s["vm"], s["cw"], s["p"],
                                      special_ids=g["specials"])
        assert O.token_within_tolerance(tok_sp, g["ref_tok_special"][r], logit, RTOL)
        assert O.token_within_tolerance(O.dense_argmax(h, s["W"]), g["ref_tok_dense"][r], logit,
                                        RTOL)


def test_oracle_config_a(config_a_head):
    head, meta = config_a_head
    g = load_golden("config_a")
    W = head.weight.float().numpy()
    assign = head.assignments.numpy()
    K = meta["shape"]["n_clusters"]
    vm = O.vocab_maps_from_assignments(assign, K)
    cw = O.bf16_round(O.normalized_cluster_weight(head.centroids.numpy()))
    w_perm = O.permute_weight(W, vm)
    H = O.bf16_bits_to_f32(g["hidden_bits"])
    p = meta["shape"]["n_probes"]
    for r in range(H.shape[0]):
        tok, probes, scores = O.greedy_token(H[r], w_perm, vm, cw, p)
        assert O.probe_set_within_tolerance(probes, g["ref_probes"][r], scores, RTOL)
        logit = lambda v, h=H[r]: W[v].astype(np.float64) @ h.astype(np.float64)
        assert O.token_within_tolerance(tok, g["ref_tok_greedy"][r], logit, RTOL)


# ---------------------------------------------------------------------------
# Sampling: distribution equivalence with the reference
# ---------------------------------------------------------------------------

def _oracle_counts(s, h, draws, temperature, seed, row):
    cd = np.ascontiguousarray(s["C"].T)  # raw centroids [K, D], bf16 like the reference
    cd = O.bf16_round(cd)
    counts = np.zeros(s["W"].shape[0], dtype=np.int64)
    for i in range(draws):
        tok, _ = O.sample_token(h, s["w_perm"], s["vm"], cd, s["p"], temperature, seed, i, row)
        counts[tok] += 1
    return counts


def test_oracle_sampling_matches_reference_distribution(small_head_np):
    g = load_golden("small_sample")
    T = float(g["temperature"])
    H = O.bf16_bits_to_f32(g["hidden_bits"])
    for r in range(2):
        ours = _oracle_counts(small_head_np, H[r], 4000, T, seed=99, row=r)
        stat, dof, pval = O.chi2_homogeneity(g["counts"][r], ours)
        assert pval > 1e-4, (r, stat, dof, pval)


def test_port_sampling_matches_reference_distribution(golden_small):
    g = load_golden("small_sample")
    port = _port_small(golden_small)
    H = _hidden(g["hidden_bits"])
    torch.manual_seed(7)
    for r in range(2):
        x = H[r].view(1, 1, -1)
        ours = np.zeros(g["counts"].shape[1], dtype=np.int64)
        for _ in range(3000):
            ours[int(port.get_next_token(x, do_sample=True, temperature=float(g["temperature"]))
                     .view(-1)[0])] += 1
        _, _, pval = O.chi2_homogeneity(g["counts"][r], ours)
        assert pval > 1e-4


def test_chi2_has_power(small_head_np):
    """The test tells T=0.8 from T=1.6 on inputs whose softmax is not flat
    (hidden states scaled x40), and accepts two T=0.8 samplers."""
    g = load_golden("small_sample")
    h = O.bf16_round(O.bf16_bits_to_f32(g["hidden_bits"])[0] * 40)
    a = _oracle_counts(small_head_np, h, 3000, 0.8, seed=5, row=0)
    b = _oracle_counts(small_head_np, h, 3000, 0.8, seed=6, row=0)
    c = _oracle_counts(small_head_np, h, 3000, 1.6, seed=7, row=0)
    assert O.chi2_homogeneity(a, b)[2] > 1e-4
    assert O.chi2_homogeneity(a, c)[2] < 1e-6


# ---------------------------------------------------------------------------
# Building blocks
# ---------------------------------------------------------------------------

def test_philox_known_answers():
    """Random123's published known-answer vectors for philox4x32-10."""
    kats = [
        ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
        ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
        ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
         (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
    ]
    for ctr, key, want in kats:
        got = O.philox4x32_10(*[np.array([c], dtype=np.uint32) for c in ctr], *key)
        assert tuple(int(x[0]) for x in got) == want


def test_uniforms_and_gumbel_are_well_formed():
    u = O.philox_uniform(123, 0, O.STAGE_TOKENS, 0, np.arange(200000))
    assert u.min() > 0 and u.max() < 1
    assert abs(u.mean() - 0.5) < 0.005
    gm = O.gumbel(123, 0, O.STAGE_CLUSTERS, 3, np.arange(200000))
    assert abs(gm.mean() - 0.5772) < 0.02  # Euler-Mascheroni


def test_packed_order_matches_reference_signed_order():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(2000).astype(np.float32) * 10,
                        np.array([0.0, -0.0, np.inf, -np.inf, 1e-40, -1e-40], dtype=np.float32)])
    x = np.concatenate([x, x[:500]])  # ties
    ids = rng.permutation(x.size).astype(np.int64)
    mine = O.pack_u64(x, ids)
    ref = O.reference_signed_pack(x, ids)
    assert np.array_equal(np.argsort(mine, kind="stable"), np.argsort(ref, kind="stable"))
    assert np.array_equal(O.unpack_id(mine), ids)


def test_top_probes_tie_rule():
    s = np.array([1.0, 3.0, 2.0, 3.0, 2.0, 2.0, 0.5])
    assert O.top_probes(s, 1).tolist() == [1]
    assert O.top_probes(s, 3).tolist() == [1, 2, 3]
    assert O.top_probes(s, 4).tolist() == [1, 2, 3, 4]
    with pytest.raises(ValueError):
        O.top_probes(s, 0)


def test_unbalanced_clusters_rejected():
    with pytest.raises(ValueError, match="balanced"):
        O.vocab_maps_from_assignments(np.array([0, 0, 1]), 2)


def test_fp8_table():
    assert O.FP8_E4M3_VALUES[0x7E] == 448.0
    assert O.FP8_E4M3_VALUES[0x01] == 2.0 ** -9
    assert np.isnan(O.FP8_E4M3_VALUES[0x7F])
    t = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    both = ~np.isnan(t)
    assert np.array_equal(t[both], O.FP8_E4M3_VALUES[both])


def test_spec_accept_restates_the_reference_loop():
    """Draft acceptance (patches/rejection_sampler.py:55-76) on hand-made
    rows: accepted prefix, first mismatch replaced by the target id, bonus
    after a fully accepted row; a row without drafts gets its bonus only in
    vLLM's semantics (the library's), not in the reference's literal loop."""
    draft = [5, 6, 7, 1, 2, 9, 9, 9]
    target = [5, 6, 7, 1, 3, 9, 8, 9]
    bonus = [40, 41, 42, 43]
    num = [3, 2, 0, 3]  # row 0 all accepted, row 1 rejects at 1, row 2 empty, row 3 rejects at 1
    out = O.spec_accept(draft, target, bonus, num, max_spec_len=3)
    assert out.tolist() == [[5, 6, 7, 40], [1, 3, -1, -1], [42, -1, -1, -1], [9, 8, -1, -1]]
    ref = O.spec_accept(draft, target, bonus, num, max_spec_len=3, bonus_without_drafts=False)
    assert ref[2].tolist() == [-1, -1, -1, -1] and ref[0].tolist() == [5, 6, 7, 40]
