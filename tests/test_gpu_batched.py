"""Batched decode steps (16 or more rows): tensor-core stage-1 GEMM, the
selection kernel, the inverted cluster -> rows index and the inverted stage 2.

Parity is checked the same way as for the other paths: probe sets equal the
oracle's top-p up to near-ties of the p-th score, and each row's token is the
oracle's argmax over the kernel's own probe set (ties to the smallest id) up
to the logit tolerance. Sampling is compared draw for draw with the oracle's
Gumbel-top-p / Gumbel-max restatement keyed by (seed, offset, row, id).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from headutil import OracleView, build_head, check_greedy_rows, to_np_f32
from oracle import flashhead_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def llama1b_heads(config_a_head):
    head, meta = config_a_head
    p = meta["shape"]["n_probes"]
    return {s: build_head(head.weight, head.centroids, head.assignments, p, stage1=s)
            for s in ("model", "fp8")}


def _tiny_head(K, cap, D, seed=0):
    from flash_head.synthetic import HeadShape, make_head
    return make_head(HeadShape(hidden=D, vocab=K * cap, n_clusters=K, cluster_size=cap), seed=seed)


def _batched_kernel_count(nh, rows, sample=False):
    n = nh.step_kernel_count(rows, sample)
    assert n > 3, f"{rows} rows did not take the batched path ({n} launches)"
    return n


@pytest.mark.parametrize("rows", [16, 64, 256])
@pytest.mark.parametrize("stage1", ["fp8", "model"])
def test_batched_matches_oracle(llama1b_heads, rows, stage1):
    from flash_head.synthetic import make_hidden
    fh = llama1b_heads[stage1]
    nh = fh.native()
    _batched_kernel_count(nh, rows)
    H = make_hidden(rows, fh._D, seed=900 + rows, device="cuda")
    toks = nh.next_token(H).cpu().numpy()
    probes = nh.top_clusters(H).cpu().numpy()
    check_greedy_rows(fh, H, toks, probes)
    assert nh.workspace_error() == 0
    # a second call on the same workspace (index and accumulator reset)
    toks2 = nh.next_token(H).cpu().numpy()
    assert np.array_equal(toks, toks2)


@pytest.mark.parametrize("K,cap,D,p,rows", [(100, 16, 512, 100, 17), (37, 4, 1024, 5, 20),
                                            (513, 8, 256, 40, 33), (300, 16, 4096, 64, 24),
                                            (4097, 16, 128, 200, 64)])
def test_batched_shapes(K, cap, D, p, rows):
    from flash_head.synthetic import make_hidden
    head = _tiny_head(K, cap, D)
    for stage1 in ("model", "fp8"):
        fh = build_head(head.weight, head.centroids, head.assignments, p, stage1=stage1)
        nh = fh.native()
        _batched_kernel_count(nh, rows)
        H = make_hidden(rows, D, seed=rows, device="cuda")
        toks = nh.next_token(H).cpu().numpy()
        check_greedy_rows(fh, H, toks, nh.top_clusters(H).cpu().numpy())
        assert nh.workspace_error() == 0


def test_batched_special_tokens():
    """Special tokens compete with every row's candidates; one far outside
    the probed clusters still wins for a row aimed at it."""
    from flash_head.synthetic import make_hidden
    head = _tiny_head(256, 16, 512, seed=3)
    specials = [0, 17, 4095]
    fh = build_head(head.weight, head.centroids, head.assignments, 12, specials=specials,
                    stage1="model")
    nh = fh.native()
    ov = OracleView(fh)
    H = make_hidden(20, 512, seed=41, device="cuda")
    H[7] = torch.from_numpy(ov.W[4095] * 50).to("cuda", torch.bfloat16)
    Hn = to_np_f32(H)
    probes = nh.top_clusters(H).cpu().numpy()
    toks = nh.next_token(H).cpu().numpy()
    for r in range(H.shape[0]):
        want = ov.greedy_given_probes(Hn[r], probes[r])
        assert O.token_within_tolerance(toks[r], want, lambda v: ov.logit(Hn[r], v), 1e-5), r
    assert toks[7] == 4095


def test_batched_rows_beyond_one_stage2_launch():
    """300 rows: stage 2 runs as launches of 256 and 44 rows (the index filled
    by its own kernel, each launch publishing its rows), special tokens scored
    once for all rows; a second call on the same workspace repeats the ids."""
    from flash_head.synthetic import make_hidden
    head = _tiny_head(256, 16, 512, seed=5)
    fh = build_head(head.weight, head.centroids, head.assignments, 12, specials=[0, 17, 4095],
                    stage1="model")
    nh = fh.native()
    ov = OracleView(fh)
    H = make_hidden(300, 512, seed=43, device="cuda")
    H[290] = torch.from_numpy(ov.W[4095] * 50).to("cuda", torch.bfloat16)
    Hn = to_np_f32(H)
    probes = nh.top_clusters(H).cpu().numpy()
    toks = nh.next_token(H).cpu().numpy()
    for r in range(H.shape[0]):
        want = ov.greedy_given_probes(Hn[r], probes[r])
        assert O.token_within_tolerance(toks[r], want, lambda v: ov.logit(Hn[r], v), 1e-5), r
    assert toks[290] == 4095
    assert np.array_equal(nh.next_token(H).cpu().numpy(), toks)
    assert nh.workspace_error() == 0


@pytest.mark.parametrize("stage1", ["model", "fp8"])
def test_batched_sampling_matches_oracle_draw_for_draw(stage1):
    from flash_head.synthetic import make_hidden
    head = _tiny_head(256, 16, 512, seed=8)
    fh = build_head(head.weight, head.centroids, head.assignments, 12, stage1=stage1)
    nh = fh.native()
    _batched_kernel_count(nh, 16, sample=True)
    ov = OracleView(fh)
    H = make_hidden(16, 512, seed=5, device="cuda", std=4.0)
    Hn = to_np_f32(H)
    cd = ov.sw * (ov.sscale[:, None] if ov.sscale is not None else 1.0)
    n, agree = 0, 0
    for off in range(12):
        toks = nh.next_token(H, do_sample=True, temperature=0.7, seed=77, offset=off).cpu().numpy()
        for r in range(16):
            want = O.sample_token(Hn[r], ov.w_perm, ov.vm, cd, ov.p, 0.7, 77, off, r)[0]
            agree += int(toks[r] == want)
            n += 1
    assert agree >= 0.98 * n, (agree, n)


def test_batched_step_replays_in_a_cuda_graph(llama1b_heads):
    from flash_head.synthetic import make_hidden
    fh = llama1b_heads["fp8"]
    nh = fh.native()
    H = make_hidden(64, fh._D, seed=3, device="cuda")
    want = nh.next_token(H).clone()  # first call: plans and workspace exist before capture
    out = torch.empty(64, dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        nh.next_token(H, out=out)
    for _ in range(3):
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, want)


@pytest.mark.parametrize("rows", [16, 40])
def test_dense_gemm_path_is_the_exact_argmax(llama1b_heads, rows):
    """The dense head (the reference's branch for more than 10 rows,
    flash_head.py:292-301) on the tensor cores: cap GEMMs against K-row blocks
    of w_perm, block argmax with the smallest-id tie rule. Tokens equal the
    exact full-vocabulary argmax up to 1e-5-relative logit ties."""
    from flash_head.synthetic import make_hidden
    fh = llama1b_heads["fp8"]
    nh = fh.native()
    ov = OracleView(fh)
    H = make_hidden(rows, fh._D, seed=1300 + rows, device="cuda")
    toks = nh.dense_next_token(H).cpu().numpy()
    Hn = to_np_f32(H)
    for r in range(rows):
        want = O.dense_argmax(Hn[r], ov.W)
        assert O.token_within_tolerance(int(toks[r]), want, lambda v: ov.logit(Hn[r], v), 1e-5), r
    # sampling over the whole vocabulary: Gumbel-max draws are deterministic in (seed, offset)
    a = nh.dense_next_token(H, do_sample=True, temperature=0.8, seed=3, offset=1)
    b = nh.dense_next_token(H, do_sample=True, temperature=0.8, seed=3, offset=1)
    assert torch.equal(a, b)


def _check_dense_tc(nh, H):
    """Runs the dense head twice (the second call under the CUDA profiler, to
    see that the tcgen05 kernel ran), then checks every row's token against
    the fp32 logits of the same w_perm and vocab map (plain PyTorch fp32
    reference) up to 1e-5-relative ties. Returns the tokens."""
    rows = H.shape[0]
    toks = nh.dense_next_token(H)
    torch.cuda.synchronize()
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        again = nh.dense_next_token(H)
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    assert any("k_dense_tc" in n for n in names), names
    assert torch.equal(toks, again)
    assert nh.workspace_error() == 0
    wp, vm = nh.bufs["w_perm"], nh.bufs["vocab_map"].long()
    logits = torch.empty(rows, wp.shape[0], dtype=torch.float32, device="cuda")
    for j0 in range(0, wp.shape[0], 16384):  # fp32 reference, by vocab blocks
        logits[:, j0:j0 + 16384] = H.float() @ wp[j0:j0 + 16384].float().t()
    best = logits.max(dim=1).values
    slot_of = torch.empty_like(vm)
    slot_of[vm] = torch.arange(vm.numel(), device="cuda")
    mine = logits.gather(1, slot_of[toks].view(-1, 1)).view(-1)
    gap = (best - mine).abs() / best.abs().clamp_min(1e-30)
    assert bool((gap <= 1e-5).all()), (int(gap.argmax()), float(gap.max()))
    return toks


@pytest.mark.parametrize("K,cap,D,rows,dtype", [
    (37, 16, 80, 17, torch.bfloat16),      # second k-block 16 of 64 elements; 37 tiles < SMs
    (513, 8, 1040, 33, torch.float16),     # f16 operands; last vocab tile 8 of 32 slots
    (300, 16, 4096, 200, torch.bfloat16),  # two hidden tiles, the second 72 of 128 rows
])
def test_dense_tensor_core_kernel_shapes(K, cap, D, rows, dtype):
    """The tcgen05 dense kernel away from the Llama head: hidden sizes that
    leave a partial last k-block (zero fill of the TMA boxes), vocabularies
    smaller than the grid and not a multiple of the vocab tile, fp16 weights
    and hidden states, and row counts that leave most of a 128-row tile
    empty; checked against the fp32 reference and the oracle's float64
    argmax on a few rows."""
    from flash_head.synthetic import make_hidden
    head = _tiny_head(K, cap, D, seed=K)
    fh = build_head(head.weight, head.centroids, head.assignments, min(K, 16), stage1="model",
                    dtype=dtype)
    nh = fh.native()
    H = make_hidden(rows, D, seed=rows + D, device="cuda").to(dtype)
    toks = _check_dense_tc(nh, H)
    ov = OracleView(fh)
    Hn = to_np_f32(H)
    for r in (0, rows // 2, rows - 1):
        want = O.dense_argmax(Hn[r], ov.W)
        assert O.token_within_tolerance(int(toks[r]), want, lambda v: ov.logit(Hn[r], v), 1e-5), r


@pytest.mark.parametrize("rows", [128, 129, 256])
def test_dense_tensor_core_kernel_row_tiles(llama1b_heads, rows):
    """Greedy dense head in one tcgen05 kernel (csrc/fh_dense_tc.cuh): one
    128-row hidden tile (double-buffered accumulators), a second tile holding
    one row, and two full tiles. Every row's token is the fp32 argmax over the
    whole vocabulary (plain PyTorch fp32 reference of the same w_perm and
    vocab map) up to 1e-5-relative logit ties; a spread of rows is also
    checked against the oracle's float64 dense argmax."""
    from flash_head.synthetic import make_hidden
    fh = llama1b_heads["fp8"]
    nh = fh.native()
    H = make_hidden(rows, fh._D, seed=1400 + rows, device="cuda")
    toks = _check_dense_tc(nh, H)
    ov = OracleView(fh)
    Hn = to_np_f32(H)
    for r in sorted({0, 1, 127, min(128, rows - 1), rows - 1}):
        want = O.dense_argmax(Hn[r], ov.W)
        assert O.token_within_tolerance(int(toks[r]), want, lambda v: ov.logit(Hn[r], v), 1e-5), r
