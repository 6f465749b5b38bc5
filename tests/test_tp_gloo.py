"""Tensor-parallel exchange with real collectives (gloo, 2 CPU ranks).

The per-rank kernels are replaced by the oracle (same packing and the same
global-id RNG keying as the CUDA kernels), so this exercises the host-side
orchestration: cluster partitioning, the candidate-word encoding, the
all-gather layout, the global selection, ownership filtering and the MAX
reduction. It also checks that a rank that never joins makes its peers fail
with an error instead of hanging.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_kernels(w_perm, vm, cw, craw, p, lo, hi, do_sample, T, seed, offset):
    """CPU stand-ins for fh_tp_local_candidates / select_and_score / finalize."""
    from oracle import flashhead_oracle as O

    def local(h):
        rows = h.shape[0]
        out = np.empty((rows, p), dtype=np.int64)
        for r in range(rows):
            if do_sample:
                s = O.cluster_scores(h[r:r + 1], craw[lo:hi])[0].astype(np.float32) / np.float32(T)
                s = s + O.gumbel(seed, offset, O.STAGE_CLUSTERS, r, np.arange(lo, hi))
            else:
                s = O.cluster_scores(h[r:r + 1], cw[lo:hi])[0].astype(np.float32)
            ids = O.top_probes(s, p)
            words = O.pack_u64(s[ids], ids + lo)
            out[r] = (words ^ np.uint64(1 << 63)).view(np.int64)
        return torch.from_numpy(out)

    def select(h, all_cand, world):
        rows = h.shape[0]
        best = np.empty(rows, dtype=np.int64)
        for r in range(rows):
            words = (all_cand[:, r, :].numpy().reshape(-1).view(np.uint64) ^ np.uint64(1 << 63))
            top = np.sort(words)[::-1][:p]
            gids = O.unpack_id(top)
            mine = gids[(gids >= lo) & (gids < hi)]
            if len(mine) == 0:
                best[r] = np.int64(-(1 << 63))
                continue
            vids, logits = O.candidate_logits(h[r], w_perm, vm, mine)
            key = logits.astype(np.float32)
            if do_sample:
                key = key / np.float32(T) + O.gumbel(seed, offset, O.STAGE_TOKENS, r, vids)
            w = O.pack_u64(key, vids).max()
            best[r] = (np.uint64(w) ^ np.uint64(1 << 63)).view(np.int64)
        return torch.from_numpy(best)

    def finalize(best):
        w = best.numpy().view(np.uint64) ^ np.uint64(1 << 63)
        return torch.from_numpy(O.unpack_id(w))

    return local, select, finalize


def _worker(rank, world, port, do_sample, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    for p_ in (os.path.join(os.path.dirname(here), "flash-head_b200"), os.path.dirname(here)):
        sys.path.insert(0, p_)
    import torch.distributed as dist

    from flash_head.synthetic import HeadShape, make_head, make_hidden
    from flash_head.tp import cluster_range, exchange_step
    from oracle import flashhead_oracle as O

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    shape = HeadShape(hidden=64, vocab=4096, n_clusters=256, n_probes=12)
    head = make_head(shape, seed=21)
    W = head.weight.float().numpy()
    vm = O.vocab_maps_from_assignments(head.assignments.numpy(), shape.n_clusters)
    w_perm = O.permute_weight(W, vm)
    cw = O.normalized_cluster_weight(head.centroids.numpy())
    craw = np.ascontiguousarray(head.centroids.numpy().T)
    H = make_hidden(6, shape.hidden, seed=22, std=3.0).float().numpy()
    lo, hi = cluster_range(shape.n_clusters, world, rank)
    local, select, finalize = _oracle_kernels(w_perm, vm, cw, craw, shape.n_probes, lo, hi,
                                              do_sample, 0.8, 5, 9)
    ids = exchange_step(H, dist.group.WORLD, local, select, finalize)
    # unsharded answer (rank 0 computes it with the same oracle)
    if rank == 0:
        want = []
        for r in range(H.shape[0]):
            if do_sample:
                want.append(O.sample_token(H[r], w_perm, vm, craw, shape.n_probes, 0.8, 5, 9, r)[0])
            else:
                want.append(O.greedy_token(H[r], w_perm, vm, cw, shape.n_probes)[0])
        result_q.put((ids.tolist(), want))
    dist.destroy_process_group()


@pytest.mark.parametrize("do_sample", [False, True])
def test_tp_exchange_gloo_two_ranks(do_sample):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, do_sample, q)) for r in range(2)]
    for p_ in procs:
        p_.start()
    got, want = q.get(timeout=180)
    for p_ in procs:
        p_.join(timeout=60)
        assert p_.exitcode == 0
    assert got == want


def _lonely_worker(port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist
    try:
        dist.init_process_group("gloo", rank=0, world_size=2,
                                timeout=datetime.timedelta(seconds=3))
        t = torch.zeros(4, dtype=torch.int64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        result_q.put("no error")
    except Exception as e:  # the peer never joined: rendezvous or collective times out
        result_q.put(type(e).__name__)


def test_missing_rank_fails_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p_ = ctx.Process(target=_lonely_worker, args=(_free_port(), q))
    p_.start()
    res = q.get(timeout=120)
    p_.join(timeout=30)
    if p_.is_alive():
        p_.kill()
    assert res != "no error"
