"""Tensor-parallel step over NCCL on two GPUs (one process per GPU).

Each rank keeps only its contiguous cluster range; the step exchanges the
[rows, p] candidate words with one all-gather and the [rows] packed winners
with one MAX all-reduce. Both ranks must return the same ids, those of the
unsharded head up to fp32 near-ties, greedy and sampling, at 6 rows and at
40 rows (tensor-core stage 1, inverted stage 2). Skipped unless two GPUs are
visible. The process group has a short timeout so a failing peer ends the
test with an error instead of a hang.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import faulthandler
    import sys
    faulthandler.dump_traceback_later(150, exit=True)  # a stuck rank reports where it is
    here = os.path.dirname(os.path.abspath(__file__))
    for p_ in (os.path.join(os.path.dirname(here), "flash-head_b200"), os.path.dirname(here), here):
        sys.path.insert(0, p_)
    import torch.distributed as dist

    from flash_head import _lib
    from flash_head.native import NativeHead
    from flash_head.synthetic import HeadShape, make_head, make_hidden
    from flash_head.tp import ShardedFlashHead
    from headutil import build_head

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        shape = HeadShape(hidden=1024, vocab=32768, n_clusters=2048, n_probes=64)
        head = make_head(shape, seed=71)
        fh = build_head(head.weight, head.centroids, head.assignments, shape.n_probes,
                        stage1="fp8")
        shard = ShardedFlashHead.from_flash_head(fh, group=dist.group.WORLD,
                                                 device=torch.device("cuda", rank))
        nh = fh.native()
        twin = NativeHead(nh.bufs, nh.D, nh.cap, nh.p, flags=_lib.FH_FLAG_NO_FUSED)
        out = {}
        # 6 rows: three-kernel shard steps; 40 rows: tensor-core stage 1 and
        # the inverted stage 2 over the owned probes
        for rows, ref in ((6, twin), (40, nh)):
            H = make_hidden(rows, shape.hidden, seed=72 + rows, device="cuda", std=2.0)
            for do_sample in (False, True):
                kw = dict(do_sample=do_sample, temperature=0.8, seed=13, offset=4)
                got = shard.get_next_token_batched(H, **kw)
                want = ref.next_token(H, **kw)
                out[(rows, do_sample)] = (got.tolist(), want.tolist())
        torch.cuda.synchronize()
        result_q.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_tp_two_gpus_nccl_matches_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p_ in procs:
        p_.start()
    results = {}
    try:
        for _ in range(2):
            rank, out = q.get(timeout=240)
            results[rank] = out
    finally:
        for p_ in procs:
            p_.join(timeout=60)
            if p_.is_alive():
                p_.kill()
    assert all(p_.exitcode == 0 for p_ in procs), [p_.exitcode for p_ in procs]
    for rank in (0, 1):
        for key, (got, want) in results[rank].items():
            # the shards' stage 1 sums other splits of the hidden dimension than
            # the whole head's (fp32 order): at most one near-tie row may differ
            assert sum(a != b for a, b in zip(got, want)) <= 1, (rank, key, got, want)
        assert results[rank] == results[1 - rank]  # every rank returns the same ids
