"""The workspace-free greedy entry point, fh_get_next_token_noalloc.

Some callers of this library cannot allocate device memory at the moment they
need a token (a CUDA graph being captured, a latency-critical thread that must
not enter the allocator, a runtime whose fixed pool forbids cudaMalloc), so
they cannot provide the workspace the other entry points take. This entry
point runs the same kernels on a fixed scratch array that the library owns.

Checked here through the C ABI: two calls in a row give the ids of the
workspace entry point (identical to its three-kernel path; within the tests'
1e-5 logit tolerance of its default one-kernel path) and the oracle's greedy
token on the same fp8 stage-1 matrix (probe sets and the token within the
tests' 1e-4 score / 1e-5 logit tolerances), zero rows is a no-op,
and sizes beyond the fixed limits are refused with FH_ERR_UNSUPPORTED. The
file is named to be collected last and needs no other test to run first.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from headutil import OracleView, build_head, check_greedy_rows, to_np_f32
from oracle import flashhead_oracle as O

pytestmark = pytest.mark.gpu


def _noalloc(nh, H):
    from flash_head import _lib
    out = torch.full((H.shape[0],), -1, dtype=torch.int64, device="cuda")
    st = nh.lib.fh_get_next_token_noalloc(nh.handle, H.data_ptr(), H.shape[0], out.data_ptr(),
                                          _lib.stream_ptr())
    assert st == _lib.FH_OK, _lib.last_error()
    return out


@pytest.fixture(scope="module")
def head():
    from flash_head.synthetic import HeadShape, make_head
    shape = HeadShape(hidden=1024, vocab=32768, n_clusters=2048, n_probes=64)
    h = make_head(shape, seed=31)
    return build_head(h.weight, h.centroids, h.assignments, shape.n_probes, stage1="fp8")


def test_noalloc_matches_the_workspace_entry_point(head):
    from flash_head import _lib
    from flash_head.native import NativeHead
    from flash_head.synthetic import make_hidden
    nh = head.native()
    three = NativeHead(nh.bufs, nh.D, nh.cap, nh.p, flags=_lib.FH_FLAG_NO_FUSED)
    ov = OracleView(head)
    for call, rows in enumerate((3, 4)):  # two calls in a row
        H = make_hidden(rows, nh.D, seed=90 + call, device="cuda")
        got = _noalloc(nh, H)
        torch.cuda.synchronize()
        assert torch.equal(got, three.next_token(H))
        default = nh.next_token(H).cpu().numpy()
        Hn = to_np_f32(H)
        for r, tok in enumerate(got.cpu().numpy()):
            assert O.token_within_tolerance(tok, default[r], lambda v: ov.logit(Hn[r], v), 1e-5)
        # directly against the oracle: the token is the argmax of the oracle's
        # candidates for the kernels' probe set, which is the oracle's top-p
        check_greedy_rows(head, H, got.cpu().numpy(), nh.top_clusters(H).cpu().numpy())
        for r in range(rows):
            want, _, _ = ov.greedy(Hn[r])
            assert O.token_within_tolerance(int(got[r]), want, lambda v: ov.logit(Hn[r], v),
                                            1e-5), (r, int(got[r]), want)


def test_noalloc_limits(head):
    from flash_head import _lib
    from flash_head.synthetic import make_hidden
    nh = head.native()
    H = make_hidden(5, nh.D, seed=3, device="cuda")
    out = torch.empty(5, dtype=torch.int64, device="cuda")
    st = nh.lib.fh_get_next_token_noalloc(nh.handle, H.data_ptr(), 5, out.data_ptr(),
                                          _lib.stream_ptr())
    assert st == _lib.FH_ERR_UNSUPPORTED and "fixed scratch" in _lib.last_error()
    assert nh.lib.fh_get_next_token_noalloc(nh.handle, H.data_ptr(), 0, out.data_ptr(),
                                            _lib.stream_ptr()) == _lib.FH_OK
    np.testing.assert_array_equal(_noalloc(nh, H[:2]).cpu().numpy(),
                                  _noalloc(nh, H[:2]).cpu().numpy())
