"""Helpers shared by the GPU tests: build a FlashHead on CUDA and compute the
oracle's answer on exactly the data the kernels read."""

from __future__ import annotations

import numpy as np
import torch

from oracle import flashhead_oracle as O

RTOL = 1e-2


def build_head(weight: torch.Tensor, centroids: torch.Tensor, assignments: torch.Tensor,
               n_probes: int, specials=None, stage1: str = "fp8",
               dtype: torch.dtype = torch.bfloat16):
    """FlashHead on cuda:0 the way the loader builds it (fp32 derivation, then cast)."""
    from torch import nn

    from flash_head.flash_head import FlashHead, vocab_maps_from_assignments
    V, D = weight.shape
    with torch.device("meta"):
        lm = nn.Linear(D, V, bias=False)
    lm.weight = nn.Parameter(weight.to("cuda", torch.float32), requires_grad=False)
    K = centroids.shape[1]
    vm = vocab_maps_from_assignments(assignments.to("cuda"), K)
    fh = FlashHead(lm, centroids.to("cuda", torch.float32), vm, n_probes=n_probes,
                   special_token_ids=specials, stage1_dtype=stage1).to("cuda", dtype)
    return fh


def to_np_f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


class OracleView:
    """The head's buffers as numpy arrays, exactly as the kernels see them."""

    def __init__(self, fh):
        nh = fh.native()
        b = nh.bufs
        self.p = fh.n_probes
        self.K, self.cap, self.D = fh._K, fh._cap, fh._D
        self.vm = fh.vocab_maps.cpu().numpy()
        self.w_perm = to_np_f32(fh.w_perm)
        flat = self.vm.reshape(-1)
        self.slot = np.empty(flat.size, dtype=np.int64)  # vocab id -> w_perm row
        self.slot[flat] = np.arange(flat.size)
        self._W = None
        self.cw, self.cscale = self._matrix(b["cluster_w"], b["cluster_scale"])
        self.sw, self.sscale = self._matrix(b["centroid_w"], b["centroid_scale"])
        self.specials = fh.special_token_ids_tensor.cpu().numpy()

    @staticmethod
    def _matrix(w, scale):
        if w.dtype == torch.float8_e4m3fn:
            q = O.fp8_e4m3_decode(w.view(torch.uint8).cpu().numpy())
            return q, scale.cpu().numpy().astype(np.float64)
        return to_np_f32(w), None

    @property
    def W(self) -> np.ndarray:
        """[V, D] rows in vocab order (built on first use: large heads)."""
        if self._W is None:
            self._W = self.w_perm.reshape(-1, self.D)[self.slot]
        return self._W

    def scores(self, H: np.ndarray) -> np.ndarray:
        return O.cluster_scores(H, self.cw, self.cscale)

    def sample_scores(self, H: np.ndarray) -> np.ndarray:
        return O.cluster_scores(H, self.sw, self.sscale)

    def logit(self, h: np.ndarray, v: int) -> float:
        row = self.w_perm.reshape(-1, self.D)[self.slot[v]]
        return float(row.astype(np.float64) @ h.astype(np.float64))

    def greedy_given_probes(self, h, probes):
        vids, logits = O.candidate_logits(h, self.w_perm, self.vm, probes, self.specials)
        return O.argmax_smallest_id(vids, logits)[0]

    def greedy(self, h):
        s = self.scores(h[None])[0]
        probes = O.top_probes(s, self.p)
        return self.greedy_given_probes(h, probes), probes, s


def check_greedy_rows(fh, H_t: torch.Tensor, toks: np.ndarray, probes: np.ndarray | None = None,
                      score_rtol: float = 1e-4):
    """Assert kernel tokens/probes agree with the oracle on the kernel's own data.

    probes: kernel probe lists [N, p] (optional). Probe sets must match the
    oracle's top-p up to clusters whose score is within score_rtol of the p-th
    (fp32 vs fp64 accumulation); the token must be the oracle's argmax over the
    kernel's probe set (ties to the smallest id) up to the logit tolerance.
    """
    ov = OracleView(fh)
    H = to_np_f32(H_t)
    S = ov.scores(H)
    for r in range(H.shape[0]):
        ref_probes = O.top_probes(S[r], ov.p)
        if probes is not None:
            assert O.probe_set_within_tolerance(probes[r], ref_probes, S[r], score_rtol), r
            use = probes[r]
        else:
            use = ref_probes
        want = ov.greedy_given_probes(H[r], use)
        assert O.token_within_tolerance(int(toks[r]), want, lambda v: ov.logit(H[r], v),
                                        1e-5), (r, int(toks[r]), want)
    return ov
