"""Device-side FlashHead: derived buffers + the C-ABI handle + workspace.

``NativeHead`` owns the device buffers the kernels read (in the layout of
``fh_head_desc``), the opaque ``fh_head`` handle and a per-device scratch
workspace. ``FlashHead`` (unsharded) and ``ShardedFlashHead`` (one cluster
range of a tensor-parallel head) both drive the kernels through it.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib


def quantize_rows_fp8(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row symmetric e4m3 quantisation: w ~= q * scale[:, None]."""
    w32 = w.to(torch.float32)
    amax = w32.abs().amax(dim=1).clamp_min(torch.finfo(torch.float32).tiny)
    scale = amax / 448.0
    q = (w32 / scale[:, None]).clamp_(-448.0, 448.0).to(torch.float8_e4m3fn)
    return q.contiguous(), scale.contiguous()


def derive_buffers(w_perm: torch.Tensor, vocab_maps: torch.Tensor, cluster_w: torch.Tensor,
                   centroids_dk: torch.Tensor, special_ids: torch.Tensor,
                   stage1_dtype: str) -> dict:
    """Kernel-side buffers of a whole head (all on w_perm's device).

    w_perm [K, cap, D] (bf16/fp16), vocab_maps [K, cap], cluster_w [K, D]
    normalised centroids, centroids_dk [D, K] raw centroids, special_ids [S].
    Returns w_perm (flat rows), vocab_map int32 [K*cap], cluster_w (+scale),
    centroid_w (+scale) as [K, D] rows, special_slots int32 [S].
    """
    dev, wdt = w_perm.device, w_perm.dtype
    K, cap, D = w_perm.shape
    with torch.no_grad():
        flat = vocab_maps.reshape(-1).to(device=dev, dtype=torch.int64)
        bufs = {"w_perm": w_perm.reshape(K * cap, D).contiguous(),
                "vocab_map": flat.to(torch.int32).contiguous()}
        cw = cluster_w.detach().to(device=dev, dtype=wdt).contiguous()
        raw = centroids_dk.detach().to(device=dev).t().to(wdt).contiguous()
        if stage1_dtype == "fp8":
            bufs["cluster_w"], bufs["cluster_scale"] = quantize_rows_fp8(cw)
            bufs["centroid_w"], bufs["centroid_scale"] = quantize_rows_fp8(raw)
        else:
            bufs["cluster_w"], bufs["centroid_w"] = cw, raw
            bufs["cluster_scale"] = bufs["centroid_scale"] = None
        # Slots of the special tokens: the vocab ids need not be a permutation
        # of [0, K*cap) (a tensor-parallel shard holds a subset of the vocab).
        sp = special_ids.to(device=dev, dtype=torch.int64)
        if sp.numel():
            span = max(int(flat.max()), int(sp.max())) + 1
            inv = torch.full((span,), -1, dtype=torch.int64, device=dev)
            inv[flat] = torch.arange(flat.numel(), device=dev)
            slots = inv[sp]
            if bool((slots < 0).any()):
                raise ValueError("special token ids missing from the vocab maps: "
                                 f"{sp[slots < 0].tolist()}")
            bufs["special_slots"] = slots.to(torch.int32).contiguous()
        else:
            bufs["special_slots"] = None
    return bufs


def shard_buffers(bufs: dict, cap: int, lo: int, hi: int) -> dict:
    """Buffers of clusters [lo, hi) of a whole head; special slots re-based."""
    out = {
        "w_perm": bufs["w_perm"][lo * cap:hi * cap].contiguous(),
        "vocab_map": bufs["vocab_map"][lo * cap:hi * cap].contiguous(),
    }
    for k in ("cluster_w", "centroid_w"):
        out[k] = bufs[k][lo:hi].contiguous()
    for k in ("cluster_scale", "centroid_scale"):
        out[k] = None if bufs[k] is None else bufs[k][lo:hi].contiguous()
    sp = bufs["special_slots"]
    if sp is not None:
        mine = sp[(sp >= lo * cap) & (sp < hi * cap)] - lo * cap
        out["special_slots"] = mine.to(torch.int32).contiguous() if mine.numel() else None
    else:
        out["special_slots"] = None
    return out


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


class NativeHead:
    """A validated ``fh_head`` over device buffers, plus its workspaces."""

    def __init__(self, bufs: dict, hidden: int, cluster_size: int, n_probes: int,
                 cluster_base: int = 0, flags: int = 0):
        self.bufs = bufs
        w = bufs["w_perm"]
        self.device = w.device
        self.dtype = w.dtype
        self.D = hidden
        self.cap = cluster_size
        self.K = w.shape[0] // cluster_size
        self.p = n_probes
        self.cluster_base = cluster_base
        d = _lib.HeadDesc()
        d.hidden, d.n_clusters, d.cluster_size, d.n_probes = hidden, self.K, cluster_size, n_probes
        d.weight_dtype = _lib.dtype_code(w.dtype)
        d.score_dtype = _lib.dtype_code(bufs["cluster_w"].dtype)
        d.sample_dtype = _lib.dtype_code(bufs["centroid_w"].dtype)
        sp = bufs["special_slots"]
        d.n_special = 0 if sp is None else sp.numel()
        d.cluster_base = cluster_base
        d.flags = flags
        d.w_perm = w.data_ptr()
        d.vocab_map = bufs["vocab_map"].data_ptr()
        d.cluster_w = bufs["cluster_w"].data_ptr()
        d.cluster_scale = _ptr(bufs["cluster_scale"])
        d.centroid_w = bufs["centroid_w"].data_ptr()
        d.centroid_scale = _ptr(bufs["centroid_scale"])
        d.special_slots = _ptr(sp)
        self.desc = d
        self.lib = _lib.load_library()
        handle = ctypes.c_void_p()
        _lib.call("fh_head_create", ctypes.byref(d), ctypes.byref(handle))
        self.handle = handle
        self._ws: dict[int, torch.Tensor] = {}

    def close(self):
        if self.handle is not None:
            self.lib.fh_head_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def workspace_bytes(self, rows: int) -> int:
        return int(self.lib.fh_workspace_bytes(self.handle, rows))

    def workspace(self, rows: int, host: bool = False) -> torch.Tensor:
        """This device's workspace, grown (zero-filled) to serve `rows` rows;
        `host`: sized for fh_get_next_token_host (device staging included)."""
        idx = self.device.index if self.device.index is not None else torch.cuda.current_device()
        need = (int(self.lib.fh_workspace_bytes_host(self.handle, rows)) if host
                else self.workspace_bytes(rows))
        ws = self._ws.get(idx)
        if ws is None or ws.numel() < need:
            # zero-filled: fh_stage2_next_token expects a clean accumulator
            ws = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device=self.device)
            self._ws[idx] = ws
        return ws

    def step_kernel_count(self, rows: int, do_sample: bool = False) -> int:
        """Launches per step for `rows` rows: 1 (one-kernel step) or 3."""
        return int(self.lib.fh_step_kernel_count(self.handle, rows, int(bool(do_sample))))

    def workspace_error(self, clear: bool = True) -> int:
        """Error bits the one-kernel step recorded in this device's workspace
        (bit 0 grid-barrier timeout, bit 1 copy timeout); synchronises."""
        idx = self.device.index if self.device.index is not None else torch.cuda.current_device()
        ws = self._ws.get(idx)
        if ws is None:
            return 0
        off = int(self.lib.fh_workspace_error_offset())
        word = ws[off:off + 4]
        torch.cuda.synchronize(self.device)
        val = int(word.view(torch.int32).item())
        if clear:
            word.zero_()
        return val

    def _h(self, hidden: torch.Tensor) -> torch.Tensor:
        h = hidden.reshape(-1, self.D)
        if h.dtype != self.dtype or h.device != self.device:
            h = h.to(device=self.device, dtype=self.dtype)
        return h.contiguous()

    # -- steps ---------------------------------------------------------------
    def next_token(self, hidden, out=None, do_sample=False, temperature=1.0, seed=0, offset=0):
        h = self._h(hidden)
        n = h.shape[0]
        if out is None:
            out = torch.empty(n, dtype=torch.int64, device=self.device)
        if n == 0:
            return out
        ws = self.workspace(n)
        s = _lib.stream_ptr()
        if do_sample:
            _lib.call("fh_get_next_token_sample", self.handle, h.data_ptr(), n, float(temperature),
                      int(seed), int(offset), out.data_ptr(), ws.data_ptr(), ws.numel(), s)
        else:
            _lib.call("fh_get_next_token", self.handle, h.data_ptr(), n, out.data_ptr(),
                      ws.data_ptr(), ws.numel(), s)
        return out

    def next_token_host(self, hidden_host: torch.Tensor, out_host: Optional[torch.Tensor] = None):
        """Greedy ids with host buffers through fh_get_next_token_host:
        [N, D] CPU hidden states (pinned for asynchronous copies) -> [N] int64
        CPU ids; returns after the ids are on the host."""
        h = hidden_host.contiguous()
        if h.device.type != "cpu" or h.dtype != self.dtype:
            raise ValueError(f"expected a CPU {self.dtype} tensor, got {h.device} {h.dtype}")
        n = h.shape[0]
        if out_host is None:
            out_host = torch.empty(n, dtype=torch.int64, pin_memory=True)
        if n == 0:
            return out_host
        ws = self.workspace(n, host=True)
        _lib.call("fh_get_next_token_host", self.handle, h.data_ptr(), n, out_host.data_ptr(),
                  ws.data_ptr(), ws.numel(), _lib.stream_ptr())
        return out_host

    def top_clusters(self, hidden, do_sample=False, temperature=1.0, seed=0, offset=0,
                     return_scores=False):
        h = self._h(hidden)
        n = h.shape[0]
        probes = torch.empty((n, self.p), dtype=torch.int32, device=self.device)
        scores = (torch.empty((n, self.K), dtype=torch.float32, device=self.device)
                  if return_scores else None)
        if n:
            ws = self.workspace(n)
            _lib.call("fh_top_clusters", self.handle, h.data_ptr(), n, int(bool(do_sample)),
                      float(temperature), int(seed), int(offset), probes.data_ptr(),
                      _ptr(scores), ws.data_ptr(), ws.numel(), _lib.stream_ptr())
        return (probes, scores) if return_scores else probes

    def cluster_scores(self, hidden, do_sample=False, temperature=1.0, seed=0, offset=0,
                       out=None):
        """Stage 1 only: [N, K] fp32 scores (or Gumbel keys when sampling)."""
        h = self._h(hidden)
        n = h.shape[0]
        out = out if out is not None else torch.empty((n, self.K), dtype=torch.float32,
                                                      device=self.device)
        if n:
            _lib.call("fh_cluster_scores", self.handle, h.data_ptr(), n, int(bool(do_sample)),
                      float(temperature), int(seed), int(offset), out.data_ptr(),
                      _lib.stream_ptr())
        return out

    def stage2_next_token(self, hidden, probes, do_sample=False, temperature=1.0, seed=0,
                          offset=0, out=None):
        """Stage 2 only for given int32 probe lists [N, p] -> [N] int64."""
        h = self._h(hidden)
        n = h.shape[0]
        pr = probes.to(device=self.device, dtype=torch.int32).contiguous()
        if pr.shape != (n, self.p):
            raise ValueError(f"probes must be [{n}, {self.p}], got {tuple(pr.shape)}")
        out = out if out is not None else torch.empty(n, dtype=torch.int64, device=self.device)
        if n:
            ws = self.workspace(n)
            _lib.call("fh_stage2_next_token", self.handle, h.data_ptr(), n, pr.data_ptr(),
                      int(bool(do_sample)), float(temperature), int(seed), int(offset),
                      out.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_ptr())
        return out

    def dense_next_token(self, hidden, do_sample=False, temperature=1.0, seed=0, offset=0,
                         out=None):
        h = self._h(hidden)
        n = h.shape[0]
        if out is None:
            out = torch.empty(n, dtype=torch.int64, device=self.device)
        if n:
            ws = self.workspace(n)
            _lib.call("fh_dense_next_token", self.handle, h.data_ptr(), n, int(bool(do_sample)),
                      float(temperature), int(seed), int(offset), out.data_ptr(), ws.data_ptr(),
                      ws.numel(), _lib.stream_ptr())
        return out

    def tp_local_candidates(self, hidden, do_sample=False, temperature=1.0, seed=0, offset=0,
                            out=None):
        h = self._h(hidden)
        n = h.shape[0]
        cand = out if out is not None else torch.empty((n, self.p), dtype=torch.int64,
                                                       device=self.device)
        if n:
            ws = self.workspace(n)
            _lib.call("fh_tp_local_candidates", self.handle, h.data_ptr(), n,
                      int(bool(do_sample)), float(temperature), int(seed), int(offset),
                      cand.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_ptr())
        return cand

    def tp_select_and_score(self, hidden, all_cand, n_ranks, do_sample=False, temperature=1.0,
                            seed=0, offset=0, out=None):
        h = self._h(hidden)
        n = h.shape[0]
        best = out if out is not None else torch.empty(n, dtype=torch.int64, device=self.device)
        if n:
            ws = self.workspace(n)
            _lib.call("fh_tp_select_and_score", self.handle, h.data_ptr(), n, int(n_ranks),
                      all_cand.data_ptr(), int(bool(do_sample)), float(temperature), int(seed),
                      int(offset), best.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_ptr())
        return best

    @staticmethod
    def tp_finalize(best: torch.Tensor, out=None):
        n = best.shape[0]
        out = out if out is not None else torch.empty(n, dtype=torch.int64, device=best.device)
        if n:
            _lib.call("fh_tp_finalize", best.data_ptr(), n, out.data_ptr(), _lib.stream_ptr())
        return out
