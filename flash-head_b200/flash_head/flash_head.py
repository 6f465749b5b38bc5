"""FlashHead: clustering-based LM head on sm_100a CUDA kernels.

Same module interface as the reference (embedl/flash-head
``src/flash_head/flash_head.py``): ``get_flash_head_parameters`` and
``FlashHead(lm_head, centroids, vocab_maps_tensor, n_probes,
special_token_ids)`` with ``get_next_token(hidden_states, do_sample,
temperature, use_identical_tiebreak)``, the same buffers (``centroids``,
``cluster_linear``, ``w_perm``, ``vocab_maps``) and the same errors. Every
per-step computation runs in ``libflashhead_b200.so``; there is no CPU or
PyTorch fallback for the step itself.

Differences from the reference, all deliberate:
  * stage 1 scores the L2-normalised centroids in the model dtype by default
    (``stage1_dtype="model"``: the reference's bf16 scores, with fp32
    accumulation), or in fp8 e4m3 with a per-row fp32 scale
    (``stage1_dtype="fp8"``: half the stage-1 bytes; on N(0, 0.25) hidden
    states of the Llama-3.2-1B-shaped head it keeps ~97.5 % of the
    reference's probes and its greedy tokens, but the fp8 score error of
    ~2 % of the boundary score breaks the 1e-2 probe-set rule on most rows);
  * ties: probe selection prefers the smaller cluster id, the token the
    smaller vocab id, on fp32 logits in every mode (``use_identical_tiebreak``
    is accepted; the reference's tiebreak branch differs only in comparing
    bf16-rounded logits);
  * sampling draws are Gumbel-top-p / Gumbel-max with Philox noise, which
    has the reference's distribution (sequential draws without replacement
    and a multinomial over the candidates) without its sequential kernel;
  * ``get_next_token_batched`` serves any number of decode rows (greedy or
    sampled) in one call; the reference-named methods keep the reference's
    shape rules and NotImplementedError cases.
"""

from __future__ import annotations

import os
from typing import Iterable, Optional, Union

import torch
from torch import nn

from .native import NativeHead, derive_buffers, quantize_rows_fp8  # noqa: F401

# Default ratio: number of probes = clusters / DEFAULT_CLUSTER_RATIO
DEFAULT_CLUSTER_RATIO = 16

STAGE1_ENV = "FLASHHEAD_STAGE1_DTYPE"


def _get_device():
    """Device of the reference's stage-1 input (lazily, no CUDA init at import)."""
    if torch.cuda.is_available():
        return "cuda"
    return "cpu"


def _get_centroids(lm_head: nn.Linear, model_or_dir: str, cache_dir: str):
    """(centroids [D, K], cluster_assignments [V]) from the model's
    clustering cache (the reference's reader, flash_head.py:41-78), on the
    head's device, centroids in its dtype."""
    from .assets import ModelFiles, clustering

    centroids, assign = clustering(ModelFiles(model_or_dir), cache_dir, lm_head.weight.shape[0])
    w = lm_head.weight
    return centroids.to(device=w.device, dtype=w.dtype), assign.to(device=w.device)


def vocab_maps_from_assignments(assign: torch.Tensor, n_clusters: int) -> torch.Tensor:
    """[K, cap] vocab ids per cluster, ascending within each cluster; balanced
    clusters required. One stable sort instead of K scans over the vocab
    (the reference's torch.where loop, flash_head.py:100-113, same result)."""
    assign = assign.to(torch.int64)
    counts = torch.bincount(assign, minlength=n_clusters)
    if counts.numel() != n_clusters or int(counts.min()) != int(counts.max()):
        raise ValueError(
            "FlashHead requires balanced clusters; got cluster sizes "
            f"{sorted(set(counts.tolist()))} across {n_clusters} clusters.")
    return torch.argsort(assign, stable=True).view(n_clusters, int(counts[0]))


def get_flash_head_parameters(lm_head: nn.Module, cache_dir: str, model_or_dir: str) -> dict:
    """Centroids [D, K] and vocab maps [K, cap] for ``FlashHead`` (flash_head.py:81-118)."""
    centroids, assign = _get_centroids(lm_head, model_or_dir, cache_dir)
    c = centroids.squeeze(0).squeeze(0)
    vocab_maps = vocab_maps_from_assignments(assign, c.shape[1])
    return {"centroids": c.to(device=lm_head.weight.device, dtype=lm_head.weight.dtype),
            "vocab_maps_tensor": vocab_maps}


class FlashHead(nn.Module):
    """Clustering-based approximate language model head.

    1. scores the hidden state against the cluster centroids and keeps the
       top ``n_probes`` clusters (or draws them, when sampling);
    2. scores only the tokens of those clusters (plus the special tokens);
    3. returns the argmax (or sampled) token id directly.

    :param lm_head: the original classification head ([V, D] weight).
    :param centroids: cluster centroids [D, K].
    :param vocab_maps_tensor: [K, cap] vocab ids of each cluster.
    :param n_probes: probes per step (default K / 16).
    :param special_token_ids: tokens always scored, independent of clusters.
    :param stage1_dtype: "fp8" (e4m3 + per-row scale) or "model"; default from
        the FLASHHEAD_STAGE1_DTYPE environment variable, else "model".
    """

    def __init__(self, lm_head: nn.Linear, centroids: torch.Tensor,
                 vocab_maps_tensor: torch.Tensor, n_probes: Optional[int] = None,
                 special_token_ids: Optional[Union[int, Iterable[int]]] = None,
                 stage1_dtype: Optional[str] = None):
        super().__init__()
        V, D = lm_head.weight.shape
        K, cap = vocab_maps_tensor.shape
        assert K * cap == V, f"unbalanced: K={K}*cap={cap} != V={V}"
        self.original_shape = lm_head.weight.shape
        self._K, self._cap, self._D = K, cap, D
        self.n_probes = int(n_probes if n_probes is not None
                            else centroids.shape[1] / DEFAULT_CLUSTER_RATIO)
        stage1_dtype = stage1_dtype or os.environ.get(STAGE1_ENV, "model")
        if stage1_dtype not in ("fp8", "model"):
            raise ValueError(f"stage1_dtype must be 'fp8' or 'model', got {stage1_dtype!r}")
        self.stage1_dtype = stage1_dtype

        self.register_buffer("centroids", centroids.contiguous())
        c32 = centroids.to(torch.float32)
        pre_norm = (c32 / c32.norm(dim=0, keepdim=True)).t().contiguous().to(centroids.dtype)
        self.cluster_linear = nn.Linear(pre_norm.shape[1], pre_norm.shape[0], bias=False)
        self.cluster_linear.weight = nn.Parameter(pre_norm, requires_grad=False)

        perm = vocab_maps_tensor.reshape(-1).to(device=lm_head.weight.device, dtype=torch.int64)
        self.register_buffer(
            "w_perm", lm_head.weight.detach().index_select(0, perm).contiguous().view(K, cap, D))
        self.register_buffer("vocab_maps", vocab_maps_tensor.to(torch.int64).contiguous())

        st = [int(t) for t in ([special_token_ids] if isinstance(special_token_ids, int)
                               else list(special_token_ids or [])) if 0 <= int(t) < V]
        if st:
            sp = torch.tensor(st, dtype=torch.int64, device=vocab_maps_tensor.device)
            found = (vocab_maps_tensor.reshape(-1).to(torch.int64).unsqueeze(0)
                     == sp.unsqueeze(1)).any(dim=1)
            missing = sp[~found].tolist()
            if missing:
                raise ValueError(f"special_token_ids missing from vocab_maps: {missing}")
        self.register_buffer("special_token_ids_tensor", torch.tensor(st, dtype=torch.int64),
                             persistent=False)
        self._native = None  # (buffer key, NativeHead)

    # ------------------------------------------------------------------
    # Native head (device buffers + C handle)
    # ------------------------------------------------------------------
    def _native_key(self):
        return (self.w_perm.device, self.w_perm.dtype, self.w_perm.data_ptr(),
                self.cluster_linear.weight.data_ptr(), self.centroids.data_ptr(),
                self.vocab_maps.data_ptr(), self.n_probes, self.stage1_dtype)

    def native(self) -> NativeHead:
        """The device-side head for the current buffers (rebuilt after .to())."""
        key = self._native_key()
        if self._native is not None and self._native[0] == key:
            return self._native[1]
        if not self.w_perm.is_cuda:
            raise RuntimeError("FlashHead runs on CUDA only: move it with .to('cuda') first")
        if self.w_perm.dtype not in (torch.bfloat16, torch.float16):
            raise RuntimeError(f"FlashHead kernels need bf16 or fp16 weights, got {self.w_perm.dtype}")
        self._release_native()
        bufs = derive_buffers(self.w_perm, self.vocab_maps, self.cluster_linear.weight,
                              self.centroids, self.special_token_ids_tensor, self.stage1_dtype)
        head = NativeHead(bufs, self._D, self._cap, self.n_probes)
        self._native = (key, head)
        return head

    def _release_native(self):
        if self._native is not None:
            self._native[1].close()
            self._native = None

    def prepare(self, max_rows: int = 1) -> None:
        """Build the device-side head and a workspace for ``max_rows`` rows.
        Call it before capturing a CUDA graph that contains FlashHead steps:
        the steps themselves allocate only their outputs."""
        self.native().workspace(max_rows)

    def _next_seed(self):
        return int(torch.randint(0, 2**62, (1,)).item()), 0

    # ------------------------------------------------------------------
    # Batched entry points (any number of decode rows)
    # ------------------------------------------------------------------
    def get_next_token_batched(self, hidden: torch.Tensor, do_sample: bool = False,
                               temperature: float = 1.0, seed: Optional[int] = None,
                               offset: int = 0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """[N, D] hidden states -> [N] int64 next-token ids (greedy or sampled).

        Sampling draws are keyed by (seed, offset, row); without a seed one is
        drawn from torch's default generator, so torch.manual_seed applies."""
        if do_sample and seed is None:
            seed, offset = self._next_seed()
        return self.native().next_token(hidden, out=out, do_sample=do_sample,
                                        temperature=temperature, seed=seed or 0, offset=offset)

    def top_clusters_batched(self, hidden: torch.Tensor, do_sample: bool = False,
                             temperature: float = 1.0, seed: Optional[int] = None,
                             offset: int = 0, return_scores: bool = False):
        """[N, D] -> probed clusters [N, p] int32 ascending (and fp32 scores [N, K])."""
        if do_sample and seed is None:
            seed, offset = self._next_seed()
        return self.native().top_clusters(hidden, do_sample, temperature, seed or 0, offset,
                                          return_scores)

    def dense_next_token(self, hidden: torch.Tensor, do_sample: bool = False,
                         temperature: float = 1.0, seed: Optional[int] = None,
                         offset: int = 0) -> torch.Tensor:
        """Full-vocabulary next token over ``w_perm`` for [N, D] rows -> [N] int64."""
        if do_sample and seed is None:
            seed, offset = self._next_seed()
        return self.native().dense_next_token(hidden, do_sample, temperature, seed or 0, offset)

    def candidate_logprobs(self, hidden: torch.Tensor, token_ids: torch.Tensor,
                           num_logprobs: int):
        """Log-probabilities of a step over its candidate set, in the layout of
        vLLM's ``Sampler.gather_logprobs``: (ids [N, k+1] int32, logprobs
        [N, k+1] float32, ranks [N] int64), column 0 the given token, then the
        k most likely candidates; rank = candidates at least as likely as the
        token.

        The reference returns no logprobs on its FlashHead path
        (patches/sampler.py:21). Here the candidate set of a row is the tokens
        of its top-p clusters (greedy stage 1), the special tokens and the
        given token; the softmax is taken over that set only, so the
        probability mass of unprobed clusters is left out (logprobs are those
        of the renormalised candidate distribution, close to the full ones
        when the probes hold the mass). Logits are the kernels' f32 sums
        rounded to the head dtype, as vLLM's own LM head returns them."""
        from .fused import block_sparse_logits
        nh = self.native()
        h = nh._h(hidden)
        N, k = h.shape[0], int(num_logprobs)
        if k < 0:
            raise ValueError("num_logprobs must be >= 0")
        tok = token_ids.to(device=h.device, dtype=torch.int64).view(-1)
        if tok.numel() != N:
            raise ValueError(f"{tok.numel()} token ids for {N} rows")
        cap = self._cap
        probes = nh.top_clusters(h).to(torch.int64)                       # [N, p]
        logits = block_sparse_logits(h, self.w_perm.view(-1), probes, self._K, cap).float()
        ids = self.vocab_maps.index_select(0, probes.view(-1)).view(N, -1)
        # special tokens and the given token, unless already among the candidates
        flat = self.vocab_maps.view(-1)
        slot_of = torch.empty_like(flat)
        slot_of[flat] = torch.arange(flat.numel(), device=flat.device)
        sp = self.special_token_ids_tensor.to(h.device)
        extra = torch.cat([sp.unsqueeze(0).expand(N, -1), tok.view(N, 1)], 1)   # [N, S+1]
        slots = slot_of.index_select(0, extra.view(-1)).view(N, -1)
        rows = self.w_perm.view(-1, self._D).index_select(0, slots.view(-1)).view(N, -1, self._D)
        ex_logits = torch.einsum("nsd,nd->ns", rows.float(), h.float()).to(h.dtype).float()
        dup = ((slots // cap).unsqueeze(2) == probes.unsqueeze(1)).any(dim=2)
        earlier = (extra.unsqueeze(2) == extra.unsqueeze(1)).tril(diagonal=-1).any(dim=2)
        ex_logits = ex_logits.masked_fill(dup | earlier, float("-inf"))
        all_ids = torch.cat([ids, extra], 1)
        lp = torch.log_softmax(torch.cat([logits, ex_logits], 1), dim=-1)
        hit = (all_ids == tok.view(N, 1)) & torch.isfinite(lp)
        tok_lp = lp.masked_fill(~hit, float("-inf")).max(dim=1).values
        top_lp, top_i = torch.topk(lp, k, dim=-1)
        out_ids = torch.cat([tok.view(N, 1), all_ids.gather(1, top_i)], 1).to(torch.int32)
        out_lp = torch.cat([tok_lp.view(N, 1), top_lp], 1)
        ranks = (lp >= tok_lp.view(N, 1)).sum(dim=1)
        return out_ids, out_lp, ranks

    # ------------------------------------------------------------------
    # Reference-named methods (flash_head.py:190-334)
    # ------------------------------------------------------------------
    def _get_top_clusters(self, hidden_states: torch.Tensor, do_sample: bool = False,
                          temperature: float = 1.0) -> torch.Tensor:
        """[1, T, D] -> [1, T, p] int64 selected clusters (flash_head.py:190-221)."""
        B, T, _ = hidden_states.shape
        if B != 1:
            raise NotImplementedError("FlashHead currently supports batch size = 1 only")
        if do_sample and T != 1:
            raise NotImplementedError
        probes = self.top_clusters_batched(hidden_states.view(T, -1), do_sample, temperature)
        return probes.to(torch.int64).view(1, T, self.n_probes)

    def _gather_cluster_logits(self, hidden_states: torch.Tensor, top_clusters: torch.Tensor,
                               use_identical_tiebreak: bool):
        """Candidate logits of row 0's probed clusters (+ special tokens):
        (logits [1, 1, N], mapping, vocab ids [N]) as in flash_head.py:223-261."""
        from .fused import block_sparse_logits
        B, _, _ = hidden_states.shape
        if B != 1:
            raise NotImplementedError("FlashHead currently supports batch size = 1 only")
        ci = top_clusters if top_clusters.dim() == 1 else top_clusters[0, 0]
        ci = ci.to(torch.int64)
        h = self.native()._h(hidden_states[:, -1:, :])
        logits = block_sparse_logits(h, self.w_perm.view(-1), ci.view(1, -1), self._K,
                                     self._cap).view(-1)
        ids = self.vocab_maps.index_select(0, ci).reshape(-1)
        if self.special_token_ids_tensor.numel() > 0:
            sp = self.special_token_ids_tensor.to(ids.device)
            flat = self.vocab_maps.view(-1)
            sp_rows = (flat.unsqueeze(0) == sp.unsqueeze(1)).int().argmax(dim=1)
            sp_logits = (self.w_perm.view(-1, self._D).index_select(0, sp_rows).float()
                         @ h[0].float()).to(logits.dtype)
            ids = torch.cat([ids, sp])
            logits = torch.cat([logits, sp_logits])
            ids, inverse = torch.unique(ids, return_inverse=True)
            logits = torch.zeros(ids.numel(), dtype=logits.dtype,
                                 device=ids.device).scatter_(0, inverse, logits)
        mapping = None
        if use_identical_tiebreak:
            srt = ids.sort()
            ids, mapping = srt.values, srt.indices
            logits = logits.index_select(0, mapping)
        return logits.view(1, 1, -1), mapping, ids

    def get_next_token_standard(self, logits: torch.Tensor, do_sample: bool = False,
                                temperature: float = 1.0):
        """Next token from full-vocabulary logits [B, T, V] (flash_head.py:263-275)."""
        if do_sample:
            probs = (logits[:, -1, :] / temperature).softmax(dim=-1)
            return torch.multinomial(probs, num_samples=1)
        return logits[:, -1:].argmax(dim=-1)

    def get_next_token(self, hidden_states: torch.Tensor, do_sample: bool = False,
                       temperature: float = 1.0, use_identical_tiebreak: bool = False
                       ) -> torch.Tensor:
        """Next token for [B, T, D] hidden states (flash_head.py:277-334).

        B > 10: full-vocabulary head -> [B, 1]. Otherwise B must be 1:
        greedy -> [T, 1] int64; sampling (T = 1 only) -> [1] int64.
        """
        if hidden_states.shape[0] > 10:
            ids = self.dense_next_token(hidden_states[:, -1, :], do_sample, temperature)
            return ids.view(-1, 1)
        B, T, _ = hidden_states.shape
        if B != 1:
            raise NotImplementedError("FlashHead currently supports batch size = 1 only")
        if do_sample:
            if T != 1:
                raise NotImplementedError
            return self.get_next_token_batched(hidden_states.view(1, -1), True, temperature)
        return self.get_next_token_batched(hidden_states.view(T, -1)).view(T, 1)

    def extra_repr(self) -> str:
        return (f"clusters={self._K}, cluster_size={self._cap}, hidden={self._D}, "
                f"n_probes={self.n_probes}, stage1={self.stage1_dtype}, "
                f"special_tokens={self.special_token_ids_tensor.numel()}")
