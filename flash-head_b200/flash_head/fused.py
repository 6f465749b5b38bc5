"""Block-sparse FlashHead kernels with the reference's call signatures.

Same functions, arguments and results as the reference's Triton module
(embedl/flash-head ``src/flash_head/fused.py``), computed by the sm_100a
kernels of ``libflashhead_b200.so``:

    block_sparse_logits(hs, w_perm_flat, ci, n_clusters, cluster_size)
        -> [T, P*cap] logits                                  (fused.py:82-93)
    block_sparse_logits_argmax(hs, w_perm_flat, ci, vocab_maps_flat, ...)
        -> ([T, P] per-probe max logits, [T, P] vocab ids)    (fused.py:96-116)
    block_sparse_argmax_atomic(hs, w_perm_flat, ci, vocab_maps_flat, ...)
        -> [T, 1] next-token ids                              (fused.py:167-188)

``ci`` must be int64 (the dtype ``torch.topk`` returns) and ``hs`` a
contiguous [T, D] CUDA tensor, as in the reference (its asserts at
fused.py:84-85, 105-106, 177-178 are kept as AssertionError). ``block_d`` is
accepted for signature compatibility; the CUDA kernels choose their own tiling.
"""

from __future__ import annotations

import torch

from . import _lib


def _check(hs: torch.Tensor, ci: torch.Tensor, w_perm_flat: torch.Tensor):
    assert hs.dim() == 2 and hs.is_contiguous()
    assert ci.dim() == 2 and ci.dtype == torch.int64
    if not hs.is_cuda:
        raise RuntimeError("FlashHead kernels need CUDA tensors (there is no CPU path)")
    if w_perm_flat.dtype != hs.dtype:
        raise ValueError(f"w_perm dtype {w_perm_flat.dtype} != hidden dtype {hs.dtype}")
    return _lib.dtype_code(hs.dtype)


def block_sparse_logits(hs, w_perm_flat, ci, n_clusters, cluster_size, block_d=128):
    """Return [T, P*cap] logits of the probed clusters (debug path)."""
    dt = _check(hs, ci, w_perm_flat)
    T, D = hs.shape
    _, P = ci.shape
    out = torch.empty((T, P, cluster_size), dtype=hs.dtype, device=hs.device)
    ci = ci.contiguous()
    _lib.call("fh_block_sparse_logits", hs.data_ptr(), T, D, w_perm_flat.data_ptr(),
              ci.data_ptr(), P, int(n_clusters), int(cluster_size), dt, out.data_ptr(),
              _lib.stream_ptr())
    return out.view(T, P * cluster_size)


def block_sparse_logits_argmax(hs, w_perm_flat, ci, vocab_maps_flat, n_clusters, cluster_size,
                               block_d=128):
    """Return (per-probe max logits [T, P] in hs dtype, their vocab ids [T, P] int64)."""
    dt = _check(hs, ci, w_perm_flat)
    T, D = hs.shape
    _, P = ci.shape
    vm = vocab_maps_flat.to(torch.int64).contiguous()
    out_logits = torch.empty((T, P), dtype=hs.dtype, device=hs.device)
    out_vocab = torch.empty((T, P), dtype=torch.int64, device=hs.device)
    ci = ci.contiguous()
    _lib.call("fh_block_sparse_logits_argmax", hs.data_ptr(), T, D, w_perm_flat.data_ptr(),
              ci.data_ptr(), P, vm.data_ptr(), int(n_clusters), int(cluster_size), dt,
              out_logits.data_ptr(), out_vocab.data_ptr(), _lib.stream_ptr())
    return out_logits, out_vocab


def block_sparse_argmax_atomic(hs, w_perm_flat, ci, vocab_maps_flat, n_clusters, cluster_size,
                               block_d=128):
    """Single-pass block-sparse logits + per-probe max + cross-probe argmax:
    [T, 1] int64 next-token ids; tied logits resolve to the smallest vocab id."""
    dt = _check(hs, ci, w_perm_flat)
    T, D = hs.shape
    _, P = ci.shape
    vm = vocab_maps_flat.to(torch.int64).contiguous()
    out = torch.empty((T,), dtype=torch.int64, device=hs.device)
    ci = ci.contiguous()
    _lib.call("fh_block_sparse_argmax_atomic", hs.data_ptr(), T, D, w_perm_flat.data_ptr(),
              ci.data_ptr(), P, vm.data_ptr(), int(n_clusters), int(cluster_size), dt,
              out.data_ptr(), _lib.stream_ptr())
    return out.view(T, 1)
