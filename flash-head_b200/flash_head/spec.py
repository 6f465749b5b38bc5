"""Speculative decoding with FlashHead token ids.

When FlashHead serves the target model's verification step it returns one
greedy token id per position instead of logits, so draft verification is an
exact comparison, done on the device by ``fh_spec_accept``
(``csrc/fh_spec.cuh``): drafts are accepted while they equal the target's id,
the first mismatch takes the target's id, and a fully accepted request gets
its bonus id. The reference does this comparison element by element in a
host loop (patches/rejection_sampler.py:55-76).
"""

from __future__ import annotations

import torch

from . import _lib

PLACEHOLDER_TOKEN_ID = -1


def _i32(t: torch.Tensor, device) -> torch.Tensor:
    return t.to(device=device, dtype=torch.int32).contiguous().view(-1)


def accept_draft_tokens(draft_ids: torch.Tensor, target_ids: torch.Tensor,
                        bonus_ids: torch.Tensor, cu_num_draft: torch.Tensor,
                        max_spec_len: int, placeholder: int = PLACEHOLDER_TOKEN_ID,
                        out: torch.Tensor | None = None) -> torch.Tensor:
    """[batch, max_spec_len + 1] int32 output ids of a verification step.

    draft_ids / target_ids: [num_drafts] flat over requests; bonus_ids:
    [batch]; cu_num_draft: [batch] inclusive prefix sum of the requests'
    draft counts (vLLM's ``cu_num_draft_tokens``). CUDA tensors."""
    dev = target_ids.device
    if dev.type != "cuda":
        raise RuntimeError("accept_draft_tokens needs CUDA tensors (there is no CPU path)")
    cu = _i32(cu_num_draft, dev)
    batch = cu.numel()
    draft, target, bonus = _i32(draft_ids, dev), _i32(target_ids, dev), _i32(bonus_ids, dev)
    if bonus.numel() != batch:
        raise ValueError(f"{bonus.numel()} bonus ids for {batch} requests")
    if draft.numel() != target.numel():
        raise ValueError(f"{draft.numel()} draft ids but {target.numel()} target ids")
    if out is None:
        out = torch.empty((batch, int(max_spec_len) + 1), dtype=torch.int32, device=dev)
    _lib.call("fh_spec_accept", draft.data_ptr() if draft.numel() else None,
              target.data_ptr() if target.numel() else None,
              bonus.data_ptr(), cu.data_ptr(), batch, int(max_spec_len), int(placeholder),
              out.data_ptr(), _lib.stream_ptr())
    return out
