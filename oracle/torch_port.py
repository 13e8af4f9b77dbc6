"""TEST INFRASTRUCTURE ONLY -- the reference's dense torch step, on host cores.

bpdecode's dense regular path is not native code: it is a handful of torch ops
(``src/bpdecode/ops.py:271-276`` for the mask, ``ops.py:301-306`` for the
commit, driven by ``batch.py:176-215``). This module restates exactly those
ops on CPU tensors so ``bench.py`` can time the reference's own CPU
implementation of the step on the GPU box's host cores (where bpdecode itself
is not installed). torch's intra-op thread pool uses every host core it is
given; the thread count is reported with the timing.
"""

from __future__ import annotations

import torch


def apply_mask_(logits: torch.Tensor, tok_next: torch.Tensor, states: torch.Tensor,
                neg_inf: float = float("-inf")) -> torch.Tensor:
    """ops.py:271-276 (dense branch of apply_mask_)."""
    s = states.long()
    broken = s < 0
    rejected = tok_next.index_select(0, s.clamp_(min=0)) == -1
    rejected |= broken.unsqueeze(1)
    return logits.masked_fill_(rejected, neg_inf)


def advance_state(tok_next: torch.Tensor, states: torch.Tensor,
                  token_ids: torch.Tensor) -> torch.Tensor:
    """ops.py:301-306 (dense branch of advance_state)."""
    s = states.long()
    t = token_ids.long()
    broken = s < 0
    nxt = tok_next[s.clamp_(min=0), t]
    return torch.where(broken, torch.full_like(nxt, -1), nxt).to(torch.int32)


def step(logits: torch.Tensor, tok_next: torch.Tensor, state: torch.Tensor,
         slots: torch.Tensor) -> torch.Tensor:
    """One ConstraintBatch step (batch.py:176-215): gather states by slot,
    mask, argmax, commit, scatter. Returns the tokens."""
    states = state[slots]
    apply_mask_(logits, tok_next, states)
    tok = logits.argmax(-1)
    state[slots] = advance_state(tok_next, state[slots], tok.to(torch.int32))
    return tok
