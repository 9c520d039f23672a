"""Model-level drivers of the streaming cache: chunked prefill and greedy decode.

The protocols the reference's harness drives its caches with
(scripts/w10_frontier.py:72-91 ``_prefill_chunked``, scripts/w10_ruler.py:150-189
``_decode``): the first chunk single-shot-prefills, every later chunk is
ingested with ``logits_to_keep=1`` and absorbed by ``consolidate()`` after its
forward; decode feeds one token per forward at its true position.  Both work
on any batch of independent sequences the cache was created for (the
reference is batch 1); with :func:`kvdlra_b200.attention.enable_factored_decode`
the decode forwards answer attention with the factored kernel.
"""

from __future__ import annotations

from typing import Any

import torch

__all__ = ["prefill_chunked", "decode_greedy"]


@torch.no_grad()
def prefill_chunked(model: Any, cache: Any, ctx: torch.Tensor, chunk: int,
                    *, keep_logits: bool = False) -> torch.Tensor | None:
    """Chunked prefill of ``ctx`` ``(B, T)`` token ids into ``cache``
    (scripts/w10_frontier.py:72-91).  Returns the last position's logits of
    the last chunk ``(B, vocab)`` when ``keep_logits``."""
    t = int(ctx.shape[1])
    last = None
    with cache.ingesting():
        for start in range(0, t, chunk):
            stop = min(t, start + chunk)
            pos = torch.arange(start, stop, device=ctx.device).unsqueeze(0).expand(ctx.shape[0], -1)
            out = model(ctx[:, start:stop], past_key_values=cache, use_cache=True, position_ids=pos,
                        logits_to_keep=1)
            cache.consolidate()
            if keep_logits:
                last = out.logits[:, -1]
    return last


@torch.no_grad()
def decode_greedy(model: Any, cache: Any, first_logits: torch.Tensor, start: int, max_new: int,
                  *, forced: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Greedy decode of ``max_new`` tokens, one forward per token at its true
    position (scripts/w10_ruler.py:176-189).  ``first_logits`` ``(B, vocab)``
    picks the first token.  ``forced`` ``(B, max_new)`` feeds those tokens
    instead of the argmax (teacher forcing, for comparisons).  Returns the
    tokens fed ``(B, max_new)`` and each step's logits ``(B, max_new, vocab)``."""
    b = int(first_logits.shape[0])
    dev = first_logits.device
    nxt = first_logits.argmax(-1)
    toks, logits = [], []
    for j in range(max_new):
        cur = forced[:, j].to(dev) if forced is not None else nxt
        toks.append(cur)
        pos = torch.full((b, 1), start + j, device=dev, dtype=torch.long)
        out = model(cur[:, None], past_key_values=cache, use_cache=True, position_ids=pos)
        lg = out.logits[:, -1]
        logits.append(lg)
        nxt = lg.argmax(-1)
    return torch.stack(toks, 1), torch.stack(logits, 1)
