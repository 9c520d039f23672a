"""Factored decode and chunk attention behind transformers' own attention call.

In the reference, a decode step of ``LlamaAttention`` on a
``BugStreamingCache`` gets the dense retained cache back from
``past_key_values.update`` -- ``[sinks | exact tier | RoPE(U_k C_k) | ring]``
re-materialised in the model dtype (bug_cache.py:1483-1519, 1540-1575) -- and
runs stock SDPA over it.  Here the same call reaches the factored decode
kernel instead: ``enable_factored_decode(model)`` registers an attention
function under the name ``"kvdlra_factored"`` (transformers'
``AttentionInterface``) and selects it for the model.  When the model runs on
a :class:`kvdlra_b200.BugStreamingCache`, the cache's decode-step ``update``
(append, due absorbs) returns the step's own key/value tagged with the layer
instead of a dense peek, and the registered function answers the query with
``kvd_factored_decode`` over the compressed state -- keys rebuilt from the
coordinates with RoPE at each token's true position, values accumulated in
coordinate space, the verbatim tiers read in place.  Chunked ingest
(bug_cache.py:1404-1423) and frozen scoring (1390-1402) are answered the same
way by ``kvd_factored_chunk_attention`` (causal over the chunk) where the
library has a chunk kernel for the shape (bf16, head_dim 64, rank <= 32);
other shapes, the single-shot prefill and any cache that is not a
``BugStreamingCache`` go to SDPA over what ``update`` returned, exactly as
before.  ``update``'s return contract is unchanged for models that
do not select the function, so lock-step comparisons against the reference's
dense peek still hold.

An attention module carrying ``kvd_heads = (h0, hc)`` (set by
:func:`kvdlra_b200.sharding.shard_attention_heads`) answers only the query
heads of KV heads ``[h0, h0 + hc)``: the factored kernels take the head range,
SDPA takes those heads of the key/value it was given.
"""

from __future__ import annotations

from typing import Any

import torch
from transformers import AttentionInterface
from transformers.integrations.sdpa_attention import sdpa_attention_forward
from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS, AttentionMaskInterface

__all__ = ["ATTN_NAME", "enable_factored_decode", "factored_attention_forward", "uses_factored_decode"]

ATTN_NAME = "kvdlra_factored"
_TAG = "_kvdlra_layer"


def factored_attention_forward(module: torch.nn.Module, query: torch.Tensor, key: torch.Tensor,
                               value: torch.Tensor, attention_mask: torch.Tensor | None,
                               dropout: float = 0.0, scaling: float | None = None,
                               **kwargs: Any) -> tuple[torch.Tensor, None]:
    """transformers attention function: factored decode where the cache
    tagged the step, SDPA otherwise.  ``query`` is ``(B, Hq, q_len, D)``; the
    output is ``(B, q_len, Hq, D)`` as transformers expects."""
    layer = getattr(key, _TAG, None)
    heads = getattr(module, "kvd_heads", None)
    if layer is None:
        if heads is not None and key.shape[1] != heads[1]:
            h0, hc = heads
            key, value = key[:, h0 : h0 + hc], value[:, h0 : h0 + hc]
        return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout,
                                      scaling=scaling, **kwargs)
    if dropout:
        raise NotImplementedError("factored attention has no dropout (inference only)")
    mode = getattr(layer, "_mode", None)
    if mode in ("ingest", "score"):
        # a chunk (or a frozen-scoring window: its own K/V are the tail)
        tail = (key, value) if mode == "score" else None
        return layer.factored_chunk_attention(query, scaling=scaling, tail=tail, heads=heads), None
    if query.shape[2] != 1:
        raise RuntimeError("factored decode answers one query token per step")
    out = layer.factored_attention(query[:, :, 0, :], scaling=scaling, heads=heads)  # (B, Hq, D)
    return out.unsqueeze(1), None


AttentionInterface.register(ATTN_NAME, factored_attention_forward)
AttentionMaskInterface.register(ATTN_NAME, ALL_MASK_ATTENTION_FUNCTIONS["sdpa"])


def enable_factored_decode(model: Any) -> Any:
    """Select the factored decode for ``model``'s attention layers (their
    non-decode calls keep SDPA).  Returns the model."""
    if hasattr(model, "set_attn_implementation"):
        model.set_attn_implementation(ATTN_NAME)
    else:
        model.config._attn_implementation = ATTN_NAME
    return model


def uses_factored_decode(config: Any) -> bool:
    """Whether a model with this config answers decode steps through the
    factored kernel (the cache then skips its dense peek)."""
    return config is not None and getattr(config, "_attn_implementation", None) == ATTN_NAME


def tag_step(key: torch.Tensor, layer: Any) -> torch.Tensor:
    """Mark a decode step's key as belonging to ``layer`` (read by
    :func:`factored_attention_forward`)."""
    setattr(key, _TAG, layer)
    return key
