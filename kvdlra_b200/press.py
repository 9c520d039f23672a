"""``BUGPress`` -- the prefill low-rank KV press on B200.

Drop-in for src/kvdlra/press/bug_press.py:83-389.  At the end of pre-fill it
replaces each layer's keys and (optionally) values by their rank-``rank``
blocked-BUG reconstruction, keeping the tensor shape: per batch element the
``(bsz, H, T, D)`` tensor is factored as the feature-by-token matrix
``(H*D, T)`` (feature index ``head*D + d``); the ``n_sink`` leading columns
and the ``n_exact`` highest-norm columns after them stay exact, the rest
become ``U U^T x`` with ``U`` tracked by augmented BUG steps over blocks of
``block_size`` columns.  All of that runs in ``kvd_blocked_project`` (exact
set by radix select, BUG steps, projection); this module only moves tensors
between the HF layout and the token-major fp32 matrix the kernel takes.

The hook plumbing restates what kvpress 0.5.1 provides to the reference
(``BasePress.__call__`` hook registration, ``extract_keys_and_values`` and
``get_prerope_key_states``), since kvpress is not a dependency here.
Only the ``"torch"`` backend exists on B200 (the reference's ``"numpy"``
backend is its fp64 CPU tracker), and the ``quant_bits`` coordinate
quantisation is outside this build; both are validated exactly like the
reference and raise ``NotImplementedError`` when used.
"""

from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass, field
from typing import Any, Iterator

import torch
from torch import Tensor, nn

from . import _native as N

__all__ = ["BUGPress", "prerope_key_states"]


def _rotate_half(x: Tensor) -> Tensor:
    """``[-x2, x1]`` over the last dimension's halves (the Llama convention)."""
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def prerope_key_states(module: nn.Module, hidden_states: Tensor) -> Tensor:
    """Keys of ``hidden_states`` before RoPE, ``(bsz, H_kv, q_len, D)``: the
    attention module's key projection, split into heads, with its key norm
    when it has one (what kvpress's ``get_prerope_key_states`` computes for
    Llama-style attention)."""
    bsz, q_len, _ = hidden_states.shape
    head_dim = int(getattr(module, "head_dim"))
    k = module.k_proj(hidden_states).view(bsz, q_len, -1, head_dim).transpose(1, 2)
    k_norm = getattr(module, "k_norm", None)
    return k_norm(k) if k_norm is not None else k


class _HookedPress:
    """The part of kvpress's ``BasePress`` a press needs: ``with press(model):``
    registers :meth:`forward_hook` on every decoder layer's attention module
    and removes the hooks on exit."""

    def forward_hook(self, module: nn.Module, input: list[Tensor], kwargs: dict[str, Any],
                     output: list[Any]) -> list[Any]:  # pragma: no cover - overridden
        return output

    @contextmanager
    def __call__(self, model: nn.Module) -> Iterator[None]:
        hooks = []
        try:
            for layer in model.model.layers:
                hooks.append(layer.self_attn.register_forward_hook(self.forward_hook, with_kwargs=True))
            yield
        finally:
            for h in hooks:
                h.remove()


@dataclass
class BUGPress(_HookedPress):
    """Streaming-BUG low-rank KV press (bug_press.py:83-152 for the fields)."""

    rank: int = 32
    pre_rope: bool = True
    compress_values: bool = True
    n_sink: int = 4
    n_exact: int = 0
    backend: str = "torch"
    block_size: int = 128
    quant_bits: int | None = None
    n_features: int = field(default=512)

    def __post_init__(self) -> None:
        """The reference's constructor guards and messages (bug_press.py:154-168)."""
        if self.rank < 1:
            raise ValueError(f"rank must be >= 1, got {self.rank}")
        if self.n_sink < 0:
            raise ValueError(f"n_sink must be >= 0, got {self.n_sink}")
        if self.n_exact < 0:
            raise ValueError(f"n_exact must be >= 0, got {self.n_exact}")
        if self.backend not in ("torch", "numpy"):
            raise ValueError(f"backend must be 'torch' or 'numpy', got {self.backend!r}")
        if self.block_size < 1:
            raise ValueError(f"block_size must be >= 1, got {self.block_size}")
        if self.quant_bits is not None:
            if self.quant_bits < 1:
                raise ValueError(f"quant_bits must be >= 1, got {self.quant_bits}")
            if self.backend != "torch":
                raise ValueError("quant_bits requires backend='torch'")

    def post_init_from_model(self, model: Any) -> None:
        """``n_features = head_dim * num_kv_heads`` from the model config."""
        cfg = model.config
        head_dim = getattr(cfg, "head_dim", cfg.hidden_size // cfg.num_attention_heads)
        self.n_features = int(head_dim * cfg.num_key_value_heads)

    @property
    def compression_ratio(self) -> float:
        """Nominal ``1 - rank / n_features`` (read-only, bug_press.py:176-189)."""
        return max(0.0, 1.0 - self.rank / self.n_features)

    @compression_ratio.setter
    def compression_ratio(self, value: float) -> None:
        raise AttributeError(f"compression_ratio cannot be set for {type(self).__name__}")

    # ------------------------------------------------------------ kernels
    def _run(self, mat: Tensor, n_sink: int, n_exact: int,
             project: bool) -> tuple[Tensor | None, Tensor]:
        """``kvd_blocked_project`` on a ``(features, T)`` matrix: returns the
        token-major fp32 reconstruction ``(T, features)`` (or None) and the
        exact-column mask ``(T,)``."""
        if self.backend != "torch":
            raise NotImplementedError("the fp64 CPU tracker (backend='numpy') is not part of the B200 build")
        if self.quant_bits is not None:
            raise NotImplementedError("quantised coordinates (quant_bits) are outside the B200 press")
        if not mat.is_cuda:
            raise RuntimeError("BUGPress runs on CUDA tensors only")
        n, t = int(mat.shape[0]), int(mat.shape[1])
        dev = mat.device
        xt = mat.T.to(torch.float32).contiguous()
        out = torch.empty_like(xt) if project else None
        mask = torch.empty(t, dtype=torch.uint8, device=dev)
        L = N.lib()
        wsb = int(L.kvd_blocked_project_workspace_bytes(n, t, self.rank, self.block_size)) + 256
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
        N.call(dev, "kvd_blocked_project", n, t, self.rank, self.block_size, n_sink, n_exact, 0, 0.0,
               xt.data_ptr(), out.data_ptr() if out is not None else None,
               mask.data_ptr(), ws.data_ptr(), wsb, N.stream_ptr(dev))
        return out, mask.bool()

    def _exact_mask(self, mat: Tensor) -> Tensor:
        """Boolean ``(T,)``: the ``n_sink`` leading columns plus the top
        ``n_exact`` non-sink columns by L2 norm (bug_press.py:231-247)."""
        _, mask = self._run(mat, self.n_sink, self.n_exact, project=False)
        return mask

    def _project_lowrank(self, cols: Tensor) -> Tensor:
        """Rank-``rank`` blocked-BUG reconstruction of a ``(features, k)`` block
        (bug_press.py:249-262 with the torch backend); fp32 compute, ``cols``'s
        dtype out."""
        out, _ = self._run(cols, 0, 0, project=True)
        return out.T.to(cols.dtype)

    def _lowrank_reconstruct(self, mat: Tensor) -> Tensor:
        """Exact columns kept byte-for-byte, the rest ``U U^T x`` with ``U``
        fit on those columns only (bug_press.py:264-304)."""
        t = int(mat.shape[1])
        if t <= self.n_sink:
            return mat
        proj, mask = self._run(mat, self.n_sink, self.n_exact, project=True)
        out = mat.clone()
        low = ~mask
        if bool(low.any()):
            out[:, low] = proj[low].T.to(mat.dtype)
        return out

    def _compress_tensor(self, x: Tensor) -> Tensor:
        """Per batch element: ``(H, T, D)`` as ``(H*D, T)``, reconstruct, back
        (bug_press.py:326-339)."""
        bsz, h, t, d = x.shape
        out = torch.empty_like(x)
        for b in range(bsz):
            mat = x[b].permute(0, 2, 1).reshape(h * d, t)
            out[b] = self._lowrank_reconstruct(mat).reshape(h, d, t).permute(0, 2, 1)
        return out

    # --------------------------------------------------------------- hooks
    def forward_hook(self, module: nn.Module, input: list[Tensor], kwargs: dict[str, Any],
                     output: list[Any]) -> list[Any]:
        """Compress the layer's cache once, at the end of pre-fill
        (bug_press.py:341-372): a forward with ``q_len > 1`` (or one whose
        ``cache_position`` ends within the query) is the pre-fill."""
        hidden_states = kwargs["hidden_states"]
        q_len = hidden_states.shape[1]
        cache_position = kwargs.get("cache_position")
        if cache_position is not None:
            if cache_position[-1] > q_len:
                return output
        elif q_len <= 1:
            return output
        cache = kwargs["past_key_values"]
        layer = cache.layers[module.layer_idx]
        keys, values = layer.keys, layer.values
        keys, values = self.compress(module, hidden_states, keys, values,
                                     output[1] if len(output) > 1 else None, kwargs)
        layer.keys = keys
        layer.values = values
        return output

    def compress(self, module: nn.Module, hidden_states: Tensor, keys: Tensor, values: Tensor,
                 attentions: Tensor | None, kwargs: dict[str, Any]) -> tuple[Tensor, Tensor]:
        """Same-shape low-rank keys and values (bug_press.py:374-389); only a
        single-shot pre-fill covering the whole cache is supported."""
        q_len = hidden_states.shape[1]
        cache_len = keys.shape[2]
        if q_len != cache_len:
            raise NotImplementedError(
                "BUGPress supports only single-shot pre-fill: the compressed forward "
                f"must cover the whole cache, but q_len={q_len} != cache_len={cache_len}. "
                "Chunked/continued pre-fill would desync keys and values."
            )
        if self.pre_rope:
            cos, sin = kwargs["position_embeddings"]
            keys_pre = prerope_key_states(module, kwargs["hidden_states"])
            keys_hat = self._compress_tensor(keys_pre)
            keys = keys_hat * cos.unsqueeze(1) + _rotate_half(keys_hat) * sin.unsqueeze(1)
        else:
            keys = self._compress_tensor(keys)
        if self.compress_values:
            values = self._compress_tensor(values)
        return keys, values
