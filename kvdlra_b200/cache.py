"""``BugStreamingCache`` -- the streaming compressed-KV cache on B200.

Drop-in for kvdlra's ``BugStreamingCache`` / ``BugStreamingLayer``
(src/kvdlra/cache/bug_cache.py:301-1938): same constructor, the same
``transformers`` ``Cache`` / ``CacheLayerMixin`` surface (``update``,
``get_mask_sizes``, ``get_seq_length``, ``ingesting``, ``consolidate``,
``frozen_scoring``, ``stored_state_numel`` ...), the same state semantics, but
the state lives in device buffers laid out for batched sm_100a kernels and
every step of the path (tier copies, surprise scoring, top-h selection, BUG
step, coordinate carry, reconstruction, factored decode) runs in the CUDA
library ``libkvdlra_b200.so`` through its C ABI.  There is no CPU fallback.

Layout: one device "group" per cache holds the state of all layers and all
sequences of a batch -- problem ``p = layer * batch + b`` -- so one absorb step
of ``consolidate()`` is one batched launch sequence over every (layer,
sequence) problem.  Verbatim tiers are token-major ``[P][slot][H*D]`` in the
model dtype (feature index ``head*D + d``, the reference's feature order);
the basis is ``[P][n][rank]`` fp32, coordinates ``[P][slot][rank]`` fp32.

In scope (bug_cache.py): retention ``"fifo"`` and ``"lowrank_surprise"``, the
surprise-selected exact tier with span boost and the warm-up seed, chunked
ingest, decode, frozen scoring, ``theta`` truncation.  The research variants
(attention-scored retention, PolarQuant / CodeBUG tiers, merge, Q-BUG
whitening, ``hh_retain=False``) keep their constructor validation and raise
``NotImplementedError``.
"""

from __future__ import annotations

import ctypes as C
import logging
import math
from collections.abc import Iterator
from contextlib import contextmanager
from typing import Any

import torch
from torch import Tensor, nn
from transformers.cache_utils import Cache, CacheLayerMixin

from . import _native as N

logger = logging.getLogger(__name__)

__all__ = ["BugStreamingCache", "BugStreamingLayer", "RopeAngles"]

RETENTION_MODES = ("fifo", "attn", "energy", "lowrank_surprise", "blend")
_IN_SCOPE_RETENTION = ("fifo", "lowrank_surprise")


class RopeAngles:
    """The model rotary's inverse frequencies and ``attention_scaling``.

    Kernels form each angle as the rotary module does -- one fp32 product
    ``position * inv_freq`` -- and scale cos/sin by ``attention_scaling``; the
    inverse rotation divides by its square (bug_cache.py:169-214, 263-272).
    Accepts a rotary module (``model.model.rotary_emb``) or explicit values."""

    def __init__(self, rotary_emb: nn.Module | None = None, *, inv_freq: Tensor | None = None,
                 attention_scaling: float | None = None) -> None:
        if rotary_emb is not None:
            inv_freq = getattr(rotary_emb, "inv_freq", None)
            if inv_freq is None:
                raise ValueError("rotary module has no inv_freq buffer")
            attention_scaling = float(getattr(rotary_emb, "attention_scaling", 1.0))
        if inv_freq is None:
            raise ValueError("RopeAngles needs a rotary module or inv_freq")
        self.inv_freq = inv_freq.detach().to(torch.float32).flatten().cpu()
        self.scaling = 1.0 if attention_scaling is None else float(attention_scaling)
        self.scale_sq = self.scaling**2
        self._dev: dict[str, Tensor] = {}

    def on(self, device: torch.device) -> Tensor:
        key = str(device)
        t = self._dev.get(key)
        if t is None:
            t = self.inv_freq.to(device).contiguous()
            self._dev[key] = t
        return t


def _validate(rank: int, coord_budget: int, recent_window: int, absorb_block: int, n_sink: int,
              prefill_block_size: int, retention: str, score_decay: float, surprise_blend: float,
              quant_bits: int | None, quant_budget: int, hh_budget: int, hh_select: str,
              hh_neighbor: int, hh_retain: bool, seed_hh_warmup: bool, w_key: Any, merge: bool,
              coord_codebook: Any, anchor_rank: int, anchor_seal_absorbs: int,
              code_budget: int) -> None:
    """The reference constructor's checks, same order and messages
    (bug_cache.py:342-494), then the scope check of this implementation."""
    if rank < 0 or coord_budget < 0:
        raise ValueError("rank and coord_budget must be >= 0")
    if recent_window < 1:
        raise ValueError(f"recent_window must be >= 1, got {recent_window}")
    if absorb_block < 1:
        raise ValueError(f"absorb_block must be >= 1, got {absorb_block}")
    if n_sink < 0:
        raise ValueError(f"n_sink must be >= 0, got {n_sink}")
    if prefill_block_size < 1:
        raise ValueError(f"prefill_block_size must be >= 1, got {prefill_block_size}")
    if retention not in RETENTION_MODES:
        raise ValueError(f"retention must be one of {RETENTION_MODES}, got {retention!r}")
    if not 0.0 < score_decay <= 1.0:
        raise ValueError(f"score_decay must be in (0, 1], got {score_decay}")
    if not 0.0 <= surprise_blend <= 1.0:
        raise ValueError(f"surprise_blend must be in [0, 1], got {surprise_blend}")
    if quant_budget < 0:
        raise ValueError(f"quant_budget must be >= 0, got {quant_budget}")
    if (quant_bits is None) != (quant_budget == 0):
        raise ValueError("quant_bits and quant_budget (> 0) must be set together")
    if quant_bits is not None and not 1 <= quant_bits <= 8:
        raise ValueError(f"quant_bits must be in [1, 8], got {quant_bits}")
    if hh_budget < 0:
        raise ValueError(f"hh_budget must be >= 0, got {hh_budget}")
    if hh_select not in ("attn", "surprise"):
        raise ValueError(f"hh_select must be 'attn' or 'surprise', got {hh_select!r}")
    if hh_neighbor < 0:
        raise ValueError(f"hh_neighbor must be >= 0, got {hh_neighbor}")
    if hh_neighbor > 0 and hh_select != "surprise":
        raise ValueError("hh_neighbor (span expansion) requires hh_select='surprise'")
    if not hh_retain and hh_budget < 1:
        raise ValueError(
            "hh_retain=False (select-and-discard ablation) requires hh_budget >= 1: "
            "with hh_budget=0 the SLASH path is disabled entirely and the config "
            "silently degenerates to plain BUG"
        )
    if not hh_retain and hh_select != "surprise":
        raise ValueError(
            "hh_retain=False requires hh_select='surprise': a discarded tier is "
            "invisible to attention, so attention-mass selection is incoherent"
        )
    if hh_budget > 0 and hh_select == "attn" and retention != "attn":
        raise ValueError(
            "hh_budget > 0 with hh_select='attn' (SLASH exact heavy-hitters) "
            "requires retention='attn'"
        )
    lowrank_enabled = rank >= 1 and coord_budget >= 1
    if quant_budget > 0 and not lowrank_enabled:
        raise ValueError("quant_budget > 0 requires an enabled low-rank middle")
    if hh_budget > 0 and not lowrank_enabled:
        raise ValueError("hh_budget > 0 requires an enabled low-rank middle")
    if w_key is not None and not lowrank_enabled:
        raise ValueError("w_key (query-metric whitening) requires an enabled low-rank middle")
    if w_key is not None and coord_codebook is not None:
        raise ValueError("w_key and the CodeBUG frozen anchor are mutually exclusive")
    if seed_hh_warmup and (coord_codebook is not None or quant_budget > 0 or merge):
        raise ValueError(
            "seed_hh_warmup operates on the fp32 low-rank tail only; it is not "
            "combined with a coded/quant tier (coord_codebook/quant_budget) or merge"
        )
    if merge and not lowrank_enabled:
        raise ValueError("merge requires an enabled low-rank middle")
    if merge and quant_budget > 0:
        raise ValueError("merge and the quantized tier are mutually exclusive")
    if merge and retention == "lowrank_surprise":
        raise ValueError("merge and retention='lowrank_surprise' are mutually exclusive")
    if coord_codebook is not None:
        if not lowrank_enabled:
            raise ValueError("coord_codebook requires an enabled low-rank middle")
        if code_budget < 1:
            raise ValueError("coord_codebook requires code_budget >= 1")
    elif code_budget > 0:
        raise ValueError("code_budget > 0 requires coord_codebook")
    # ---- scope of this implementation
    unsupported = []
    if retention not in _IN_SCOPE_RETENTION:
        unsupported.append(f"retention={retention!r}")
    if quant_bits is not None:
        unsupported.append("the PolarQuant tier (quant_bits/quant_budget)")
    if coord_codebook is not None:
        unsupported.append("the CodeBUG coded tier (coord_codebook)")
    if merge:
        unsupported.append("merge")
    if w_key is not None:
        unsupported.append("Q-BUG key whitening (w_key)")
    if not hh_retain:
        unsupported.append("hh_retain=False")
    if unsupported:
        raise NotImplementedError(
            "kvdlra_b200 implements the surprise-selected streaming path only; "
            "not supported: " + ", ".join(unsupported)
        )


class _Group:
    """Device state of every (layer, sequence) problem of one cache."""

    def __init__(self, spec: dict, n_layers: int, batch: int, num_heads: int, head_dim: int,
                 dtype: torch.dtype, device: torch.device, rope: RopeAngles,
                 ring_cap: int) -> None:
        self.spec = spec
        self.n_layers, self.batch = n_layers, batch
        self.P = n_layers * batch
        self.H, self.D = num_heads, head_dim
        self.n = num_heads * head_dim
        self.dtype, self.device = dtype, device
        self.rope = rope
        self.inv_freq = rope.on(device)
        self.lowrank = spec["rank"] >= 1 and spec["coord_budget"] >= 1
        self.rank = max(1, spec["rank"])
        self.h = spec["hh_budget"]
        self.max_block = max(spec["absorb_block"], spec["prefill_block_size"])
        self.ring_cap = 0
        self.w_cap = 0
        self.t: dict[str, Tensor] = {}
        P, n, r = self.P, self.n, self.rank
        dev = device
        self.t["sink_k"] = torch.zeros(P, max(1, spec["n_sink"]), n, dtype=dtype, device=dev)
        self.t["sink_v"] = torch.zeros_like(self.t["sink_k"])
        hh = max(1, self.h)
        self.t["hh_k"] = torch.zeros(2, P, hh, n, dtype=dtype, device=dev)
        self.t["hh_v"] = torch.zeros_like(self.t["hh_k"])
        self.t["hh_pos"] = torch.zeros(2, P, hh, dtype=torch.int32, device=dev)
        self.t["u_k"] = torch.zeros(2, P, n, r, dtype=torch.float32, device=dev)
        self.t["u_v"] = torch.zeros_like(self.t["u_k"])
        self.t["sig_k"] = torch.zeros(P, r, dtype=torch.float32, device=dev)
        self.t["sig_v"] = torch.zeros_like(self.t["sig_k"])
        self.t["r_k"] = torch.zeros(P, dtype=torch.int32, device=dev)
        self.t["r_v"] = torch.zeros_like(self.t["r_k"])
        self.t["status"] = torch.zeros(4, dtype=torch.int32, device=dev)
        self._grow_ring(ring_cap, [])
        self._grow_w(max(64, self.max_block * 2), [])
        self._ws: Tensor | None = None
        self._dec_ws: Tensor | None = None
        self._chunk_ws: torch.Tensor | None = None

    # ------------------------------------------------------------ capacity

    def _grow_ring(self, cap: int, live: list[tuple[int, int, int]]) -> None:
        """(Re)allocate the ring with ``cap`` slots; ``live`` lists (layer, head,
        len) regions to move to slot 0 of the new buffer."""
        old_k, old_v = self.t.get("ring_k"), self.t.get("ring_v")
        new_k = torch.zeros(self.P, cap, self.n, dtype=self.dtype, device=self.device)
        new_v = torch.zeros_like(new_k)
        B = self.batch
        for layer, head, length in live:
            if length > 0 and old_k is not None:
                sl = slice(layer * B, (layer + 1) * B)
                new_k[sl, :length] = old_k[sl, head : head + length]
                new_v[sl, :length] = old_v[sl, head : head + length]
        self.t["ring_k"], self.t["ring_v"] = new_k, new_v
        self.ring_cap = cap
        self._ws = None

    def _grow_w(self, cap: int, live: list[tuple[int, int]]) -> None:
        """(Re)allocate coordinate storage with ``cap`` slots, keeping (layer, len) rows."""
        P, r = self.P, self.rank
        ck = torch.zeros(P, cap, r, dtype=torch.float32, device=self.device)
        cv = torch.zeros_like(ck)
        pos = torch.zeros(P, cap, dtype=torch.int32, device=self.device)
        sur = torch.zeros(P, cap, dtype=torch.float32, device=self.device)
        B = self.batch
        for layer, length in live:
            if length > 0 and "c_k" in self.t:
                sl = slice(layer * B, (layer + 1) * B)
                ck[sl, :length] = self.t["c_k"][sl, :length]
                cv[sl, :length] = self.t["c_v"][sl, :length]
                pos[sl, :length] = self.t["mid_pos"][sl, :length]
                sur[sl, :length] = self.t["mid_surprise"][sl, :length]
        self.t.update(c_k=ck, c_v=cv, mid_pos=pos, mid_surprise=sur)
        self.w_cap = cap
        self._ws = None
        self._dec_ws = None

    def ensure(self, layers: list["BugStreamingLayer"], ring_need: int, w_need: int) -> None:
        if ring_need > self.ring_cap:
            cap = max(ring_need, int(self.ring_cap * 1.5))
            self._grow_ring(cap, [(ly.layer_idx_in_group, ly._ctr.ring_head, ly._ctr.ring_len)
                                  for ly in layers])
            for ly in layers:
                ly._ctr.ring_head = 0
        if w_need > self.w_cap:
            cap = max(w_need, int(self.w_cap * 1.5))
            self._grow_w(cap, [(ly.layer_idx_in_group, ly._ctr.w_len) for ly in layers])

    # ----------------------------------------------------------- C structs

    def config(self, n_problems: int) -> N.Config:
        s = self.spec
        cfg = N.Config()
        cfg.n_problems = n_problems
        cfg.num_heads, cfg.head_dim = self.H, self.D
        cfg.dtype = N.dtype_code(self.dtype)
        cfg.rank = self.rank
        cfg.coord_budget = s["coord_budget"] if self.lowrank else 0
        cfg.recent_window, cfg.absorb_block = s["recent_window"], s["absorb_block"]
        cfg.n_sink, cfg.prefill_block_size = s["n_sink"], s["prefill_block_size"]
        cfg.retention = (N.KVD_RETENTION_FIFO if s["retention"] == "fifo"
                         else N.KVD_RETENTION_LOWRANK_SURPRISE)
        cfg.hh_budget, cfg.hh_neighbor = self.h, s["hh_neighbor"]
        cfg.seed_hh_warmup = int(s["seed_hh_warmup"])
        cfg.has_theta = int(s["theta"] is not None)
        cfg.theta = float(s["theta"] or 0.0)
        cfg.rope_scaling = self.rope.scaling
        cfg.inv_freq = self.inv_freq.data_ptr()
        cfg.ring_cap, cfg.w_cap, cfg.max_block = self.ring_cap, self.w_cap, self.max_block
        return cfg

    def buffers(self, p0: int) -> N.Buffers:
        """Buffer pointers offset to problem ``p0`` (a sub-range view)."""
        t = self.t
        b = N.Buffers()

        def at(x: Tensor, idx: tuple = ()) -> int:
            v = x[idx] if idx else x
            return v.data_ptr() + p0 * v.stride(0) * v.element_size()

        b.sink_k, b.sink_v = at(t["sink_k"]), at(t["sink_v"])
        b.ring_k, b.ring_v = at(t["ring_k"]), at(t["ring_v"])
        for s in (0, 1):
            b.hh_k[s] = at(t["hh_k"], (s,))
            b.hh_v[s] = at(t["hh_v"], (s,))
            b.hh_pos[s] = at(t["hh_pos"], (s,))
            b.u_k[s] = at(t["u_k"], (s,))
            b.u_v[s] = at(t["u_v"], (s,))
        b.sig_k, b.sig_v = at(t["sig_k"]), at(t["sig_v"])
        b.r_k, b.r_v = at(t["r_k"]), at(t["r_v"])
        b.c_k, b.c_v = at(t["c_k"]), at(t["c_v"])
        b.mid_pos, b.mid_surprise = at(t["mid_pos"]), at(t["mid_surprise"])
        b.status = t["status"].data_ptr()
        return b

    def workspace(self) -> tuple[int, int]:
        cfg = self.config(self.P)
        need = int(N.lib().kvd_workspace_bytes(C.byref(cfg)))
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._ws.data_ptr(), self._ws.numel()

    def decode_workspace(self, count: int, hq: int) -> tuple[int, int]:
        cfg = self.config(self.P)
        need = int(N.lib().kvd_decode_workspace_bytes(C.byref(cfg), count, hq))
        if self._dec_ws is None or self._dec_ws.numel() < need:
            self._dec_ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._dec_ws.data_ptr(), self._dec_ws.numel()

    def chunk_workspace(self, count: int, hq: int, q_len: int) -> tuple[int, int]:
        cfg = self.config(self.P)
        need = int(N.lib().kvd_chunk_attention_workspace_bytes(C.byref(cfg), count, hq, q_len))
        if self._chunk_ws is None or self._chunk_ws.numel() < need:
            self._chunk_ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._chunk_ws.data_ptr(), self._chunk_ws.numel()

    def stream(self) -> int:
        return N.stream_ptr(self.device)

    def check_status(self) -> None:
        b = self.buffers(0)
        N.call(self.device, "kvd_check_status", C.byref(b), self.stream())


class BugStreamingLayer(CacheLayerMixin):  # type: ignore[misc]
    """One layer's streaming-BUG KV state (bug_cache.py:301-1685) on device.

    Stand-alone layers (constructed directly, as the reference's tests do) own
    a one-layer device group; layers created by :class:`BugStreamingCache`
    share the cache's group so ``consolidate()`` batches across layers."""

    is_sliding = False
    is_compileable = False

    def __init__(
        self,
        rope: Any,
        rank: int,
        coord_budget: int,
        recent_window: int = 64,
        absorb_block: int = 32,
        n_sink: int = 4,
        theta: float | None = None,
        prefill_block_size: int = 128,
        retention: str = "fifo",
        score_decay: float = 0.97,
        surprise_blend: float = 0.5,
        quant_bits: int | None = None,
        quant_budget: int = 0,
        quant_bank: Any = None,
        hh_budget: int = 0,
        hh_select: str = "attn",
        hh_neighbor: int = 0,
        hh_retain: bool = True,
        seed_hh_warmup: bool = False,
        w_key: Any = None,
        merge: bool = False,
        coord_codebook: Any = None,
        anchor_rank: int = 0,
        anchor_seal_absorbs: int = 4,
        code_budget: int = 0,
        *,
        _owner: "BugStreamingCache | None" = None,
        _layer_idx: int = 0,
    ) -> None:
        super().__init__()
        _validate(rank, coord_budget, recent_window, absorb_block, n_sink, prefill_block_size,
                  retention, score_decay, surprise_blend, quant_bits, quant_budget, hh_budget,
                  hh_select, hh_neighbor, hh_retain, seed_hh_warmup, w_key, merge, coord_codebook,
                  anchor_rank, anchor_seal_absorbs, code_budget)
        self.rope = rope if isinstance(rope, RopeAngles) else RopeAngles(rope)
        self.rank, self.coord_budget = rank, coord_budget
        self.recent_window, self.absorb_block = recent_window, absorb_block
        self.n_sink, self.theta = n_sink, theta
        self.prefill_block_size = prefill_block_size
        self.retention = retention
        self.score_decay = score_decay
        self.hh_budget, self.hh_select, self.hh_neighbor = hh_budget, hh_select, hh_neighbor
        self.hh_retain = hh_retain
        self.seed_hh_warmup = seed_hh_warmup
        self.lowrank_enabled = rank >= 1 and coord_budget >= 1
        self.hh_enabled = hh_budget >= 1 and self.lowrank_enabled
        self.track_positions = self.lowrank_enabled and retention != "fifo"
        self.track_surprise = self.lowrank_enabled and retention == "lowrank_surprise"
        self._spec = dict(rank=rank, coord_budget=coord_budget, recent_window=recent_window,
                          absorb_block=absorb_block, n_sink=n_sink, prefill_block_size=prefill_block_size,
                          retention=retention, hh_budget=hh_budget if self.hh_enabled else 0,
                          hh_neighbor=hh_neighbor, seed_hh_warmup=seed_hh_warmup, theta=theta)
        self._owner = _owner
        self.layer_idx_in_group = _layer_idx
        self._group: _Group | None = None
        self._mode = "normal"
        self._ctr = N.Counters()
        self.cumulative_length = 0
        self._reset_state()

    # ----------------------------------------------------------------- state

    def _reset_state(self) -> None:
        self._ctr = N.Counters()
        self._ctr.ingest_mode = int(self._mode == "ingest")
        self._started = False
        self._r_cache: tuple[int, int] | None = None

    @property
    def cumulative_length(self) -> int:  # type: ignore[override]
        return int(self._ctr.cumulative_length)

    @cumulative_length.setter
    def cumulative_length(self, v: int) -> None:
        self._ctr.cumulative_length = int(v)

    def lazy_initialization(self, key_states: Tensor, value_states: Tensor) -> None:
        if not key_states.is_cuda:
            raise RuntimeError(
                "kvdlra_b200.BugStreamingLayer runs on CUDA devices only (no CPU fallback); "
                f"got a tensor on {key_states.device}"
            )
        self.dtype, self.device = key_states.dtype, key_states.device
        self.num_heads = int(key_states.shape[1])
        self.head_dim = int(key_states.shape[3])
        self.n_features = self.num_heads * self.head_dim
        self.batch = int(key_states.shape[0])
        if self._owner is not None:
            self._group = self._owner._group_for(key_states)
            if self._group.batch != self.batch:
                raise ValueError(f"batch size changed from {self._group.batch} to {self.batch}")
        else:
            t = int(key_states.shape[2])
            self._group = _Group(self._spec, 1, self.batch, self.num_heads, self.head_dim,
                                 self.dtype, self.device, self.rope,
                                 ring_cap=max(t, self.recent_window + self.absorb_block + t))
        self.is_initialized = True

    def _group_layers(self) -> list["BugStreamingLayer"]:
        if self._owner is not None:
            return self._owner._bug_layers()
        return [self]

    def _p0(self) -> int:
        assert self._group is not None
        return self.layer_idx_in_group * self._group.batch

    def _cfg_buf(self) -> tuple[N.Config, N.Buffers]:
        g = self._group
        assert g is not None
        return g.config(g.batch), g.buffers(self._p0())

    # --------------------------------------------------------------- lengths

    def _sink_len(self) -> int:
        return int(self._ctr.sink_len)

    def _recent_len(self) -> int:
        return int(self._ctr.ring_len)

    def _f_len(self) -> int:
        return int(self._ctr.w_len)

    def _q_len(self) -> int:
        return 0

    def _hh_len(self) -> int:
        return int(self._ctr.hh_len)

    def _hh_attended_len(self) -> int:
        return self._hh_len()

    def _mid_len(self) -> int:
        return self._hh_attended_len() + self._q_len() + self._f_len()

    def attended_length(self) -> int:
        """Tokens attention currently sees (sinks + middle + recent)."""
        return self._sink_len() + self._mid_len() + self._recent_len()

    def _post_update_lengths(self, query_length: int) -> tuple[int, int, int]:
        """bug_cache.py:695-721: predicted (sink, mid, recent) after an update."""
        if self.cumulative_length == 0:
            return 0, 0, query_length
        recent = self._recent_len() + query_length
        mid = self._mid_len()
        mid_cap = self.coord_budget + self.hh_budget
        while recent >= self.recent_window + self.absorb_block:
            recent -= self.absorb_block
            if self.lowrank_enabled:
                mid = min(mid_cap, mid + self.absorb_block)
        return self._sink_len(), mid, recent

    def get_mask_sizes(self, query_length: int) -> tuple[int, int]:  # type: ignore[override]
        """bug_cache.py:1579-1595."""
        if isinstance(query_length, Tensor):  # tolerate cache_position tensors
            query_length = int(query_length.shape[0])
        if self._mode in ("score", "ingest"):
            attended = self.attended_length()
            return attended + query_length, self.cumulative_length - attended
        sink, mid, recent = self._post_update_lengths(query_length)
        kv_length = sink + mid + recent
        return kv_length, self.cumulative_length + query_length - kv_length

    def get_seq_length(self) -> int:
        """*Cumulative* token count -- keeps true positions advancing."""
        return self.cumulative_length

    def get_max_cache_shape(self) -> int:
        return -1

    def reset(self) -> None:
        self._reset_state()
        g = self._group
        if g is not None:
            p0 = self._p0()
            g.t["r_k"][p0 : p0 + g.batch].zero_()
            g.t["r_v"][p0 : p0 + g.batch].zero_()
            g.t["status"].zero_()

    # ---------------------------------------------------------------- update

    def update(self, key_states: Tensor, value_states: Tensor, *args: object,
               **kwargs: object) -> tuple[Tensor, Tensor]:
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        if key_states.shape[0] != self.batch:
            raise NotImplementedError(
                f"BugStreamingLayer was initialised for batch size {self.batch}, got {key_states.shape[0]}"
            )
        q_len = int(key_states.shape[2])
        if self.cumulative_length == 0:
            return self._prefill(key_states, value_states)
        if self._mode == "score":
            return self._score_forward(key_states, value_states)
        if self._mode == "ingest":
            return self._ingest_chunk(key_states, value_states)
        if q_len != 1:
            raise NotImplementedError(
                "BugStreamingCache supports single-shot pre-fill + one-token decode "
                f"steps only, got q_len={q_len} with {self.cumulative_length} cached "
                "tokens (chunked/continued pre-fill would desync the streaming state)."
            )
        return self._decode_step(key_states, value_states)

    def _check_kv(self, k: Tensor, v: Tensor) -> tuple[Tensor, Tensor]:
        if k.dtype != self.dtype or v.dtype != self.dtype:
            raise ValueError(f"cache dtype is {self.dtype}, got {k.dtype}/{v.dtype}")
        if k.stride(3) != 1:
            k = k.contiguous()
        if v.stride(3) != 1:
            v = v.contiguous()
        return k, v

    def _prefill(self, key_states: Tensor, value_states: Tensor) -> tuple[Tensor, Tensor]:
        """bug_cache.py:1431-1481 (returns the input K/V: full prefill attention)."""
        g = self._group
        assert g is not None
        k, v = self._check_kv(key_states, value_states)
        t = int(k.shape[2])
        mid = max(0, t - min(self.n_sink, t) - min(self.recent_window, t - min(self.n_sink, t)))
        g.ensure(self._group_layers(), t, min(self.coord_budget, mid) + g.max_block + 1)
        self._ctr.ingest_mode = int(self._mode == "ingest")
        cfg, buf = self._cfg_buf()
        ws, wsb = g.workspace()
        N.call(g.device, "kvd_prefill", C.byref(cfg), C.byref(buf), C.byref(self._ctr), N.hf_view(k),
               N.hf_view(v), ws, wsb, g.stream())
        self._started = True
        self._r_cache = None
        return key_states, value_states

    def _append(self, k: Tensor, v: Tensor) -> None:
        g = self._group
        assert g is not None
        k, v = self._check_kv(k, v)
        q = int(k.shape[2])
        g.ensure(self._group_layers(), self._recent_len() + q, 0)
        cfg, buf = self._cfg_buf()
        N.call(g.device, "kvd_append", C.byref(cfg), C.byref(buf), C.byref(self._ctr), N.hf_view(k),
               N.hf_view(v), g.stream())

    def _ingest_chunk(self, key_states: Tensor, value_states: Tensor) -> tuple[Tensor, Tensor]:
        """bug_cache.py:1404-1423: append to the ring, defer the absorb.  When
        the owning model answers attention with the factored kernels and the
        shape has a chunk kernel, the chunk's own K/V come back tagged with
        this layer instead of the dense peek."""
        self._append(key_states, value_states)
        if self._chunk_factored():
            from .attention import tag_step

            return tag_step(key_states, self), value_states
        return self._decode_peek()

    def _score_forward(self, key_states: Tensor, value_states: Tensor) -> tuple[Tensor, Tensor]:
        """bug_cache.py:1390-1402: ``[retained | window]`` without mutation
        (the window as the factored chunk kernel's tail when the model
        selected it)."""
        k, v = self._check_kv(key_states, value_states)
        if self._chunk_factored():
            from .attention import tag_step

            return tag_step(k, self), v
        return self._decode_peek(tail=(k, v))

    def _chunk_factored(self) -> bool:
        """Whether chunk queries of this layer go to the factored chunk kernel:
        the model selected the factored attention and the library has a chunk
        kernel for this shape (bf16, head_dim 64, rank <= 32)."""
        own = self._owner
        if own is None or not own._factored_decode():
            return False
        hq = getattr(own._model_config, "num_attention_heads", None)
        if hq is None:
            return False
        g = self._group
        assert g is not None
        return bool(N.lib().kvd_chunk_attention_supported(C.byref(g.config(g.P)), int(hq)))

    def _w_need(self) -> int:
        g = self._group
        assert g is not None
        grad = max(0, self._recent_len() - self.recent_window + 1)
        return min(self.coord_budget, self._f_len() + grad + self._hh_len()) + g.max_block + 1

    def consolidate(self) -> None:
        """bug_cache.py:1425-1429 for this layer only."""
        g = self._group
        if g is None or not self._started:
            return
        if self._recent_len() < self.recent_window + self.absorb_block:
            return
        g.ensure(self._group_layers(), 0, self._w_need())
        cfg, buf = self._cfg_buf()
        ws, wsb = g.workspace()
        N.call(g.device, "kvd_consolidate", C.byref(cfg), C.byref(buf), C.byref(self._ctr), ws, wsb,
               g.stream())
        self._r_cache = None

    def _absorb_block_into_stream(self, m: int | None = None) -> None:
        """Graduate one absorb block if the ring is over-full (bug_cache.py:725-750)."""
        if m is not None and m != self.absorb_block:
            raise NotImplementedError("blocks graduate in units of absorb_block")
        g = self._group
        assert g is not None
        g.ensure(self._group_layers(), 0, self._w_need())
        cfg, buf = self._cfg_buf()
        ws, wsb = g.workspace()
        N.call(g.device, "kvd_absorb_block", C.byref(cfg), C.byref(buf), C.byref(self._ctr), ws, wsb,
               g.stream())
        self._r_cache = None

    def _decode_step(self, key_states: Tensor, value_states: Tensor) -> tuple[Tensor, Tensor]:
        """bug_cache.py:1483-1494.  When the owning model answers decode steps
        with the factored kernel (:func:`kvdlra_b200.attention.enable_factored_decode`),
        the dense peek is skipped: the step's own K/V come back tagged with
        this layer and the model's attention call reads the compressed state."""
        self._append(key_states, value_states)
        self.consolidate()
        if self._owner is not None and self._owner._factored_decode():
            from .attention import tag_step

            return tag_step(key_states, self), value_states
        return self._decode_peek()

    def _decode_peek(self, tail: tuple[Tensor, Tensor] | None = None) -> tuple[Tensor, Tensor]:
        """``[sinks | hh | RoPE(U_k C_k) | recent (| tail)]`` in HF layout
        (bug_cache.py:1496-1575), assembled by the peek kernels."""
        g = self._group
        assert g is not None
        tl = 0 if tail is None else int(tail[0].shape[2])
        L = self.attended_length() + tl
        out_k = torch.empty(self.batch, self.num_heads, L, self.head_dim, dtype=self.dtype, device=self.device)
        out_v = torch.empty_like(out_k)
        cfg, buf = g.config(g.P), g.buffers(0)
        tk = N.hf_view(tail[0] if tail else None)
        tv = N.hf_view(tail[1] if tail else None)
        N.call(g.device, "kvd_peek", C.byref(cfg), C.byref(buf), C.byref(self._ctr), self._p0(),
               self.batch, N.hf_view(out_k), N.hf_view(out_v), tk, tv,
               g.stream())
        return out_k, out_v

    # -------------------------------------------------------- factored decode

    def _head_range(self, heads: tuple[int, int] | None, hq: int) -> tuple[int, int, int]:
        """(first KV head, KV heads, query heads of the whole cache) of a call
        answering ``hq`` query heads of KV heads ``heads`` (all when None)."""
        h0, hc = (0, self.num_heads) if heads is None else (int(heads[0]), int(heads[1]))
        if h0 < 0 or hc < 1 or h0 + hc > self.num_heads or hq % hc:
            raise ValueError(f"KV heads [{h0}, {h0 + hc}) of {self.num_heads} cannot answer {hq} query heads")
        return h0, hc, hq // hc * self.num_heads

    def factored_attention(self, query: Tensor, scaling: float | None = None,
                           heads: tuple[int, int] | None = None) -> Tensor:
        """Decode attention of one post-RoPE query token per sequence,
        ``query`` ``(B, Hq, D)`` or ``(B, Hq, 1, D)``, against the retained cache
        without materialising the middle.  Returns ``(B, Hq, D)``; equal to
        softmax attention over :meth:`_decode_peek` up to rounding.

        ``heads=(h0, hc)`` answers only KV heads ``[h0, h0 + hc)``: ``query``
        then holds their query heads (grouped as in the model) and the result
        is the matching slice of the full call's (head-sharded attention)."""
        g = self._group
        assert g is not None
        q = query.reshape(self.batch, -1, self.head_dim)
        if q.dtype != self.dtype:
            raise ValueError(f"query dtype {q.dtype} != cache dtype {self.dtype}")
        q = q.contiguous()
        hq = int(q.shape[1])
        h0, hc, hq_all = self._head_range(heads, hq)
        out = torch.empty_like(q)
        sc = (1.0 / math.sqrt(self.head_dim)) if scaling is None else float(scaling)
        cfg, buf = g.config(g.P), g.buffers(0)
        ws, wsb = g.decode_workspace(self.batch, hq_all)
        if heads is None:
            N.call(g.device, "kvd_factored_decode", C.byref(cfg), C.byref(buf), C.byref(self._ctr),
                   self._p0(), self.batch, q.data_ptr(), hq, sc,
                   out.data_ptr(), ws, wsb, g.stream())
        else:
            N.call(g.device, "kvd_factored_decode_heads", C.byref(cfg), C.byref(buf), C.byref(self._ctr),
                   self._p0(), self.batch, h0, hc, q.data_ptr(), hq, sc,
                   out.data_ptr(), ws, wsb, g.stream())
        return out

    def factored_chunk_attention(self, query: Tensor, scaling: float | None = None,
                                 tail: tuple[Tensor, Tensor] | None = None,
                                 heads: tuple[int, int] | None = None) -> Tensor:
        """Attention of a chunk of post-RoPE queries ``(B, Hq, q, D)`` against
        the retained cache, causal over the last ``q`` keys, without
        materialising the middle tier: ingest (the chunk is the end of the
        ring, ``tail`` None) or frozen scoring (the chunk is ``tail``, not
        appended).  Returns ``(B, q, Hq, D)``; equal to softmax attention over
        :meth:`_decode_peek` (with the tail) and the bottom-right causal mask
        up to bf16 rounding.  ``heads=(h0, hc)`` answers only KV heads
        ``[h0, h0 + hc)`` (query heads of those only; ``tail`` holds every KV
        head), as :meth:`factored_attention` does."""
        g = self._group
        assert g is not None
        if query.dim() != 4 or query.shape[0] != self.batch or query.shape[3] != self.head_dim:
            raise ValueError(f"expected a ({self.batch}, Hq, q, {self.head_dim}) query, got {tuple(query.shape)}")
        if query.dtype != self.dtype:
            raise ValueError(f"query dtype {query.dtype} != cache dtype {self.dtype}")
        q = query if query.stride(3) == 1 else query.contiguous()
        hq, q_len = int(q.shape[1]), int(q.shape[2])
        h0, hc, hq_all = self._head_range(heads, hq)
        out = torch.empty(self.batch, q_len, hq, self.head_dim, dtype=self.dtype, device=self.device)
        sc = (1.0 / math.sqrt(self.head_dim)) if scaling is None else float(scaling)
        tk = tv = None
        if tail is not None:
            tk, tv = self._check_kv(tail[0], tail[1])
        cfg, buf = g.config(g.P), g.buffers(0)
        ws, wsb = g.chunk_workspace(self.batch, hq_all, q_len)
        if heads is None:
            N.call(g.device, "kvd_factored_chunk_attention", C.byref(cfg), C.byref(buf), C.byref(self._ctr),
                   self._p0(), self.batch, q.data_ptr(), q.stride(0), q.stride(1), q.stride(2), hq, q_len, sc,
                   N.hf_view(tk), N.hf_view(tv), out.data_ptr(), ws, wsb, g.stream())
        else:
            N.call(g.device, "kvd_factored_chunk_attention_heads", C.byref(cfg), C.byref(buf),
                   C.byref(self._ctr), self._p0(), self.batch, h0, hc, q.data_ptr(), q.stride(0), q.stride(1),
                   q.stride(2), hq, q_len, sc, N.hf_view(tk), N.hf_view(tv), out.data_ptr(), ws, wsb,
                   g.stream())
        return out

    # ------------------------------------------------------------ state views

    def _ranks(self) -> tuple[int, int]:
        if self._r_cache is None:
            g = self._group
            assert g is not None
            p = self._p0()
            self._r_cache = (int(g.t["r_k"][p]), int(g.t["r_v"][p]))
        return self._r_cache

    def _rows(self, name: str, length: int, b: int = 0, start: int = 0) -> Tensor:
        g = self._group
        assert g is not None
        x = g.t[name][self._p0() + b, start : start + length]  # (len, n)
        return x.transpose(0, 1)

    @property
    def sink_k(self) -> Tensor | None:
        return self._rows("sink_k", self._sink_len()) if self._started else None

    @property
    def sink_v(self) -> Tensor | None:
        return self._rows("sink_v", self._sink_len()) if self._started else None

    @property
    def recent_k(self) -> Tensor | None:
        return self._rows("ring_k", self._recent_len(), start=self._ctr.ring_head) if self._started else None

    @property
    def recent_v(self) -> Tensor | None:
        return self._rows("ring_v", self._recent_len(), start=self._ctr.ring_head) if self._started else None

    def _hh(self, name: str, b: int = 0) -> Tensor | None:
        if not self.hh_enabled or self._ctr.n_absorbs == 0 and self._hh_len() == 0:
            return None
        g = self._group
        assert g is not None
        return g.t[name][self._ctr.hh_sel, self._p0() + b, : self._hh_len()]

    @property
    def hh_k(self) -> Tensor | None:
        x = self._hh("hh_k")
        return None if x is None else x.transpose(0, 1)

    @property
    def hh_v(self) -> Tensor | None:
        x = self._hh("hh_v")
        return None if x is None else x.transpose(0, 1)

    @property
    def hh_pos(self) -> Tensor | None:
        x = self._hh("hh_pos")
        return None if x is None else x.to(torch.int64)

    def _basis(self, name: str, r: int, b: int = 0) -> Tensor | None:
        if not self._ctr.seeded:
            return None
        g = self._group
        assert g is not None
        return g.t[name][self._ctr.u_sel, self._p0() + b, :, :r]

    @property
    def u_k(self) -> Tensor | None:
        return self._basis("u_k", self._ranks()[0]) if self._ctr.seeded else None

    @property
    def u_v(self) -> Tensor | None:
        return self._basis("u_v", self._ranks()[1]) if self._ctr.seeded else None

    def _core(self, name: str, r: int) -> Tensor | None:
        if not self._ctr.seeded:
            return None
        g = self._group
        assert g is not None
        return torch.diag(g.t[name][self._p0(), :r])

    @property
    def b_k(self) -> Tensor | None:
        return self._core("sig_k", self._ranks()[0]) if self._ctr.seeded else None

    @property
    def b_v(self) -> Tensor | None:
        return self._core("sig_v", self._ranks()[1]) if self._ctr.seeded else None

    def _coords(self, name: str, r: int) -> Tensor | None:
        if not self._ctr.seeded or self._f_len() == 0:
            return None
        g = self._group
        assert g is not None
        return g.t[name][self._p0(), : self._f_len(), :r].transpose(0, 1)

    @property
    def c_k(self) -> Tensor | None:
        return self._coords("c_k", self._ranks()[0]) if self._ctr.seeded else None

    @property
    def c_v(self) -> Tensor | None:
        return self._coords("c_v", self._ranks()[1]) if self._ctr.seeded else None

    @property
    def mid_pos(self) -> Tensor | None:
        if not self.track_positions or self._f_len() == 0:
            return None
        g = self._group
        assert g is not None
        return g.t["mid_pos"][self._p0(), : self._f_len()].to(torch.int64)

    @property
    def mid_surprise(self) -> Tensor | None:
        if not self.track_surprise or self._f_len() == 0:
            return None
        g = self._group
        assert g is not None
        return g.t["mid_surprise"][self._p0(), : self._f_len()]

    # ------------------------------------------------------------ accounting

    def stored_state_numel(self) -> int:
        """Float-equivalents of the stored per-layer state, summed over the
        batch (bug_cache.py:1609-1675; for batch 1 identical to the reference)."""
        if not self._started:
            return 0
        n = self.n_features
        total = 0
        g = self._group
        assert g is not None
        p0 = self._p0()
        rks = g.t["r_k"][p0 : p0 + self.batch].tolist() if self._ctr.seeded else [0] * self.batch
        rvs = g.t["r_v"][p0 : p0 + self.batch].tolist() if self._ctr.seeded else [0] * self.batch
        W, hh = self._f_len(), self._hh_len()
        hh_present = self.hh_enabled and (hh > 0 or self._ctr.n_absorbs > 0)
        for rk, rv in zip(rks, rvs):
            total += 2 * n * self._sink_len() + 2 * n * self._recent_len()
            if self._ctr.seeded:
                total += n * rk + n * rv + rk + rv  # U_k, U_v, diagonal cores
                if W > 0:
                    total += rk * W + rv * W
            if hh_present:
                total += 2 * n * hh + hh  # verbatim tier + hh_pos
            if self.track_positions:
                total += W
            if self.track_surprise:
                total += W
        return int(total)

    def workspace_numel(self) -> int:
        """The reference caches a dense middle reconstruction; this
        implementation rebuilds it on demand and caches nothing."""
        return 0

    # ------------------------------------------------------ lock-step support

    def state_dict(self, b: int = 0) -> dict[str, Any]:
        """Host copy of sequence ``b``'s state in the reference's layouts
        (feature-by-token), for comparisons and re-synchronisation."""
        g = self._group
        assert g is not None
        p = self._p0() + b
        out: dict[str, Any] = {"counters": self._ctr.as_tuple()}
        rk, rv = (int(g.t["r_k"][p]), int(g.t["r_v"][p]))
        W, hh = self._f_len(), self._hh_len()
        out["sink_k"] = g.t["sink_k"][p, : self._sink_len()].T.float().cpu()
        out["recent_k"] = g.t["ring_k"][p, self._ctr.ring_head : self._ctr.ring_head + self._recent_len()].T.float().cpu()
        out["recent_v"] = g.t["ring_v"][p, self._ctr.ring_head : self._ctr.ring_head + self._recent_len()].T.float().cpu()
        out["hh_k"] = g.t["hh_k"][self._ctr.hh_sel, p, :hh].T.float().cpu()
        out["hh_v"] = g.t["hh_v"][self._ctr.hh_sel, p, :hh].T.float().cpu()
        out["hh_pos"] = g.t["hh_pos"][self._ctr.hh_sel, p, :hh].long().cpu()
        out["u_k"] = g.t["u_k"][self._ctr.u_sel, p, :, :rk].cpu()
        out["u_v"] = g.t["u_v"][self._ctr.u_sel, p, :, :rv].cpu()
        out["sigma_k"] = g.t["sig_k"][p, :rk].cpu()
        out["sigma_v"] = g.t["sig_v"][p, :rv].cpu()
        out["c_k"] = g.t["c_k"][p, :W, :rk].T.cpu()
        out["c_v"] = g.t["c_v"][p, :W, :rv].T.cpu()
        out["mid_pos"] = g.t["mid_pos"][p, :W].long().cpu()
        out["mid_surprise"] = g.t["mid_surprise"][p, :W].cpu()
        return out

    def load_state(self, st: dict[str, Any], b: int = 0) -> None:
        """Overwrite sequence ``b``'s tiers, basis and coordinates from host
        arrays in the reference layouts (feature-by-token).  Lengths must
        match this layer's counters; used to re-synchronise a lock-step
        comparison after a flagged near-tie."""
        g = self._group
        assert g is not None
        p = self._p0() + b
        dev = self.device

        def t(x: Any, dtype: torch.dtype) -> Tensor:
            return torch.as_tensor(x).to(device=dev, dtype=dtype)

        hh = int(st["hh_pos"].shape[0])
        W = int(st["mid_pos"].shape[0]) if st.get("mid_pos") is not None else int(st["c_k"].shape[1])
        if hh != self._hh_len() or W != self._f_len():
            raise ValueError(f"state lengths (hh={hh}, W={W}) differ from the layer's "
                             f"({self._hh_len()}, {self._f_len()})")
        sel, us = self._ctr.hh_sel, self._ctr.u_sel
        if hh:
            g.t["hh_k"][sel, p, :hh] = t(st["hh_k"], self.dtype).T
            g.t["hh_v"][sel, p, :hh] = t(st["hh_v"], self.dtype).T
            g.t["hh_pos"][sel, p, :hh] = t(st["hh_pos"], torch.int32)
        if st.get("u_k") is not None:
            rk, rv = int(st["u_k"].shape[1]), int(st["u_v"].shape[1])
            g.t["u_k"][us, p].zero_()
            g.t["u_v"][us, p].zero_()
            g.t["u_k"][us, p, :, :rk] = t(st["u_k"], torch.float32)
            g.t["u_v"][us, p, :, :rv] = t(st["u_v"], torch.float32)
            g.t["sig_k"][p, :rk] = t(st["sigma_k"], torch.float32)
            g.t["sig_v"][p, :rv] = t(st["sigma_v"], torch.float32)
            g.t["r_k"][p], g.t["r_v"][p] = rk, rv
            if W:
                g.t["c_k"][p, :W, :rk] = t(st["c_k"], torch.float32).T
                g.t["c_v"][p, :W, :rv] = t(st["c_v"], torch.float32).T
        if W and st.get("mid_pos") is not None:
            g.t["mid_pos"][p, :W] = t(st["mid_pos"], torch.int32)
        if W and st.get("mid_surprise") is not None:
            g.t["mid_surprise"][p, :W] = t(st["mid_surprise"], torch.float32)
        self._r_cache = None


class BugStreamingCache(Cache):
    """Model-level streaming-BUG cache (bug_cache.py:1688-1938), one
    :class:`BugStreamingLayer` per model layer over one shared device group.

    Pass as ``past_key_values`` to ``model(...)`` / ``model.generate(...)``.
    Besides the reference API it offers batched whole-cache entry points
    (:meth:`ingest_all`, :meth:`decode_all`) that step every layer with one
    launch sequence, and factored decode attention
    (:meth:`BugStreamingLayer.factored_attention`)."""

    def __init__(
        self,
        model: Any,
        rank: int = 128,
        coord_budget: int = 1024,
        recent_window: int = 64,
        absorb_block: int = 32,
        n_sink: int = 4,
        theta: float | None = None,
        prefill_block_size: int = 128,
        retention: str = "fifo",
        score_decay: float = 0.97,
        surprise_blend: float = 0.5,
        quant_bits: int | None = None,
        quant_budget: int = 0,
        quant_seed: int = 0,
        hh_budget: int = 0,
        hh_select: str = "attn",
        hh_neighbor: int = 0,
        hh_retain: bool = True,
        seed_hh_warmup: bool = False,
        w_key: Any = None,
        merge: bool = False,
        coord_codebook: Any = None,
        anchor_rank: int = 0,
        anchor_seal_absorbs: int = 4,
        code_budget: int = 0,
        *,
        num_layers: int | None = None,
        rope: RopeAngles | None = None,
    ) -> None:
        if rope is None:
            base = getattr(model, "model", model)
            rotary = getattr(base, "rotary_emb", None)
            if rotary is None:
                raise ValueError(
                    f"could not find a `rotary_emb` module on {type(model).__name__}; "
                    "BugStreamingCache needs the model's own rotary embedding for the "
                    "exact RoPE round trip"
                )
            rope = RopeAngles(rotary)
        if num_layers is None:
            num_layers = int(model.config.num_hidden_layers)
        self._retention = retention
        self._rope = rope
        self._model_config = getattr(model, "config", None)
        kw = dict(rank=rank, coord_budget=coord_budget, recent_window=recent_window,
                  absorb_block=absorb_block, n_sink=n_sink, theta=theta,
                  prefill_block_size=prefill_block_size, retention=retention,
                  score_decay=score_decay, surprise_blend=surprise_blend, quant_bits=quant_bits,
                  quant_budget=quant_budget, hh_budget=hh_budget, hh_select=hh_select,
                  hh_neighbor=hh_neighbor, hh_retain=hh_retain, seed_hh_warmup=seed_hh_warmup,
                  w_key=w_key, merge=merge, coord_codebook=coord_codebook,
                  anchor_rank=anchor_rank, anchor_seal_absorbs=anchor_seal_absorbs,
                  code_budget=code_budget)
        layers = [BugStreamingLayer(rope, _owner=self, _layer_idx=i, **kw) for i in range(num_layers)]
        self._group: _Group | None = None
        super().__init__(layers=layers)

    # -------------------------------------------------------------- plumbing

    def _group_for(self, key_states: Tensor) -> _Group:
        if self._group is None:
            first: BugStreamingLayer = self.layers[0]  # type: ignore[assignment]
            t = int(key_states.shape[2])
            self._group = _Group(first._spec, len(self.layers), int(key_states.shape[0]),
                                 int(key_states.shape[1]), int(key_states.shape[3]),
                                 key_states.dtype, key_states.device, self._rope,
                                 ring_cap=max(t, first.recent_window + first.absorb_block + t))
        return self._group

    def _factored_decode(self) -> bool:
        from .attention import uses_factored_decode

        return uses_factored_decode(self._model_config)

    def _bug_layers(self) -> list[BugStreamingLayer]:
        return [ly for ly in self.layers if isinstance(ly, BugStreamingLayer)]

    def reset(self) -> None:
        """Empty every layer (device buffers stay allocated for reuse)."""
        for ly in self._bug_layers():
            ly.reset()

    def _set_mode(self, mode: str) -> None:
        for ly in self._bug_layers():
            ly._mode = mode

    @contextmanager
    def attach(self, model: Any) -> Iterator[None]:
        """Attention-scored retention hook (bug_cache.py:1807-1862): a no-op
        for the in-scope retention rules."""
        yield

    @contextmanager
    def frozen_scoring(self) -> Iterator[None]:
        """Non-mutating ``[retained | window]`` scoring (bug_cache.py:1871-1882)."""
        self._set_mode("score")
        try:
            yield
        finally:
            self._set_mode("normal")

    @contextmanager
    def ingesting(self) -> Iterator[None]:
        """Chunked pre-fill mode (bug_cache.py:1884-1895)."""
        self._set_mode("ingest")
        try:
            yield
        finally:
            self._set_mode("normal")

    def consolidate(self) -> None:
        """Run every layer's deferred absorb (bug_cache.py:1897-1900).  When all
        layers are at the same point of the schedule -- the normal case after a
        chunk forward -- the whole cache is consolidated by one batched call."""
        layers = [ly for ly in self._bug_layers() if ly._started]
        if not layers:
            return
        g = self._group
        first = layers[0]
        same = (len(layers) == len(self.layers)
                and all(ly._ctr.as_tuple() == first._ctr.as_tuple() for ly in layers))
        if not same or g is None:
            for ly in layers:
                ly.consolidate()
            return
        if first._recent_len() < first.recent_window + first.absorb_block:
            return
        g.ensure(layers, 0, first._w_need())
        ctr = first._ctr.clone()
        cfg, buf = g.config(g.P), g.buffers(0)
        ws, wsb = g.workspace()
        N.call(g.device, "kvd_consolidate", C.byref(cfg), C.byref(buf), C.byref(ctr), ws, wsb,
               g.stream())
        for ly in layers:
            ly._ctr.copy_from(ctr)
            ly._r_cache = None

    # ------------------------------------------------- batched whole-cache API

    def ingest_all(self, keys: Tensor, values: Tensor, *, peek: bool = True) -> tuple[Tensor, Tensor] | None:
        """One ingest chunk for every layer at once: ``keys``/``values``
        ``(layers, B, H, q, D)`` post-RoPE.  The first chunk prefills (as
        ``update`` would), later chunks append to the ring; then the whole
        cache is consolidated.  Returns the dense retained K/V of every layer
        ``(layers*B, H, L, D)`` when ``peek`` (what ``update`` returns per layer)."""
        Ls, B, H, q, D = keys.shape
        if Ls != len(self.layers):
            raise ValueError(f"expected {len(self.layers)} layers, got {Ls}")
        k = keys.reshape(Ls * B, H, q, D)
        v = values.reshape(Ls * B, H, q, D)
        layers = self._bug_layers()
        first = layers[0]
        if not first.is_initialized:
            for ly in layers:
                ly.lazy_initialization(keys[0], values[0])
        g = self._group
        assert g is not None
        ctr = first._ctr.clone()
        ctr.ingest_mode = 1
        cfg, buf = g.config(g.P), g.buffers(0)
        if ctr.cumulative_length == 0:
            mid = max(0, q - min(first.n_sink, q) - min(first.recent_window, q - min(first.n_sink, q)))
            g.ensure(layers, q, min(first.coord_budget, mid) + g.max_block + 1)
            cfg, buf = g.config(g.P), g.buffers(0)
            ws, wsb = g.workspace()
            N.call(g.device, "kvd_prefill", C.byref(cfg), C.byref(buf), C.byref(ctr), N.hf_view(k),
                   N.hf_view(v), ws, wsb, g.stream())
            for ly in layers:
                ly._ctr.copy_from(ctr)
                ly._started = True
                ly._r_cache = None
            out = None
        else:
            g.ensure(layers, first._recent_len() + q, 0)
            cfg, buf = g.config(g.P), g.buffers(0)
            N.call(g.device, "kvd_append", C.byref(cfg), C.byref(buf), C.byref(ctr), N.hf_view(k),
                   N.hf_view(v), g.stream())
            for ly in layers:
                ly._ctr.copy_from(ctr)
            out = self._peek_all() if peek else None
        self.consolidate()
        return out

    def _peek_all(self) -> tuple[Tensor, Tensor]:
        layers = self._bug_layers()
        first = layers[0]
        g = self._group
        assert g is not None
        L = first.attended_length()
        out_k = torch.empty(g.P, g.H, L, g.D, dtype=g.dtype, device=g.device)
        out_v = torch.empty_like(out_k)
        cfg, buf = g.config(g.P), g.buffers(0)
        empty = N.hf_view(None)
        N.call(g.device, "kvd_peek", C.byref(cfg), C.byref(buf), C.byref(first._ctr), 0, g.P,
               N.hf_view(out_k), N.hf_view(out_v), empty, empty, g.stream())
        return out_k, out_v

    def decode_all(self, keys: Tensor, values: Tensor, queries: Tensor,
                   scaling: float | None = None, heads: tuple[int, int] | None = None) -> Tensor:
        """One decode step for every layer: append ``(layers, B, H, 1, D)`` K/V,
        run due absorbs, then factored attention of ``queries`` ``(layers, B,
        Hq, D)``.  Returns ``(layers, B, Hq, D)``.  ``heads=(h0, hc)``: the
        queries and the result cover KV heads ``[h0, h0 + hc)`` only."""
        Ls, B, H, q, D = keys.shape
        layers = self._bug_layers()
        first = layers[0]
        g = self._group
        assert g is not None and q == 1
        g.ensure(layers, first._recent_len() + 1, 0)
        ctr = first._ctr.clone()
        cfg, buf = g.config(g.P), g.buffers(0)
        N.call(g.device, "kvd_append", C.byref(cfg), C.byref(buf), C.byref(ctr),
               N.hf_view(keys.reshape(Ls * B, H, 1, D)),
               N.hf_view(values.reshape(Ls * B, H, 1, D)), g.stream())
        for ly in layers:
            ly._ctr.copy_from(ctr)
        self.consolidate()
        hq = int(queries.shape[2])
        h0, hc, hq_all = first._head_range(heads, hq)
        qq = queries.reshape(Ls * B, hq, D).contiguous()
        out = torch.empty_like(qq)
        sc = (1.0 / math.sqrt(D)) if scaling is None else float(scaling)
        cfg, buf = g.config(g.P), g.buffers(0)
        ws, wsb = g.decode_workspace(g.P, hq_all)
        N.call(g.device, "kvd_factored_decode_heads", C.byref(cfg), C.byref(buf), C.byref(first._ctr), 0, g.P,
               h0, hc, qq.data_ptr(), hq, sc, out.data_ptr(), ws, wsb,
               g.stream())
        return out.reshape(Ls, B, hq, D)

    # ------------------------------------------------------------ accounting

    def stored_state_numel(self) -> int:
        """Total stored float-equivalents across layers (bug_cache.py:1916-1926)."""
        return sum(ly.stored_state_numel() for ly in self._bug_layers())

    def workspace_numel(self) -> int:
        return sum(ly.workspace_numel() for ly in self._bug_layers())

    def attended_length(self) -> int:
        if not self.layers:
            return 0
        first = self.layers[0]
        assert isinstance(first, BugStreamingLayer)
        return first.attended_length()

    def check_status(self) -> None:
        """Raise if a kernel flagged a device-side failure (synchronises)."""
        if self._group is not None:
            self._group.check_status()
