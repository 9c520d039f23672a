"""ctypes binding of ``libkvdlra_b200.so`` (declared in ``include/kvdlra_b200.h``).

Only plain pointers, sizes and the C structs of the header cross this
boundary; tensors are passed as ``data_ptr()`` values.  There is no fallback:
if the library is missing or a call fails, a ``KvdError`` is raised.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libkvdlra_b200.so"

KVD_OK = 0
KVD_DTYPE_F32 = 0
KVD_DTYPE_BF16 = 1
KVD_RETENTION_FIFO = 0
KVD_RETENTION_LOWRANK_SURPRISE = 1

_ERRORS = {1: "bad argument", 2: "unsupported dtype", 3: "workspace too small", 4: "CUDA error",
           5: "device wait timed out", 6: "numerical failure"}


class KvdError(RuntimeError):
    """A kvdlra_b200 library call returned a non-zero status."""

    def __init__(self, code: int, what: str, msg: str) -> None:
        super().__init__(f"{what}: {_ERRORS.get(code, 'error')} ({code}): {msg}")
        self.code = code


class Config(C.Structure):
    _fields_ = [
        ("n_problems", C.c_int32), ("num_heads", C.c_int32), ("head_dim", C.c_int32),
        ("dtype", C.c_int32), ("rank", C.c_int32), ("coord_budget", C.c_int32),
        ("recent_window", C.c_int32), ("absorb_block", C.c_int32), ("n_sink", C.c_int32),
        ("prefill_block_size", C.c_int32), ("retention", C.c_int32), ("hh_budget", C.c_int32),
        ("hh_neighbor", C.c_int32), ("seed_hh_warmup", C.c_int32), ("has_theta", C.c_int32),
        ("theta", C.c_float), ("rope_scaling", C.c_float), ("inv_freq", C.c_void_p),
        ("ring_cap", C.c_int32), ("w_cap", C.c_int32), ("max_block", C.c_int32),
    ]


class Buffers(C.Structure):
    _fields_ = [
        ("sink_k", C.c_void_p), ("sink_v", C.c_void_p),
        ("ring_k", C.c_void_p), ("ring_v", C.c_void_p),
        ("hh_k", C.c_void_p * 2), ("hh_v", C.c_void_p * 2), ("hh_pos", C.c_void_p * 2),
        ("u_k", C.c_void_p * 2), ("u_v", C.c_void_p * 2),
        ("sig_k", C.c_void_p), ("sig_v", C.c_void_p),
        ("r_k", C.c_void_p), ("r_v", C.c_void_p),
        ("c_k", C.c_void_p), ("c_v", C.c_void_p),
        ("mid_pos", C.c_void_p), ("mid_surprise", C.c_void_p),
        ("status", C.c_void_p),
    ]


class Counters(C.Structure):
    _fields_ = [
        ("cumulative_length", C.c_int64), ("sink_len", C.c_int32), ("ring_head", C.c_int32),
        ("ring_len", C.c_int32), ("hh_len", C.c_int32), ("hh_sel", C.c_int32),
        ("u_sel", C.c_int32), ("w_len", C.c_int32), ("seeded", C.c_int32),
        ("n_absorbs", C.c_int32), ("ingest_mode", C.c_int32),
    ]

    def as_tuple(self) -> tuple:
        return tuple(getattr(self, f) for f, _ in self._fields_)

    def copy_from(self, other: "Counters") -> None:
        C.memmove(C.addressof(self), C.addressof(other), C.sizeof(Counters))

    def clone(self) -> "Counters":
        c = Counters()
        c.copy_from(self)
        return c


class HFView(C.Structure):
    _fields_ = [("ptr", C.c_void_p), ("stride_b", C.c_int64), ("stride_h", C.c_int64),
                ("stride_t", C.c_int64), ("tokens", C.c_int32)]


def hf_view(t: torch.Tensor | None) -> HFView:
    """View of a (B, H, T, D) tensor (last dim contiguous)."""
    if t is None:
        return HFView(None, 0, 0, 0, 0)
    if t.dim() != 4 or t.stride(3) != 1:
        raise ValueError(f"expected a (B, H, T, D) tensor with contiguous D, got {tuple(t.shape)}")
    return HFView(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2), t.shape[2])


_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """Load the CUDA library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("KVDLRA_B200_LIB", LIB_PATH))
    if not path.exists():
        raise RuntimeError(
            f"kvdlra_b200 CUDA library not found at {path}; build it with "
            "`python -m kvdlra_b200.build` (there is no CPU fallback)"
        )
    L = C.CDLL(str(path))
    vp, i32, sz, f32 = C.c_void_p, C.c_int32, C.c_size_t, C.c_float
    P = C.POINTER
    L.kvd_last_error.restype = C.c_char_p
    L.kvd_version.restype = C.c_int
    L.kvd_workspace_bytes.argtypes = [P(Config)]
    L.kvd_workspace_bytes.restype = sz
    L.kvd_decode_workspace_bytes.argtypes = [P(Config), i32, i32]
    L.kvd_decode_workspace_bytes.restype = sz
    L.kvd_check_status.argtypes = [P(Buffers), vp]
    L.kvd_prefill.argtypes = [P(Config), P(Buffers), P(Counters), HFView, HFView, vp, sz, vp]
    L.kvd_append.argtypes = [P(Config), P(Buffers), P(Counters), HFView, HFView, vp]
    L.kvd_consolidate.argtypes = [P(Config), P(Buffers), P(Counters), vp, sz, vp]
    L.kvd_absorb_block.argtypes = [P(Config), P(Buffers), P(Counters), vp, sz, vp]
    L.kvd_peek.argtypes = [P(Config), P(Buffers), P(Counters), i32, i32, HFView, HFView, HFView,
                           HFView, vp]
    L.kvd_factored_decode.argtypes = [P(Config), P(Buffers), P(Counters), i32, i32, vp, i32, f32,
                                      vp, vp, sz, vp]
    i64 = C.c_int64
    L.kvd_factored_chunk_attention.argtypes = [P(Config), P(Buffers), P(Counters), i32, i32, vp, i64, i64,
                                               i64, i32, i32, f32, HFView, HFView, vp, vp, sz, vp]
    L.kvd_factored_decode_heads.argtypes = [P(Config), P(Buffers), P(Counters), i32, i32, i32, i32, vp, i32,
                                            f32, vp, vp, sz, vp]
    L.kvd_factored_chunk_attention_heads.argtypes = [P(Config), P(Buffers), P(Counters), i32, i32, i32, i32, vp,
                                                     i64, i64, i64, i32, i32, f32, HFView, HFView, vp, vp, sz,
                                                     vp]
    L.kvd_chunk_attention_workspace_bytes.argtypes = [P(Config), i32, i32, i32]
    L.kvd_chunk_attention_workspace_bytes.restype = sz
    L.kvd_chunk_attention_supported.argtypes = [P(Config), i32]
    L.kvd_chunk_attention_supported.restype = C.c_int
    L.kvd_bug_step.argtypes = [i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, i32, f32,
                               vp, vp, sz, vp]
    L.kvd_bug_step_workspace_bytes.argtypes = [i32, i32, i32, i32]
    L.kvd_bug_step_workspace_bytes.restype = sz
    L.kvd_surprise.argtypes = [i32, i32, i32, i32, vp, vp, vp, vp, vp]
    L.kvd_select_topk.argtypes = [i32, i32, i32, vp, vp, vp, vp]
    L.kvd_rope_table.argtypes = [i32, vp, i32, vp, f32, i32, vp, vp, vp]
    L.kvd_profile.argtypes = [i32]
    L.kvd_profile_read.argtypes = [C.c_char_p, sz]
    L.kvd_blocked_project.argtypes = [i32, i32, i32, i32, i32, i32, i32, f32, vp, vp, vp, vp, sz, vp]
    L.kvd_blocked_project_workspace_bytes.argtypes = [i32, i32, i32, i32]
    L.kvd_blocked_project_workspace_bytes.restype = sz
    for name in ("kvd_check_status", "kvd_prefill", "kvd_append", "kvd_consolidate", "kvd_absorb_block", "kvd_peek",
                 "kvd_factored_decode", "kvd_factored_chunk_attention", "kvd_factored_decode_heads",
                 "kvd_factored_chunk_attention_heads", "kvd_bug_step", "kvd_surprise",
                 "kvd_select_topk",
                 "kvd_profile", "kvd_profile_read", "kvd_blocked_project", "kvd_rope_table"):
        getattr(L, name).restype = C.c_int
    _lib = L
    return L


def check(code: int, what: str) -> None:
    if code != KVD_OK:
        msg = lib().kvd_last_error().decode(errors="replace")
        raise KvdError(code, what, msg)


def call(device: torch.device, name: str, *args: object) -> None:
    """Call entry point ``name`` with ``device`` current (the library launches
    on, and sizes its per-device tables for, the calling thread's current
    device) and raise on a non-zero status."""
    with torch.cuda.device(device):
        check(getattr(lib(), name)(*args), name)


def profile(enable: bool) -> None:
    """Start (clearing previous totals) or stop per-kernel event timing."""
    check(lib().kvd_profile(int(enable)), "kvd_profile")


def profile_read() -> dict[str, tuple[float, int]]:
    """``{kernel: (total_ms, launches)}`` recorded since ``profile(True)``."""
    import json

    buf = C.create_string_buffer(1 << 16)
    check(lib().kvd_profile_read(buf, len(buf)), "kvd_profile_read")
    return {k: (float(v[0]), int(v[1])) for k, v in json.loads(buf.value.decode()).items()}


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return KVD_DTYPE_F32
    if dtype == torch.bfloat16:
        return KVD_DTYPE_BF16
    raise NotImplementedError(f"kvdlra_b200 supports float32 and bfloat16 caches, got {dtype}")
