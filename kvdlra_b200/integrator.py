"""GPU augmented rank-adaptive BUG integrator (``kvd_bug_step``).

Drop-in for src/kvdlra/integrators/streaming_torch.py: ``augmented_bug_step``
(82-189), ``blocked_bug_subspace`` (192-238) and ``blocked_bug_project``
(241-258), computed by the batched sm_100a BUG-step kernel.  Inputs and
outputs are CUDA tensors; the math runs in fp32 with fp64 eigen-solves of
the small Gram matrices.
"""

from __future__ import annotations

import ctypes as C

import torch
from torch import Tensor

from . import _native as N

__all__ = ["augmented_bug_step", "blocked_bug_subspace", "blocked_bug_project", "bug_step_batched"]


def bug_step_batched(u: Tensor, sigma: Tensor, r: Tensor, block: Tensor, rank_cap: int, *,
                     theta: float | None = None) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """One BUG step on ``nb`` independent problems.

    ``u`` ``(nb, n, ld)`` fp32 basis (first ``r[i]`` columns live), ``sigma``
    ``(nb, ld)``, ``r`` ``(nb,)`` int32 (0 = seed), ``block`` ``(nb, b, n)``
    token-major fp32.  Returns ``(u_new, sigma_new, r_new, rot, m)`` where
    ``rot[i, :r_new, :r_old]`` is ``u_new^T u_old`` and ``m`` the admitted
    residual directions.  ``sigma``/``r`` are updated in place."""
    if not u.is_cuda:
        raise RuntimeError("kvdlra_b200 integrator runs on CUDA tensors only")
    nb, n, ld = u.shape
    b = int(block.shape[1])
    if rank_cap > ld:
        raise ValueError(f"rank_cap {rank_cap} exceeds the basis width {ld}")
    u = u.contiguous()
    u_out = torch.zeros_like(u)
    rot = torch.zeros(nb, ld, ld, dtype=torch.float32, device=u.device)
    m = torch.zeros(nb, dtype=torch.int32, device=u.device)
    coords = torch.zeros(nb, b, ld, dtype=torch.float32, device=u.device)
    status = torch.zeros(4, dtype=torch.int32, device=u.device)
    L = N.lib()
    wsb = int(L.kvd_bug_step_workspace_bytes(nb, n, b, ld)) + 16 * nb + 64
    ws = torch.empty(wsb, dtype=torch.uint8, device=u.device)
    N.call(u.device, "kvd_bug_step", nb, n, b, rank_cap, ld, u.data_ptr(), u_out.data_ptr(),
           sigma.data_ptr(), r.data_ptr(), block.contiguous().data_ptr(), rot.data_ptr(),
           m.data_ptr(), coords.data_ptr(), int(theta is not None), float(theta or 0.0),
           status.data_ptr(), ws.data_ptr(), wsb, N.stream_ptr(u.device))
    if int(status.sum()) != 0:
        raise N.KvdError(6, "kvd_bug_step", f"device status {status.tolist()}")
    return u_out, sigma, r, rot, m


def augmented_bug_step(u: Tensor | None, b_core: Tensor | None, block: Tensor, rank_cap: int, *,
                       theta: float | None = None) -> tuple[Tensor, Tensor, Tensor]:
    """streaming_torch.py:82-189: ``(u_new, b_new, rot)`` for a feature-by-token
    ``block`` ``(n, b)``; ``b_new`` is ``diag(sigma)``, ``rot = u_new^T u_old``."""
    if (u is None) != (b_core is None):
        raise ValueError("u and b_core must be provided together (or both None)")
    if rank_cap < 1:
        raise ValueError(f"rank_cap must be >= 1, got {rank_cap}")
    n, bsz = block.shape
    dev = block.device
    r_old = 0 if u is None else int(u.shape[1])
    ld = max(rank_cap, r_old, 1)
    U = torch.zeros(1, n, ld, dtype=torch.float32, device=dev)
    sig = torch.zeros(1, ld, dtype=torch.float32, device=dev)
    if u is not None:
        U[0, :, :r_old] = u.to(torch.float32)
        sig[0, :r_old] = torch.diagonal(b_core).to(torch.float32)
    r = torch.tensor([r_old], dtype=torch.int32, device=dev)
    x = block.to(torch.float32).T.contiguous()[None]
    u_out, sig, r, rot, _ = bug_step_batched(U, sig, r, x, rank_cap, theta=theta)
    keep = int(r[0])
    u_new = u_out[0, :, :keep].to(block.dtype)
    b_new = torch.diag(sig[0, :keep]).to(block.dtype)
    rot_out = rot[0, :keep, :r_old].to(block.dtype)
    return u_new, b_new, rot_out


def blocked_bug_subspace(M: Tensor, rank_cap: int, block_size: int = 128, *,
                         theta: float | None = None,
                         compute_dtype: torch.dtype = torch.float32) -> Tensor:
    """streaming_torch.py:192-238 (compute in fp32)."""
    if rank_cap < 1:
        raise ValueError(f"rank_cap must be >= 1, got {rank_cap}")
    if block_size < 1:
        raise ValueError(f"block_size must be >= 1, got {block_size}")
    if compute_dtype != torch.float32:
        raise NotImplementedError("the GPU integrator computes in float32")
    n, t = M.shape
    dev = M.device
    ld = rank_cap
    U = torch.zeros(1, n, ld, dtype=torch.float32, device=dev)
    sig = torch.zeros(1, ld, dtype=torch.float32, device=dev)
    r = torch.zeros(1, dtype=torch.int32, device=dev)
    mt = M.to(torch.float32).T.contiguous()  # (t, n) token-major
    for start in range(0, t, block_size):
        blk = mt[start : start + block_size][None]
        U, sig, r, _, _ = bug_step_batched(U, sig, r, blk, rank_cap, theta=theta)
    if t == 0:
        return torch.zeros(n, 1, dtype=torch.float32, device=dev)
    return U[0, :, : int(r[0])].clone()


def blocked_bug_project(M: Tensor, rank_cap: int, block_size: int = 128, *,
                        theta: float | None = None,
                        compute_dtype: torch.dtype = torch.float32) -> Tensor:
    """``U (U^T M)`` onto the tracked subspace (streaming_torch.py:241-258):
    the BUG sweep and the projection run in ``kvd_blocked_project``."""
    if not M.is_cuda:
        raise RuntimeError("kvdlra_b200 integrator runs on CUDA tensors only")
    if rank_cap < 1:
        raise ValueError(f"rank_cap must be >= 1, got {rank_cap}")
    if block_size < 1:
        raise ValueError(f"block_size must be >= 1, got {block_size}")
    if compute_dtype != torch.float32:
        raise NotImplementedError("the GPU integrator computes in float32")
    n, t = M.shape
    if t == 0:
        return M.clone()
    xt = M.T.to(torch.float32).contiguous()
    out = torch.empty_like(xt)
    L = N.lib()
    wsb = int(L.kvd_blocked_project_workspace_bytes(n, t, rank_cap, block_size)) + 256
    ws = torch.empty(wsb, dtype=torch.uint8, device=M.device)
    N.call(M.device, "kvd_blocked_project", n, t, rank_cap, block_size, 0, 0, int(theta is not None),
           float(theta or 0.0), xt.data_ptr(), out.data_ptr(), None,
           ws.data_ptr(), wsb, N.stream_ptr(M.device))
    return out.T.to(M.dtype)
