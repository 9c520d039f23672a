"""The workspace-free BUG step against the workspace one, through the C ABI.

``kvd_bug_step_noalloc`` exists for callers that may not allocate device
memory (a host runtime that owns a pre-reserved pool, or a plugin inside one):
it takes no workspace and runs in a fixed scratch array inside the library.
Here it must give the same bases, cores, ranks, carry maps and coordinates as
``kvd_bug_step`` with a caller-provided workspace, on two steps in a row (a
seeding step, then a step that builds on it), and must refuse a request larger
than its scratch with an error instead of launching.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from kvdlra_b200 import _native as N

    L = N.lib()
    vp, i32, f32 = C.c_void_p, C.c_int32, C.c_float
    L.kvd_bug_step_noalloc.argtypes = [i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp,
                                       i32, f32, vp, vp]
    L.kvd_bug_step_noalloc.restype = C.c_int
    L.kvd_bug_step_noalloc_max_scratch.restype = C.c_size_t
    return L, N


def _state(nb, n, ld, dev):
    return (torch.zeros(nb, n, ld, device=dev), torch.zeros(nb, ld, device=dev),
            torch.zeros(nb, dtype=torch.int32, device=dev))


def _step(L, N, noalloc: bool, u, sig, r, x, rank_cap):
    nb, n, ld = u.shape
    b = x.shape[1]
    dev = u.device
    u_out = torch.zeros_like(u)
    rot = torch.zeros(nb, ld, ld, device=dev)
    m = torch.zeros(nb, dtype=torch.int32, device=dev)
    coords = torch.zeros(nb, b, ld, device=dev)
    status = torch.zeros(4, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    if noalloc:
        rc = L.kvd_bug_step_noalloc(nb, n, b, rank_cap, ld, u.data_ptr(), u_out.data_ptr(),
                                    sig.data_ptr(), r.data_ptr(), x.data_ptr(), rot.data_ptr(),
                                    m.data_ptr(), coords.data_ptr(), 0, 0.0, status.data_ptr(), stream)
    else:
        wsb = int(L.kvd_bug_step_workspace_bytes(nb, n, b, ld)) + 16 * nb + 64
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
        rc = L.kvd_bug_step(nb, n, b, rank_cap, ld, u.data_ptr(), u_out.data_ptr(), sig.data_ptr(),
                            r.data_ptr(), x.data_ptr(), rot.data_ptr(), m.data_ptr(),
                            coords.data_ptr(), 0, 0.0, status.data_ptr(), ws.data_ptr(), wsb, stream)
    N.check(rc, "bug step")
    torch.cuda.synchronize(dev)
    assert int(status.sum()) == 0
    return u_out, sig, r, rot, m, coords


@pytest.mark.parametrize("nb,n,ld,rank_cap,b", [
    (6, 256, 24, 20, 16),  # every working region in shared memory
    # a 128-column block's residual SVD does not fit in shared memory: the
    # kernel keeps its working regions in the scratch array itself, so the
    # second call runs over what the first one left there
    (4, 512, 32, 32, 128),
])
def test_noalloc_step_matches_workspace_step_twice(nb: int, n: int, ld: int, rank_cap: int, b: int) -> None:
    L, N = _lib()
    dev = torch.device("cuda")
    rng = np.random.default_rng(42 + b)
    basis = np.linalg.qr(rng.standard_normal((n, 30)))[0]
    blocks = []
    for _ in range(2):
        coef = rng.standard_normal((nb, 30, b)) * (2.0 ** (-np.arange(30) / 4))[None, :, None]
        x = np.einsum("nk,pkb->pbn", basis, coef) + 0.01 * rng.standard_normal((nb, b, n))
        blocks.append(torch.from_numpy(x.astype(np.float32)).to(dev).contiguous())
    results = {}
    for noalloc in (False, True):
        u, sig, r = _state(nb, n, ld, dev)
        outs = []
        for x in blocks:  # seeding step, then a step on the new basis
            r_old = r.clone()
            u_out, sig, r, rot, m, coords = _step(L, N, noalloc, u, sig, r, x, rank_cap)
            outs.append((u_out.clone(), sig.clone(), r.clone(), rot.clone(), m.clone(),
                         coords.clone(), r_old))
            u = u_out
        results[noalloc] = outs
    for (ua, sa, ra, rota, ma, ca, r0a), (ub, sb, rb, rotb, mb, cb, r0b) in zip(results[False], results[True]):
        assert torch.equal(ra, rb) and torch.equal(ma, mb) and torch.equal(r0a, r0b)
        for i in range(nb):
            k, k0 = int(ra[i]), int(r0a[i])
            np.testing.assert_allclose(ub[i, :, :k].cpu(), ua[i, :, :k].cpu(), rtol=1e-5, atol=1e-6)
            np.testing.assert_allclose(sb[i, :k].cpu(), sa[i, :k].cpu(), rtol=1e-5, atol=1e-6)
            np.testing.assert_allclose(rotb[i, :k, :k0].cpu(), rota[i, :k, :k0].cpu(), rtol=1e-5, atol=1e-6)
            np.testing.assert_allclose(cb[i, :, :k].cpu(), ca[i, :, :k].cpu(), rtol=1e-5, atol=1e-6)


def test_noalloc_rejects_requests_beyond_its_scratch() -> None:
    L, N = _lib()
    cap = int(L.kvd_bug_step_noalloc_max_scratch())
    assert cap == 16 << 20
    nb = 4096  # far more problems than the fixed scratch holds; nothing launches
    rc = L.kvd_bug_step_noalloc(nb, 1024, 16, 32, 32, None, None, None, None, None, None, None, None,
                                0, 0.0, None, None)
    assert rc == 3  # KVD_ERR_WORKSPACE
    assert b"scratch" in L.kvd_last_error()
