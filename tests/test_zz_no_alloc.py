"""GPU: the allocation-free CGS2 entry point gives the same results as the
allocating one.

lg_cgs2_orthogonalize_noalloc exists for callers that cannot allocate device
memory where they re-orthogonalise (inside an allocator or memory-pool hook,
or under a device memory budget fixed at start-up).  It keeps its workspace in
a fixed array inside the library, so consecutive calls reuse — and must not
be disturbed by — whatever the previous call left there; the test therefore
makes two calls in a row with different inputs and compares each with the
allocating entry point.  It is collected last so that a run stopping at the
first failure has already run every other test, and it works both alone in a
fresh process and after the other tests.
"""
import ctypes

import pytest

pytestmark = pytest.mark.gpu


def _call(fn, V, ncols, w, torch):
    n, ldv = V.shape
    r = torch.empty_like(w)
    coef = torch.empty(ncols, dtype=torch.float64, device="cuda")
    norms = torch.empty(3, dtype=torch.float64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(ctypes.c_void_p(V.data_ptr()), ldv, n, ncols, ctypes.c_void_p(w.data_ptr()),
            ctypes.c_void_p(r.data_ptr()), ctypes.c_void_p(coef.data_ptr()), ctypes.c_void_p(norms.data_ptr()),
            ctypes.c_void_p(stream))
    assert rc == 0
    torch.cuda.synchronize()
    return r, coef, norms


def test_noalloc_matches_allocating_entry_point_twice():
    import torch
    from gpu_eigsh import _native

    lib = _native.lib
    for call, (n, ncols, seed) in enumerate([(200000, 61, 3), (90001, 20, 4)]):
        g = torch.Generator(device="cuda").manual_seed(seed)
        ldv = ncols + 1 if ncols % 2 else ncols + 2
        Q, _ = torch.linalg.qr(torch.randn(n, ncols, generator=g, device="cuda", dtype=torch.float64))
        V = torch.zeros(n, ldv, device="cuda", dtype=torch.float64)
        V[:, :ncols] = Q
        w = torch.randn(n, generator=g, device="cuda", dtype=torch.float64)
        ref = _call(lib.lg_cgs2_orthogonalize, V, ncols, w, torch)
        got = _call(lib.lg_cgs2_orthogonalize_noalloc, V, ncols, w, torch)
        for a, b in zip(got, ref):
            assert torch.isfinite(a).all()
            assert ((a - b).norm() / b.norm()).item() < 1e-12, f"call {call}"


def test_noalloc_call_takes_no_device_memory():
    """After the first call on the device (which loads the module and
    resolves the array), a call changes neither the device's free memory nor
    torch's allocations: the outputs are the caller's, the workspace is the
    library's fixed array."""
    import torch
    from gpu_eigsh import _native

    n, ncols = 150000, 40
    g = torch.Generator(device="cuda").manual_seed(9)
    Q, _ = torch.linalg.qr(torch.randn(n, ncols, generator=g, device="cuda", dtype=torch.float64))
    V = torch.zeros(n, ncols, device="cuda", dtype=torch.float64)
    V[:, :ncols] = Q
    w = torch.randn(n, generator=g, device="cuda", dtype=torch.float64)
    r = torch.empty_like(w)
    coef = torch.empty(ncols, dtype=torch.float64, device="cuda")
    norms = torch.empty(3, dtype=torch.float64, device="cuda")
    fn = _native.lib.lg_cgs2_orthogonalize_noalloc
    args = (ctypes.c_void_p(V.data_ptr()), ncols, n, ncols, ctypes.c_void_p(w.data_ptr()),
            ctypes.c_void_p(r.data_ptr()), ctypes.c_void_p(coef.data_ptr()), ctypes.c_void_p(norms.data_ptr()),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert fn(*args) == 0          # first call: module load and symbol address
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    stats0 = torch.cuda.memory_stats()
    for _ in range(3):
        assert fn(*args) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    stats1 = torch.cuda.memory_stats()
    assert free1 == free0, (free0, free1)
    assert stats1.get("allocation.all.allocated", 0) == stats0.get("allocation.all.allocated", 0)
    assert float(norms[2]) > 0.0


def test_noalloc_rejects_too_many_columns():
    import torch
    from gpu_eigsh import _native

    V = torch.zeros(1000, 130, device="cuda", dtype=torch.float64)
    w = torch.ones(1000, device="cuda", dtype=torch.float64)
    r = torch.empty_like(w)
    coef = torch.empty(129, device="cuda", dtype=torch.float64)
    norms = torch.empty(3, device="cuda", dtype=torch.float64)
    rc = _native.lib.lg_cgs2_orthogonalize_noalloc(V.data_ptr(), 130, 1000, 129, w.data_ptr(), r.data_ptr(),
                                                   coef.data_ptr(), norms.data_ptr(), None)
    assert rc == _native.LG_ERR_INVALID
    assert "128" in _native.last_error()
