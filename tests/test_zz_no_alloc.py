"""anvil_gemm_requant_noalloc through the C-ABI, against anvil_gemm_requant (marked gpu).

The no-allocation entry point serves callers that cannot let this library allocate device memory; it must give
exactly what the allocating entry point gives. Each case calls it twice in a row (the two calls share the
library's static status words, so the second call also shows that a call starts from cleared words), and an
overflowing checked call followed by a clean one shows the words are cleared between calls. Integer outputs:
the tolerance is exact equality, as everywhere in these tests. The file is named to be collected last.
"""
import ctypes

import numpy as np
import pytest

from anvil.runtime import cuda as C

pytestmark = pytest.mark.gpu


def _noalloc():
    lib = C.load_library()
    f = lib.anvil_gemm_requant_noalloc
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    f.argtypes = [vp, vp, vp, i64, i64, i64, ctypes.c_int32, ctypes.c_int32, ctypes.c_uint32, vp]
    f.restype = ctypes.c_int
    return f


def _operands(torch, m, n, k, seed):
    from anvil.frontend.numerics import fixed_point
    rng = np.random.default_rng(seed)
    a = rng.integers(-127, 128, (m, k))
    b = rng.integers(-127, 128, (k, n))
    (mult,), s = fixed_point([float(rng.uniform(2 ** -12, 2 ** -6))], [k * 127 * 127])
    ta = torch.tensor(a, dtype=torch.int8, device="cuda")
    tbt = torch.tensor(b.T.copy(), dtype=torch.int8, device="cuda")
    return ta, tbt, mult, s


@pytest.mark.parametrize("m,n,k", [(256, 256, 256), (1000, 300, 768), (130, 70, 48), (77, 33, 19)])
@pytest.mark.parametrize("flags", [0, C.F_CHECKED, C.F_CHECKED | C.F_SIMT])
def test_noalloc_matches_allocating_entry_point(m, n, k, flags):
    import torch
    assert torch.cuda.is_available()
    f = _noalloc()
    ta, tbt, mult, s = _operands(torch, m, n, k, m + n + k)
    stream = torch.cuda.current_stream().cuda_stream
    want = torch.empty((m, n), dtype=torch.int8, device="cuda")
    C.gemm_requant(ta.data_ptr(), tbt.data_ptr(), want.data_ptr(), m, n, k, mult, s, flags, stream)
    torch.cuda.synchronize()
    for _ in range(2):                                           # two calls in a row
        got = torch.full((m, n), 99, dtype=torch.int8, device="cuda")
        C.check(f(ta.data_ptr(), tbt.data_ptr(), got.data_ptr(), m, n, k, mult, s, flags, stream or None),
                "anvil_gemm_requant_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(got, want)


def test_noalloc_status_words_cleared_between_calls():
    import torch
    f = _noalloc()
    m, n, k = 64, 64, 64
    stream = torch.cuda.current_stream().cuda_stream
    big = torch.full((m, k), 127, dtype=torch.int8, device="cuda")
    bt = torch.full((n, k), 127, dtype=torch.int8, device="cuda")
    out = torch.empty((m, n), dtype=torch.int8, device="cuda")
    rc = f(big.data_ptr(), bt.data_ptr(), out.data_ptr(), m, n, k, 1 << 20, 4, C.F_CHECKED, stream or None)
    with pytest.raises(OverflowError):                           # acc * M leaves int32: the words record it
        C.check(rc, "anvil_gemm_requant_noalloc")
    zero = torch.zeros((m, k), dtype=torch.int8, device="cuda")
    rc = f(zero.data_ptr(), bt.data_ptr(), out.data_ptr(), m, n, k, 1 << 20, 4, C.F_CHECKED, stream or None)
    C.check(rc, "anvil_gemm_requant_noalloc")                   # cleared at the start of this call
    torch.cuda.synchronize()
    assert not out.any()


def test_noalloc_rejects_bad_arguments():
    f = _noalloc()
    with pytest.raises(ValueError):
        C.check(f(None, None, None, 0, 1, 1, 1, 0, 0, None), "anvil_gemm_requant_noalloc")


@pytest.mark.parametrize("flags", [0, C.F_CHECKED])
def test_both_entry_points_report_the_same_status(flags):
    """On operands whose products leave int32 both entry points return the same status for the same flags: the
    overflow (OverflowError) when checked, success when unchecked; and they write the same bytes."""
    import torch
    f = _noalloc()
    m, n, k = 64, 64, 64
    stream = torch.cuda.current_stream().cuda_stream
    a = torch.full((m, k), 127, dtype=torch.int8, device="cuda")
    bt = torch.full((n, k), 127, dtype=torch.int8, device="cuda")
    outs, codes = [], []
    for call in ("alloc", "noalloc"):
        out = torch.zeros((m, n), dtype=torch.int8, device="cuda")
        if call == "alloc":
            rc = C.load_library().anvil_gemm_requant(a.data_ptr(), bt.data_ptr(), out.data_ptr(), m, n, k, 1 << 20, 4,
                                                     flags, stream or None)
        else:
            rc = f(a.data_ptr(), bt.data_ptr(), out.data_ptr(), m, n, k, 1 << 20, 4, flags, stream or None)
        torch.cuda.synchronize()
        outs.append(out.cpu())
        codes.append(rc)
    assert codes[0] == codes[1] == (-5 if flags else 0)
    assert torch.equal(outs[0], outs[1])
