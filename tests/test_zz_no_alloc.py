# SPDX-License-Identifier: Apache-2.0
"""GPU: the allocation-free reuse lookup equals the allocating two-step path.

``reuse_lookup_static`` serves callers that cannot allocate device memory
when they look up the reuse cache; it keeps its comparison flags in a fixed
array inside the library.  Called through the C ABI twice in a row (the
second call must not see the first call's flags), its rows and hit index
must equal ``coords_mismatch`` + ``reuse_rows`` on the same inputs.  This
file is collected last so that a failure here comes after every other test.
"""

import ctypes

import pytest
import torch

from tests import abi

pytestmark = pytest.mark.gpu

P, I, LL = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong


def _lib():
    lib = abi.bvh_lib()
    lib.reuse_lookup_static.argtypes = [I, P, LL, P, LL, P, P, P, I, I, I, P, P, P]
    lib.reuse_lookup_static.restype = I
    return lib


def _ptrs(ts, kind=ctypes.c_void_p):
    return (kind * len(ts))(*[t.data_ptr() for t in ts])


def _two_step(lib, x, q, sx, sq, cached, rows, cols):
    """The existing path: one flag per comparison in a caller buffer."""
    n = len(sx)
    flags = torch.empty(2 * n, dtype=torch.int32, device="cuda")
    A = (ctypes.c_void_p * (2 * n))(*[t.data_ptr() for pair in zip([x] * n, [q] * n) for t in pair])
    B = (ctypes.c_void_p * (2 * n))(*[t.data_ptr() for pair in zip(sx, sq) for t in pair])
    C = (ctypes.c_longlong * (2 * n))(*[v for _ in range(n) for v in (x.numel(), q.numel())])
    assert lib.coords_mismatch(2 * n, A, B, C, flags.data_ptr(), abi.stream()) == 0
    dst = torch.full((rows, cols), -1, dtype=torch.int32, device="cuda")
    hit = torch.full((1,), -9, dtype=torch.int32, device="cuda")
    assert lib.reuse_rows(n, _ptrs(cached), flags.data_ptr(), 32, rows, cols, dst.data_ptr(), hit.data_ptr(), abi.stream()) == 0
    return dst, hit


def _static(lib, x, q, sx, sq, cached, rows, cols):
    dst = torch.full((rows, cols), -1, dtype=torch.int32, device="cuda")
    hit = torch.full((1,), -9, dtype=torch.int32, device="cuda")
    code = lib.reuse_lookup_static(
        len(sx), x.data_ptr(), x.numel(), q.data_ptr(), q.numel(), _ptrs(sx), _ptrs(sq), _ptrs(cached),
        32, rows, cols, dst.data_ptr(), hit.data_ptr(), abi.stream(),
    )
    assert code == 0
    return dst, hit


def test_static_lookup_equals_two_step_path_on_consecutive_calls():
    lib = _lib()
    g = torch.Generator(device="cuda").manual_seed(17)
    n, nq = 5000, 1200
    x = torch.randn(n, 3, device="cuda", generator=g)
    q = x[:nq].clone()
    other = x.clone()
    other[4321, 2] = torch.nextafter(other[4321, 2], torch.tensor(float("inf"), device="cuda"))
    cached = [torch.randint(0, 5000, (nq, 32), dtype=torch.int32, device="cuda", generator=g) for _ in range(4)]
    # call 1: candidates 0 and 1 differ in the support, candidate 2 matches
    sx1 = [other, other, x.clone(), x]
    sq1 = [q, q, x[:nq].clone(), q]
    # call 2: only the last candidate's query prefix differs from the first's
    # flags of call 1 set candidate 0/1 as mismatching; they must be cleared
    q2 = x[:700].clone()
    sx2 = [x, x.clone(), other]
    sq2 = [q2, q2, q2]
    results = []
    for (sx, sq, qq, rows, cols) in [(sx1, sq1, q, nq, 32), (sx2, sq2, q2, 700, 8)]:
        want = _two_step(lib, x, qq, sx, sq, cached[: len(sx)], rows, cols)
        got = _static(lib, x, qq, sx, sq, cached[: len(sx)], rows, cols)
        torch.cuda.synchronize()
        assert torch.equal(got[1], want[1])
        assert torch.equal(got[0], want[0])
        results.append(int(got[1].item()))
    assert results == [2, 0]
    # a lookup with no match leaves dst untouched and reports -1
    sx3, sq3 = [other, other], [q, q]
    want = _two_step(lib, x, q, sx3, sq3, cached[:2], nq, 32)
    got = _static(lib, x, q, sx3, sq3, cached[:2], nq, 32)
    assert int(got[1].item()) == int(want[1].item()) == -1
    assert torch.equal(got[0], want[0])


def test_static_lookup_allocates_no_device_memory():
    """After one warm-up call (which looks up the array's address), further
    calls change neither torch's allocated bytes nor the device's free bytes
    as cudaMemGetInfo reports them: every buffer is passed in."""
    lib = _lib()
    g = torch.Generator(device="cuda").manual_seed(5)
    n, nq = 4096, 1024
    x = torch.randn(n, 3, device="cuda", generator=g)
    q = x[:nq]
    sx = [x.clone(), x.clone()]
    sq = [q.clone(), q.clone()]
    sx[0][7, 1] += 1.0
    cached = [torch.randint(0, n, (nq, 32), dtype=torch.int32, device="cuda", generator=g) for _ in range(2)]
    dst = torch.full((nq, 32), -1, dtype=torch.int32, device="cuda")
    hit = torch.full((1,), -9, dtype=torch.int32, device="cuda")
    args = (2, x.data_ptr(), x.numel(), q.data_ptr(), q.numel(), _ptrs(sx), _ptrs(sq), _ptrs(cached),
            32, nq, 32, dst.data_ptr(), hit.data_ptr(), abi.stream())
    assert lib.reuse_lookup_static(*args) == 0
    torch.cuda.synchronize()
    torch_bytes = torch.cuda.memory_allocated()
    free_bytes = torch.cuda.mem_get_info()[0]
    for _ in range(8):
        assert lib.reuse_lookup_static(*args) == 0
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == torch_bytes
    assert torch.cuda.mem_get_info()[0] == free_bytes
    assert int(hit.item()) == 1
    assert torch.equal(dst, cached[1])


def test_static_lookup_rejects_more_candidates_than_its_array():
    lib = _lib()
    x = torch.zeros(10, 3, device="cuda")
    rows = torch.zeros(10, 32, dtype=torch.int32, device="cuda")
    many = [x] * 65
    dst = torch.empty(10, 32, dtype=torch.int32, device="cuda")
    code = lib.reuse_lookup_static(
        65, x.data_ptr(), x.numel(), x.data_ptr(), x.numel(), _ptrs(many), _ptrs(many), _ptrs([rows] * 65),
        32, 10, 32, dst.data_ptr(), None, abi.stream(),
    )
    assert code == -4
