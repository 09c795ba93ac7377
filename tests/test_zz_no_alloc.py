"""The allocation-free density entry point, called through the C ABI.

y3b_density_accumulate_noalloc exists for hosts that cannot allocate device
memory while they run (an MD engine's per-timestep force loop, a server that
reserves its memory at start-up): it uses a fixed scratch array inside the
library instead of a caller workspace.  Its results must equal those of
y3b_density_accumulate, including on a second call that finds the previous
call's data still in the shared scratch array.  This file is collected last.
"""


import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
NOALLOC_SCRATCH_BYTES = 16 * 1024 * 1024  # Y3B_NOALLOC_SCRATCH_BYTES in include/ye3t_b200.h


def _with_workspace(lib, code, values, centers, atoms):
    E = values.shape[0]
    C = int(np.prod(values.shape[1:]))
    out = torch.empty((atoms,) + tuple(values.shape[1:]), dtype=values.dtype, device=DEV)
    nbytes = int(lib.y3b_density_accumulate_workspace_bytes(E, atoms))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    rc = lib.y3b_density_accumulate(code, values.data_ptr(), centers.data_ptr(), E, C, atoms, ws.data_ptr(),
                                    nbytes, out.data_ptr(), None, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.y3b_last_error()
    return out


def _without_allocation(lib, code, values, centers, atoms, status):
    E = values.shape[0]
    C = int(np.prod(values.shape[1:]))
    out = torch.empty((atoms,) + tuple(values.shape[1:]), dtype=values.dtype, device=DEV)
    rc = lib.y3b_density_accumulate_noalloc(code, values.data_ptr(), centers.data_ptr(), E, C, atoms,
                                            out.data_ptr(), status.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.y3b_last_error()
    return out


def test_noalloc_density_matches_workspace_entry_point_twice():
    from ye3t_b200 import _native
    lib = _native.lib()
    rng = np.random.default_rng(2027)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    # call 1: complex128, many short rows plus one long row
    E1, N1, C1 = 60000, 5000, 48
    c1 = rng.integers(0, N1, size=E1)
    c1[:3000] = 17
    v1 = torch.as_tensor(rng.normal(size=(E1, C1)) + 1j * rng.normal(size=(E1, C1)), device=DEV)
    t1 = torch.as_tensor(c1, device=DEV)
    # call 2: float64, different sizes, so stale scratch contents from call 1 would show
    E2, N2, C2 = 41000, 7000, 31
    c2 = rng.integers(0, N2, size=E2)
    v2 = torch.as_tensor(rng.normal(size=(E2, C2)), device=DEV)
    t2 = torch.as_tensor(c2, device=DEV)
    for (v, t, N) in ((v1, t1, N1), (v2, t2, N2)):
        code = _native.dtype_code(v.dtype)
        got = _without_allocation(lib, code, v, t, N, status)
        ref = _with_workspace(lib, code, v, t, N)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        # both entry points run the same deterministic kernels on the same data
        assert torch.equal(got, ref)


def test_noalloc_density_rejects_problems_beyond_its_scratch():
    from ye3t_b200 import _native
    lib = _native.lib()
    E, N = 2_000_000, 100_000
    assert lib.y3b_density_accumulate_workspace_bytes(E, N) > NOALLOC_SCRATCH_BYTES
    rc = lib.y3b_density_accumulate_noalloc(_native.F64, None, None, E, 4, N, None, None,
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == -3  # Y3B_ERR_WORKSPACE
    assert b"scratch" in lib.y3b_last_error()
