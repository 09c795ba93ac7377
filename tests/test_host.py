"""Host-side checks that need no GPU: the C-ABI library loads and exports every
symbol include/ye3t_b200.h declares; bundle files round-trip; argument errors."""

import os
import re

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    src = open(os.path.join(REPO, "include", "ye3t_b200.h")).read()
    return sorted(set(re.findall(r"\b(y3b_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from ye3t_b200 import _native
    lib = _native.lib()
    declared = _declared_symbols()
    assert declared, "no declarations found"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in include/ye3t_b200.h but not exported"
    assert set(declared) == set(_native.exported_symbols())
    assert lib.y3b_abi_version() == _native.ABI_VERSION


def test_library_argument_errors_without_gpu():
    from ye3t_b200 import _native
    lib = _native.lib()
    rc = lib.y3b_cheb_exp_cos_radial_table(_native.F64, 0, 0, 0, 10, -1, 0, 0, 0)
    assert rc == -1 and b"maximum_radial_index" in lib.y3b_last_error()
    assert lib.y3b_density_accumulate_workspace_bytes(100, 10) > 0
    assert lib.y3b_density_accumulate_workspace_bytes(-1, 10) == -1
    assert lib.y3b_neighbor_workspace_bytes(1000, 30.0, 5.0) > 0
    rc = lib.y3b_ace_features(None, 0, 10, 0, 0)
    assert rc == -1


def test_bundle_round_trip(tmp_path):
    from ye3t_b200.schedules import ACEBundle
    b = ACEBundle.load(os.path.join(REPO, "ye3t_b200", "bundles", "ace_n8_l3_nu3_L0.npz"))
    p = tmp_path / "b.npz"
    b.save(str(p))
    c = ACEBundle.load(str(p))
    assert c.table_hash() == b.table_hash()
    assert c.word_count == b.word_count == 2344 and c.feature_count == 2344
    np.testing.assert_array_equal(c.word_n_map, b.word_n_map)


def test_runtime_rejects_reference_backend_and_cpu():
    import torch
    from ye3t_b200 import runtime
    with pytest.raises(ValueError):
        runtime.density_accumulate(torch.zeros(2, 2), torch.zeros(2, dtype=torch.int64), 1, backend="reference")
    with pytest.raises(ValueError):
        runtime.density_accumulate(torch.zeros(2, 2), torch.zeros(2, dtype=torch.int64), 1)
    caps = runtime.native_execution_plan_capabilities()
    assert caps["loaded"] and caps["cpu"] is False


def test_torch_ops_registered_with_fake_kernels():
    """torch.ops.ye3t_b200.*: registered at import, with fake kernels that give the output
    shapes and dtypes without running anything (what torch.compile tracing uses)."""
    import torch
    from torch._subclasses.fake_tensor import FakeTensorMode
    import ye3t_b200.torch_ops  # noqa: F401
    ops = torch.ops.ye3t_b200
    with FakeTensorMode():
        dev = "cuda"
        ev = torch.empty(11, 16, device=dev, dtype=torch.complex128)
        c = torch.empty(11, device=dev, dtype=torch.int64)
        assert ops.density_accumulate(ev, c, 5).shape == (5, 16)
        assert ops.density_accumulate_adjoint(torch.empty(5, 16, device=dev), c).shape == (11, 16)
        r = torch.empty(9, device=dev, dtype=torch.float64)
        v, d = ops.cheb_exp_cos_radial_table_with_derivative(r, r, r, 8)
        assert v.shape == d.shape == (9, 9)
        y, dy = ops.spherical_harmonics_table_with_derivative(torch.empty(9, 3, device=dev, dtype=torch.float64),
                                                             3, False, 1e-12)
        assert y.shape == (9, 16) and dy.shape == (9, 16, 3) and y.dtype == torch.complex128
        x = torch.empty(4, 7, 3, device=dev, dtype=torch.complex128)
        counts = torch.empty(6, 3, device=dev, dtype=torch.int64)
        offs = torch.empty(4, device=dev, dtype=torch.int64)
        idx = torch.empty(6, device=dev, dtype=torch.int64)
        vals = torch.empty(6, device=dev, dtype=torch.complex128)
        assert ops.symmetric_power_monomial(x, counts, offs, idx, vals).shape == (4, 7, 3)
        assert ops.symmetric_power_monomial_adjoint(torch.empty(4, 7, 3, device=dev, dtype=torch.complex128), x,
                                                    counts, offs, idx, vals).shape == x.shape
        assert ops.symmetric_power_shared_monomial(x, counts, offs, idx, idx, vals).shape == (4, 7, 3)
        bv = torch.empty(5, 2, 3, 7, device=dev, dtype=torch.complex128)
        out = ops.factorized_schedule(bv, torch.empty(13, device=dev, dtype=torch.int64),
                                      torch.empty(12, device=dev, dtype=torch.int64),
                                      torch.empty(20, 3, device=dev, dtype=torch.int64),
                                      torch.empty(20, device=dev, dtype=torch.complex128))
        assert out.shape == (5, 12)
        a, b = ops.scheduled_radial_angular_channels_with_derivative(
            torch.empty(9, 4, device=dev), torch.empty(9, 4, device=dev), torch.empty(9, 16, device=dev),
            torch.empty(9, 16, 3, device=dev), torch.empty(9, 3, device=dev),
            torch.empty(9, device=dev, dtype=torch.int64), torch.empty(6, device=dev, dtype=torch.int64),
            torch.empty(6, device=dev, dtype=torch.int64), torch.empty(6, device=dev, dtype=torch.int64),
            torch.empty(6, device=dev))
        assert a.shape == (9, 6) and b.shape == (9, 6, 3)


@pytest.mark.parametrize("struct, c_name", [("AceTables", "y3b_ace_tables"),
                                             ("RecoupledTables", "y3b_recoupled_tables"),
                                             ("RecoupledSymTables", "y3b_recoupled_sym_tables")])
def test_tables_struct_layout_matches_header(tmp_path, struct, c_name):
    """The ctypes mirrors of the table structs (y3b_ace_tables is passed by value to every
    fused kernel) have the C structs' sizes and field offsets, read from include/ye3t_b200.h
    by a small C program."""
    import ctypes
    import shutil
    import subprocess
    from ye3t_b200 import _native
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    cls = getattr(_native, struct)
    fields = [name for name, _ in cls._fields_]
    src = tmp_path / "layout.c"
    src.write_text("#include <stdio.h>\n#include <stddef.h>\n#include \"ye3t_b200.h\"\nint main(void) {\n"
                   f"  printf(\"%zu\\n\", sizeof({c_name}));\n"
                   + "".join(f"  printf(\"%zu\\n\", offsetof({c_name}, {f}));\n" for f in fields)
                   + "  return 0;\n}\n")
    exe = tmp_path / "layout"
    include = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")
    subprocess.run([gcc, "-I", include, str(src), "-o", str(exe)], check=True)
    out = [int(v) for v in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]
    assert out[0] == ctypes.sizeof(cls)
    assert out[1:] == [getattr(cls, f).offset for f in fields]


def test_ctypes_signatures_match_header_parameter_counts():
    """Every entry point's ctypes argument list has as many entries as its declaration in
    include/ye3t_b200.h has parameters (a short or long list would pass arguments misaligned)."""
    from ye3t_b200 import _native
    src = open(os.path.join(REPO, "include", "ye3t_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    counts = {}
    for m in re.finditer(r"\b(y3b_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", src):
        params = m.group(2).strip()
        counts[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    assert counts and set(counts) == set(_native._SIGS)
    for name, (_, args) in _native._SIGS.items():
        assert len(args) == counts[name], (name, len(args), counts[name])


def test_bench_cell_order_makes_rank_blocks_slabs():
    """bench.cell_order sorts atoms by (z, y, x) cell, so that the contiguous atom blocks of
    the ranks are slabs of the box: block r's z cells form one run, and consecutive blocks
    meet at most in one cell layer."""
    import sys

    import numpy as np
    if REPO not in sys.path:
        sys.path.insert(0, REPO)
    import bench
    from ye3t_b200.distributed import atom_block
    N = 20000
    box = (N / 0.05) ** (1 / 3)
    pos = np.random.default_rng(0).uniform(0, box, (N, 3))
    order = bench.cell_order(pos, box, 5.0)
    assert sorted(order.tolist()) == list(range(N))
    n = int(box / 5.0)
    cz = np.floor(pos[order, 2] / box * n).astype(int)
    assert np.all(np.diff(cz) >= 0)
    last = -1
    for r in range(4):
        b, e = atom_block(r, 4, N)
        assert cz[b] >= last
        last = cz[e - 1]
    # the default C5 run takes the recoupled passes
    argv = sys.argv
    try:
        sys.argv = ["bench.py"]
        args = bench.parse()
    finally:
        sys.argv = argv
    assert args.b_basis == "recoupled" and not args.recoupled_general and args.config == "c5"
