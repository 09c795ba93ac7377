"""Compiler and linker flags for building a torch C++ extension with plain g++.

Test infrastructure only: ``oracle/Makefile`` (target ``ref``) builds the reference's
compiled schedule evaluator (ye3t/core/csrc/factorized_runtime.cpp, a torch extension
that the reference itself JIT-builds with ``torch.utils.cpp_extension.load`` and
``-O3``, ye3t/core/_factorized_runtime_cpp.py:54-83) from its source in place into
``oracle/_ref/``.  The flags are the ones ``torch.utils.cpp_extension`` would give a
CPU-only extension: torch's include directories, the Python headers, the C++11 ABI
switch and the torch libraries with an rpath.

Usage: ``python torch_ext_flags.py cflags|ldflags <module name>``.
"""

from __future__ import annotations

import os
import sys
import sysconfig


def cflags(name: str) -> list:
    import torch
    from torch.utils import cpp_extension as ce
    out = [f"-I{p}" for p in ce.include_paths()]
    out.append(f"-I{sysconfig.get_paths()['include']}")
    out += ["-DTORCH_API_INCLUDE_EXTENSION_H", f"-DTORCH_EXTENSION_NAME={name}",
            f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}"]
    return out


def ldflags() -> list:
    import torch
    lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    return [f"-L{lib}", f"-Wl,-rpath,{lib}", "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python"]


if __name__ == "__main__":
    kind = sys.argv[1]
    flags = cflags(sys.argv[2]) if kind == "cflags" else ldflags()
    print(" ".join(flags))
