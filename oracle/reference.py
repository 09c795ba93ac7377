"""Location of the reference ye3t checkout, for the steps that read or build it.

Test infrastructure only: the oracle's build of the reference's own runtime core
(``oracle/_ref``, ``make -C oracle ref REF=<dir>``), the golden-fixture generator
(``tests/golden/make_golden.py``) and the build entry point (``__graft_entry__.build``)
take it from here.  The environment variable ``YE3T_REFERENCE`` names the checkout;
unset, a checkout named ``reference`` beside this repository is used when it exists.
Without either, the reference-dependent steps are skipped and the committed fixtures
(and an existing ``oracle/_ref``) are used as they are.  Nothing on the product path
or on the GPU box reads it.
"""

from __future__ import annotations

import os
from typing import Optional

ENV = "YE3T_REFERENCE"
_REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def reference_dir() -> Optional[str]:
    """The reference checkout (a directory holding ``ye3t/``), or None."""
    for d in (os.environ.get(ENV, ""), os.path.join(os.path.dirname(_REPO), "reference")):
        if d and os.path.isdir(os.path.join(d, "ye3t")):
            return os.path.abspath(d)
    return None
