"""CPU oracle for the token-merged global-attention path — TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference algorithms (shuang-yang18/4D_TTT_merging, files cited
per function in ``oracle/ref.py``), used as the checker for the B200 kernels and as the CPU
baseline timed by ``bench.py``.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference legs may import it; the product package never does.

Parity pin: the restatement is checked against golden vectors produced by running the
reference's own PyTorch code (imported read-only) in the build container; the vectors and
the script that made them live in ``tests/golden/``.
"""
from .ref import *  # noqa: F401,F403
from .synth import *  # noqa: F401,F403
from . import pipeline  # noqa: F401
from . import ttt_planner  # noqa: F401
from . import ttt_prepass  # noqa: F401
