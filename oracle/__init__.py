"""CPU oracle for the token-selection path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
package, and only as the checker.  The product (paged_moe_b200) never imports
it.  The arithmetic lives in pm_oracle.c; this module is its ctypes driver plus
the host-side parameter rounding and the verify (draft acceptance) logic.

Parity status: greedy argmax, equality acceptance and the allowed-token mask
are pinned against the reference's own code (tests/golden/make_golden.py);
penalties, top-k/top-p/min-p, temperature and the categorical draw are PARITY
UNPINNED (they restate mlx-lm 0.31.3, which is not in the reference tree);
residual rejection sampling is PARITY UNPINNED (no reference implementation).
"""

from .oracle import *  # noqa: F401,F403
from .oracle import __all__  # noqa: F401
