"""CPU oracle for the q6 affine linear / image feed-forward path.

TEST INFRASTRUCTURE ONLY.  Only tests/, ``__graft_entry__.smoke()`` and
bench.py's CPU-baseline leg may import this package, and only as the checker
(or, for the baseline, as the thing timed on the host cores).  The product
package never imports it and has no CPU fallback.
"""

from oracle.oracle import *  # noqa: F401,F403
