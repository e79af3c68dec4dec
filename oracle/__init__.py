"""CPU oracle for the sparse paged-attention hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm
may import this package, and only to check results or as the timed CPU baseline.  The
product (attention_b200) never imports it.

Parity pin: tests/golden/ holds fixtures produced by running the reference's
own PyTorch functions (experiments/triton_paged_attention.py,
triton_paged_gather_decode_benchmark.py, triton_paged_decode_benchmark.py,
triton_local_prefill.py) in a container where the reference is importable
(tests/golden/make_golden.py); tests/test_oracle_golden.py checks this oracle
against them.  Two parts have no reference implementation to pin against and
are parity-unpinned: the superblock->page tree router (the reference's
hierarchy is block->token) and the promotion table.
"""

from .sparse_paged import *  # noqa: F401,F403
