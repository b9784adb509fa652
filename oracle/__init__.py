"""CPU oracle for the wavefront attention / KV-slot hot path — TEST INFRASTRUCTURE.

A numpy restatement of the reference's own algorithm for this path
(summerbro-hhj/wavefront-decoding, src/decoding/fa4_attention.py `sdpa` twins,
src/decoding/batch_kv_cache.py, src/decoding/scheduler_batch.py, src/decoding/emu.py),
each function citing the reference file:line it follows.  It is pinned by the
golden vectors under tests/golden/ (produced by importing the reference itself,
tests/golden/make_golden.py).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm
may import this package, and only as the checker or the timed CPU baseline.
The product (wavefront-decoding_b200/) never imports it: it has no CPU path.
"""
