"""CPU oracle for the Kev scoring forward -- TEST INFRASTRUCTURE ONLY.

This package restates the reference's CPU fp32 Kev forward (crates/huncho-backend
src/qwen3_5.rs, kev.rs, delta_cpu.rs, conv_cpu.rs and huncho-core calibration.rs /
engine.rs) so that the CUDA path can be checked against it. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it, and
only as the checker or the timed CPU baseline. The product package ``huncho_b200``
never imports, links or calls anything here.

Parity is pinned: ``tests/test_oracle_golden.py`` checks this restatement against
the reference's own golden vectors (tests/fixtures/tiny_kev/golden.json, produced
by upstream PyTorch) at the reference test's tolerances
(crates/huncho-backend/tests/kev_reference.rs:64-76).
"""
