"""CPU oracle for the Theorem forward hot path -- TEST INFRASTRUCTURE ONLY.

Nothing in the shipped library (``theorem_b200``) imports this package. It is
the checker: ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` are its only users.

* ``oracle.ops``    -- numpy restatement (float64) of the reference's four
  PyTorch ``ref_kernel``s plus the extensions the north star asks for
  (SiLU / channel-last conv, fused WY matrix with either sign, delta-rule
  state recurrence with h0 / final state / v_new, the chained layer forward).
* ``oracle.inputs`` -- restatement of the reference's seeded input
  generators (``generate_input`` / ``generate_data`` / ``_build_inputs``) on
  the CPU, plus the BASELINE.json synthetic distributions.

Parity pin: ``tests/golden/make_golden.py`` ran the reference's own
``ref_kernel``s (imported from the reference checkout, CPU) on the task.yml
test shapes and stored their outputs under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks this oracle against them.
"""
