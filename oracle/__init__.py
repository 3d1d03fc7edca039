"""CPU oracle for the folded multi-branch verify forward.

TEST INFRASTRUCTURE ONLY.  Nothing in ``specfold_b200`` imports this package; only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` use it, and there only as the checker or as the timed CPU
baseline, never as the product path.
"""
