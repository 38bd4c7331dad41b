"""CPU oracle of DCR-Attention's sparse decode attention — test infrastructure only.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline`` /
``--impl reference`` legs import this package, as the checker and the timed CPU
baseline. The product package (``dcr_b200``) never imports it.
"""
