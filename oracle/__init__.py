"""CPU oracle for the SEM stiffness path -- TEST INFRASTRUCTURE ONLY.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
legs, as the checker and the timed CPU port; the product never imports it.
"""
