"""CPU oracle of the reference E-step -- test infrastructure only.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
legs; the product package never imports it."""
