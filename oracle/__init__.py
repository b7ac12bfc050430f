"""CPU oracle for the recurrent ensemble step - test infrastructure only.

Nothing in the product package imports this; tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline leg use it as the checker.
"""
