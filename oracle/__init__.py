"""Parity checkers — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
``--impl reference`` legs may import this package.  Nothing in navi_b200/
imports it.
"""
