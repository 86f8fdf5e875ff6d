"""TEST INFRASTRUCTURE: the CPU oracle for the mixture-of-experts path (checker only).

Importable by tests/, bench.py's cpu_baseline / --impl reference legs and
__graft_entry__.smoke(); never by the product package.
"""
