"""CPU oracle for the textsift forward path (test infrastructure only).

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
legs; the CUDA product path never touches this package.
"""
