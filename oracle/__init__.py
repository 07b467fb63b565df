"""TEST INFRASTRUCTURE ONLY: CPU oracle for the Sinkhorn half-step and solver (see trnopt_oracle.py).

Importable only from tests/, __graft_entry__.smoke() and bench.py's CPU baseline; the CUDA product path never
uses it.
"""
