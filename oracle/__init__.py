"""CPU oracle for the GEMM path and the reference-compiled descriptor probes.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg, never by the product (maia_b200/). See gemm_oracle.c for what is restated and how it is pinned.
"""
