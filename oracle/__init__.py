"""TEST INFRASTRUCTURE ONLY: the CPU oracle for the RBF hot path.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this package; the
product library (nl2cuda-kernel-agent_b200/) never does.
"""
