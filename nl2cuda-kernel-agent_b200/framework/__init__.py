"""Harness of the RBF hot path: the Case protocol, the tolerance/timing protocol, the sm_100a
loader, the verifier and the benchmarker.  Same module names and call signatures as the
reference's ``framework/`` package, so ``verify_all(CASE, candidate)`` and
``compare(CASE, candidate)`` drive this implementation exactly as they drive the reference's."""
