"""Test-infrastructure oracle for the iris.c DiT hot path.

CPU restatements of the reference algorithms (flux_oracle, sample_oracle,
zimage_oracle), the seeded model generator (model_gen) and a ctypes loader
for the reference compiled from its own sources (ref_lib).  Imported only by
tests/, __graft_entry__.smoke() and bench.py's CPU/reference legs.
"""
