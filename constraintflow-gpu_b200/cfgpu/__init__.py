"""cfgpu: B200 (sm_100a) runtime for ConstraintFlow's DeepPoly certification hot path.

``cfgpu._lib`` binds libcfgpu.so (include/cfgpu.h); ``cfgpu.engine`` runs a whole
chain network per call; ``cfgpu.nets`` builds the seeded synthetic workloads.
"""
__all__ = ["engine", "nets"]
