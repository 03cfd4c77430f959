"""Distributed runtime: environment, mesh, collectives, data / tensor / expert parallelism,
sharded checkpoints and the fused peer-memory communication kernels."""
