"""Tensor-parallel plumbing: process groups, the symmetric NVLink workspace and the collectives
(fused peer-memory all-reduce + norm; NCCL as the measured baseline; host ring for CPU ranks)."""
