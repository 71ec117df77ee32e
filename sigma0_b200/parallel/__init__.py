"""Parallelism: fused NVLink data-parallel sync, tensor and context parallelism."""
