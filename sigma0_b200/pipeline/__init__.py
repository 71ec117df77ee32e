"""Evaluation pipeline: LOB-Bench style scoring, injection verification, model store,
packaging, integrity records."""
