"""Folded virtual pipeline: schedule, stage compute, boundary transport."""
