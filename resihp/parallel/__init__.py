"""Tensor, pipeline and data parallel runtime."""
