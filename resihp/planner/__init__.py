"""Torch-free TP, PP and DP planners."""
