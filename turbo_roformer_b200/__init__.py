"""Blackwell (sm_100a) CUDA backend for the BS-RoFormer forward."""
