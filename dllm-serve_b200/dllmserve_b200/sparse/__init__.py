"""Subpackage of dllmserve_b200."""
