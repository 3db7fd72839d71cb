"""Utilities: profiling, FLOP accounting, grid helpers, spherical harmonics."""
