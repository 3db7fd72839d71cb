"""Rank grid, process groups, collective primitives and gradient reduction."""

from . import comm  # noqa: F401
