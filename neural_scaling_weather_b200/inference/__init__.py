"""Autoregressive inference and scoring."""
