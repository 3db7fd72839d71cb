"""Trainer, optimizer and learning-rate schedules."""
