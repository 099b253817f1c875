"""Timing, clock sampling and distributed helpers."""
