"""Utilities: tracing."""
