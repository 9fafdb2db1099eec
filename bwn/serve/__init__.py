"""Batched generation engine and an HTTP completion server."""
