"""Trace-driven cluster simulation of one long training job under resilience policies."""
