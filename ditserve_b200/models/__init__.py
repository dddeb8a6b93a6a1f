"""Model backends behind the worker protocol (mock fixture, Wan, SD3.5)."""
