"""Test-only ``mlx`` package stand-in (see ``core.py``)."""
