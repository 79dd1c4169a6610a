"""Exceptions shared with the reference engine (engine/src/rec_mlx/prefix.py)."""


class PrefillCancelled(Exception):
    """Raised between prefill chunks when the caller asks to stop."""
