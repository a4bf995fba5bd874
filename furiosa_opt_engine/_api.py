"""Placeholder surface; the engine classes are added as they land."""

__all__: list[str] = []
