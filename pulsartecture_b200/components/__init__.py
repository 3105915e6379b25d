"""Building blocks around the FA-KLA path."""
from .projections import LinearProjection  # noqa: F401
