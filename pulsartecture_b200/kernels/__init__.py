"""Feature maps (phi) for FA-KLA."""
from .feature_maps import FeatureMap, LearnablePositiveMap  # noqa: F401
