"""Feature maps (phi) for FA-KLA and their dynamic mixture."""
from .feature_maps import (  # noqa: F401
    FeatureMap,
    LearnablePositiveMap,
    OrthogonalRandomFeatures,
    RandomFourierFeatures,
)
from .mixer import GateNet, KernelFeatureMixer  # noqa: F401
