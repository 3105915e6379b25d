"""TM-KLA attention: module API and functional FA-KLA ops."""
from .tm_kla import TemperatureFunction, TMLinKernelAttn, fa_kla, fa_kla_decode, fa_kla_host  # noqa: F401
