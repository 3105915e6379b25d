"""Native FA-KLA backend (the libfakla.so C ABI behind a torch-tensor API)."""
from .interface import (  # noqa: F401
    fa_kla_attention,
    fa_kla_attention_with_state,
    fa_kla_decode_step,
    fa_kla_prefill,
    phi_map,
)
