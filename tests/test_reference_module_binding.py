"""Binding this library into the reference's own module (CPU).

* The committed boundary fixture (tests/golden/module_boundary.npz) agrees
  with the oracle: what the reference kernel returned for the captured
  arguments, and the module output as its reshape.
* Where a reference checkout is named by FAKLA_REFERENCE_ROOT: the reference's
  TMLinKernelAttn, loaded through the golden generator's loader shim, with its
  backend name bound to pulsartecture_b200.backend.interface.fa_kla_attention
  (the binding INTEGRATION.md describes), hands this library its (B, T, H, D)
  tensors; on CPU tensors the library raises RuntimeError (it has no CPU path)
  and the module re-raises it, as its error contract says (tm_kla.py:323-327).
  The GPU replay of the same call is tests/test_gpu_reference_module.py.
"""
import os

import numpy as np
import pytest
import torch

from oracle import fakla_oracle as O
from tests.helpers import rel_l2

FIXTURE = os.path.join(os.path.dirname(__file__), "golden", "module_boundary.npz")


@pytest.mark.parametrize("tag", ["plain", "temp"])
def test_boundary_fixture_matches_oracle(tag):
    with np.load(FIXTURE) as f:
        a = {k.split("/", 1)[1]: f[k] for k in f.files if k.startswith(tag + "/")}
    e, _, _ = O.attention(a["q_mapped"], a["k_mapped"], a["v"], a["temp"])
    assert rel_l2(a["backend_out"], e) < 1e-5
    B, T, H, Dv = a["backend_out"].shape
    np.testing.assert_array_equal(a["backend_out"].reshape(B, T, H * Dv), a["module_out"])
    assert (a["q_mapped"] > 0).all() and (a["k_mapped"] > 0).all()  # elu+1 features


def test_reference_module_reaches_this_library():
    from oracle import build_ref

    root = os.environ.get(build_ref.REF_ENV)
    if not root or not os.path.isdir(root):
        pytest.skip(f"no reference checkout named by {build_ref.REF_ENV}")
    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
    import make_golden

    from pulsartecture_b200.backend import interface as ours

    ref = build_ref.load() if build_ref.built_module_path() else None
    if ref is None:
        pytest.skip("reference kernel not built")
    fm, _, tm = make_golden.load_reference_modules(root, ref)
    seen = []

    def bound(q_mapped, k_mapped, v_reshaped, temp):
        seen.append([(tuple(t.shape), t.dtype, t.is_contiguous()) for t in (q_mapped, k_mapped, v_reshaped, temp)])
        return ours.fa_kla_attention(q_mapped, k_mapped, v_reshaped, temp)

    tm.fa_kla_attention = bound
    torch.manual_seed(0)
    mod = tm.TMLinKernelAttn(128, fm.LearnablePositiveMap(128, 128), num_heads=4, qk_dim=32, v_dim=32)
    with pytest.raises(RuntimeError):
        with torch.no_grad():
            mod(torch.randn(2, 48, 128))
    assert seen == [[((2, 48, 4, 32), torch.float32, True)] * 3 + [((2, 48, 4), torch.float32, True)]]
