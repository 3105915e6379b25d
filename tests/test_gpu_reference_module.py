"""The reference module's own backend call, replayed on this library (GPU).

tests/golden/module_boundary.npz holds, for two configurations of the
reference's TMLinKernelAttn (ultra_rwka/attention/tm_kla.py:110-337, run on
the CPU where the reference checkout lives), the four tensors the module
passed to its backend `fa_kla_attention` (tm_kla.py:319), what the reference's
own fa_kla_attention_cpu returned, and the module's output. Here those exact
arguments go through pulsartecture_b200.backend.interface.fa_kla_attention on
the GPU, which must return the reference kernel's result within the fp32 bar,
and the module's remaining step (the (B, T, H*Dv) reshape, tm_kla.py:332)
must give the module's output.
"""
import os

import numpy as np
import pytest
import torch

from tests.helpers import F32_REL_L2, rel_l2

pytestmark = pytest.mark.gpu

FIXTURE = os.path.join(os.path.dirname(__file__), "golden", "module_boundary.npz")


@pytest.mark.parametrize("tag", ["plain", "temp"])
def test_reference_module_backend_call_on_gpu(cuda, tag):
    from pulsartecture_b200.backend.interface import fa_kla_attention

    with np.load(FIXTURE) as f:
        a = {k.split("/", 1)[1]: f[k] for k in f.files if k.startswith(tag + "/")}
    args = [torch.from_numpy(a[n]).to(cuda) for n in ("q_mapped", "k_mapped", "v", "temp")]
    out = fa_kla_attention(*args)
    assert out.dtype == torch.float32 and tuple(out.shape) == a["backend_out"].shape
    got = out.cpu().numpy()
    assert rel_l2(got, a["backend_out"]) < F32_REL_L2
    B, T, H, Dv = got.shape
    assert rel_l2(got.reshape(B, T, H * Dv), a["module_out"]) < F32_REL_L2
    if tag == "temp":
        assert not np.allclose(a["temp"], 1.0), "the temperature case must carry a non-trivial temperature"
