"""Host-side argument rules of ennx_b200.ops that stop a call before any device work."""
import pytest

torch = pytest.importorskip("torch")

from ennx_b200 import ops  # noqa: E402


def test_noise_step_form_needs_plus_and_no_minus():
    with pytest.raises(ValueError):
        ops.perturb_bf16(None, 1, 0, 0, 1e-3)
    t = torch.empty(8, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ops.perturb_bf16(None, 1, 0, 0, 1e-3, plus=t, minus=t)
