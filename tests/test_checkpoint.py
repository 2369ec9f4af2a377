"""Gaussian checkpoints in the reference's format (model.py:610-624)."""
import torch

from complex_valued_holographic_radiance_fields_b200 import scene as SC


def test_roundtrip_and_reference_layout(tmp_path):
    params = SC.make_gaussians(50, K=3, C=3, seed=1, device="cpu")
    path = tmp_path / "g.pth"
    SC.save_gaussians(params, path)
    raw = torch.load(path)
    assert set(raw) == set(SC.CHECKPOINT_KEYS)        # exactly the reference's keys
    assert all(v.device.type == "cpu" for v in raw.values())
    back = SC.load_gaussians(path, device="cpu")
    for k in SC.CHECKPOINT_KEYS:
        assert torch.equal(back[k], params[k]) and back[k].requires_grad
