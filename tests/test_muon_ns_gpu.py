"""Newton–Schulz on the tensor cores (``mimir_b200.optim.newton_schulz``) against the fp32 chain
of the reference (``orthogonalize``), on every logical matrix shape of the 1.3B bench model."""
import pytest
import torch

pytestmark = pytest.mark.gpu

# (rows, cols) of the Muon pieces: gate/q/o, k/v (4 KV heads), gate/up (tall), down (wide)
SHAPES = [(2048, 2048), (512, 2048), (5632, 2048), (2048, 5632)]


@pytest.mark.parametrize("rows,cols", SHAPES)
def test_bf16_chain_matches_fp32_chain(rows, cols):
    from mimir_b200.optim.muon import orthogonalize
    from mimir_b200.optim.newton_schulz import orthogonalize_batch
    g = torch.Generator(device="cuda").manual_seed(rows + cols)
    m = torch.randn(3, rows, cols, device="cuda", generator=g)
    ours = orthogonalize_batch(m, 5)
    ref = orthogonalize(m, 5)
    assert ours.shape == ref.shape and ours.dtype == torch.float32
    rel = (ours - ref).norm() / ref.norm()
    assert rel < 3e-2, f"relative difference {rel.item():.3e}"
    # The iteration drives the singular values into the same band as the fp32 chain does.
    wide = ours if rows <= cols else ours.mT
    wide_ref = ref if rows <= cols else ref.mT
    eye = torch.eye(wide.shape[-2], device="cuda")
    dev = (wide @ wide.mT - eye).norm(dim=(-2, -1)) / eye.norm()
    dev_ref = (wide_ref @ wide_ref.mT - eye).norm(dim=(-2, -1)) / eye.norm()
    assert torch.allclose(dev, dev_ref, atol=2e-2), (dev, dev_ref)
    from mimir_b200.ops import gemm as G
    assert G.status(0) == 0
