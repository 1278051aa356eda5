"""Small shared helpers for the parity tests."""

import numpy as np
import torch

SEED = 20261201


def rng(seed_offset=0):
    return np.random.default_rng(SEED + seed_offset)


def f16(a) -> torch.Tensor:
    """float32 CPU tensor holding fp16-representable values."""
    return torch.from_numpy(np.asarray(a, dtype=np.float32)).to(torch.float16).to(torch.float32)


def dev(t: torch.Tensor, dtype=torch.float16) -> torch.Tensor:
    return t.to(dtype).contiguous().cuda()


def host(t: torch.Tensor) -> torch.Tensor:
    return t.float().cpu()


def rel_l2(got: torch.Tensor, want: torch.Tensor) -> float:
    got, want = got.double(), want.double()
    den = torch.linalg.vector_norm(want).item()
    return torch.linalg.vector_norm(got - want).item() / max(den, 1e-30)


def assert_close(got, want, max_abs=2e-2, rel=1e-3, what=""):
    """FP16 activation parity bar: max-abs 2e-2 and relative L2 1e-3."""
    got = got.float()
    want = want.float()
    assert got.shape == want.shape, f"{what}: shape {tuple(got.shape)} != {tuple(want.shape)}"
    assert torch.isfinite(got).all(), f"{what}: non-finite output"
    diff = (got - want).abs()
    ma = diff.max().item() if diff.numel() else 0.0
    r = rel_l2(got, want) if diff.numel() else 0.0
    where = np.unravel_index(int(diff.argmax()), tuple(diff.shape)) if diff.numel() else ()
    assert ma <= max_abs and r <= rel, (
        f"{what}: max_abs={ma:.4g} (at {where}: got {got[where].item() if diff.numel() else 0:.5g} "
        f"want {want[where].item() if diff.numel() else 0:.5g}) rel_l2={r:.3g}")
