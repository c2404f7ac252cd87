"""Comparison helpers shared by the GPU parity tests."""
import torch


def rel_l2(a, b) -> float:
    a = torch.as_tensor(a).detach().double().cpu()
    b = torch.as_tensor(b).detach().double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def assert_parity(actual, expected, tol=1e-5, atol=1e-6, what=""):
    """fp32 parity: relative L2 error <= tol (the north-star 1e-5 relative
    bound, in the rel-L2 form of validate_cign_acceleration.py:33) and an
    elementwise guard against isolated outliers,
    |a - e| <= atol + 100*tol*(|e| + rms(e)) -- sums with cancellation
    (e.g. softmax-backward row sums) are judged on the tensor's scale."""
    a = torch.as_tensor(actual).detach().double().cpu()
    e = torch.as_tensor(expected).detach().double().cpu()
    assert a.shape == e.shape, (what, a.shape, e.shape)
    assert torch.isfinite(a).all(), what
    err = rel_l2(a, e)
    assert err <= tol, f"{what}: rel-L2 {err:.3e} > {tol:.1e}"
    rms = float(e.pow(2).mean().sqrt()) if e.numel() else 0.0
    bad = (a - e).abs() > atol + 100 * tol * (e.abs() + rms)
    assert not bool(bad.any()), f"{what}: {int(bad.sum())} elements off, max {float((a - e).abs().max()):.3e}"
