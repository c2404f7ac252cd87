"""The allocation-free dropout-LayerNorm backward (cign_dropout_ln_bwd_static)
against the workspace version (cign_dropout_ln_bwd), both called through the
C ABI.

The static entry point exists for callers that cannot allocate device
memory (for instance a plugin inside a host framework that owns every byte
of device memory and hands kernels only their inputs and outputs): its
reduction scratch is a fixed array inside the library instead of a buffer
the caller passes.  This file is named so that pytest collects it last; it
also passes on its own in a fresh process.
"""
import pytest
import torch

from cign_b200 import _lib
from tests.helpers import assert_parity

pytestmark = pytest.mark.gpu


def _inputs(n, d, dev, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(n, d, generator=g).to(dev)
    w = (1 + 0.1 * torch.randn(d, generator=g)).to(dev)
    gy = torch.randn(n, d, generator=g).to(dev)
    mean = torch.randn(n, generator=g).to(dev) * 0.1
    rstd = (1 + 0.1 * torch.rand(n, generator=g)).to(dev)
    return x, w, gy, mean, rstd


def _workspace_version(lib, n, d, x, w, gy, mean, rstd, p, seed, stream):
    gx = torch.empty_like(x)
    gw = torch.empty(d, device=x.device)
    gb = torch.empty(d, device=x.device)
    ws = torch.empty(max(int(lib.cign_ln_bwd_workspace_bytes(n, d)), 16), dtype=torch.uint8,
                     device=x.device)
    rc = lib.cign_dropout_ln_bwd(n, d, _lib.ptr(gy), _lib.ptr(x), _lib.ptr(w), _lib.ptr(mean),
                                 _lib.ptr(rstd), p, seed, None, _lib.ptr(gx), _lib.ptr(gw),
                                 _lib.ptr(gb),
                                 _lib.ptr(ws), ws.numel(), stream)
    _lib.check(rc, "cign_dropout_ln_bwd")
    return gx, gw, gb


def _static_version(lib, n, d, x, w, gy, mean, rstd, p, seed, stream):
    gx = torch.empty_like(x)
    gw = torch.empty(d, device=x.device)
    gb = torch.empty(d, device=x.device)
    rc = lib.cign_dropout_ln_bwd_static(n, d, _lib.ptr(gy), _lib.ptr(x), _lib.ptr(w),
                                        _lib.ptr(mean), _lib.ptr(rstd), p, seed, _lib.ptr(gx),
                                        _lib.ptr(gw), _lib.ptr(gb), stream)
    _lib.check(rc, "cign_dropout_ln_bwd_static")
    return gx, gw, gb


@pytest.mark.parametrize("n,d,p", [(24492, 512, 0.5), (3001, 1024, 0.0), (777, 30, 0.28)])
def test_static_scratch_matches_workspace_version(cuda, n, d, p):
    lib = _lib.load_library()
    stream = _lib.stream_on(cuda)
    seed = 0x1234_5678_9ABC_DEF0 & ((1 << 63) - 1)
    # two calls in a row, with different inputs, each against the workspace version
    for call in range(2):
        x, w, gy, mean, rstd = _inputs(n, d, cuda, seed=17 * call + d)
        ref = _workspace_version(lib, n, d, x, w, gy, mean, rstd, p, seed + call, stream)
        got = _static_version(lib, n, d, x, w, gy, mean, rstd, p, seed + call, stream)
        torch.cuda.synchronize()
        for a, e, name in zip(got, ref, ("grad_x", "grad_w", "grad_b")):
            assert_parity(a, e, what=f"{name} n={n} d={d} call={call}")


def test_static_scratch_allocates_nothing(cuda):
    """Around a call of the static entry point neither torch's allocator nor
    the device's free memory changes (inputs and outputs exist beforehand;
    the device address of the scratch is looked up before the measurement)."""
    lib = _lib.load_library()
    stream = _lib.stream_on(cuda)
    n, d, p, seed = 24492, 512, 0.5, 99
    x, w, gy, mean, rstd = _inputs(n, d, cuda, seed=5)
    gx, gw, gb = torch.empty_like(x), torch.empty(d, device=cuda), torch.empty(d, device=cuda)

    def call():
        rc = lib.cign_dropout_ln_bwd_static(n, d, _lib.ptr(gy), _lib.ptr(x), _lib.ptr(w),
                                            _lib.ptr(mean), _lib.ptr(rstd), p, seed,
                                            _lib.ptr(gx), _lib.ptr(gw), _lib.ptr(gb), stream)
        _lib.check(rc, "cign_dropout_ln_bwd_static")

    call()  # first call on this device: symbol lookup
    torch.cuda.synchronize()
    stats0 = torch.cuda.memory_stats(cuda)["allocation.all.current"]
    free0, _ = torch.cuda.mem_get_info(cuda)
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    assert torch.cuda.memory_stats(cuda)["allocation.all.current"] == stats0
    assert torch.cuda.mem_get_info(cuda)[0] == free0


def test_static_scratch_zero_rows(cuda):
    """n = 0: the parameter gradients are zeros (no rows contribute)."""
    lib = _lib.load_library()
    gw = torch.full((64,), 7.0, device=cuda)
    gb = torch.full((64,), 7.0, device=cuda)
    rc = lib.cign_dropout_ln_bwd_static(0, 64, None, None, None, None, None, 0.0, 0, None,
                                        _lib.ptr(gw), _lib.ptr(gb), _lib.stream_on(cuda))
    _lib.check(rc, "cign_dropout_ln_bwd_static")
    torch.cuda.synchronize()
    assert bool((gw == 0).all()) and bool((gb == 0).all())


def test_static_scratch_rejects_oversize(cuda):
    lib = _lib.load_library()
    rc = lib.cign_dropout_ln_bwd_static(8, 2048, None, None, None, None, None, 0.0, 0, None, None,
                                        None, _lib.stream_on(cuda))
    assert rc != 0
    assert "1024" in _lib.last_error() or "exceeds" in _lib.last_error()
