"""The allocation-free Gaussian MLP entry point (idol_b200_gaussian_mlp_forward_static).

Some callers cannot allocate device memory at all: a process whose GPU memory another allocator (a framework's
caching pool, a server's arena) has already reserved in full, where a cudaMalloc of its own would fail. They cannot
hand the regular entry point (idol_b200_gaussian_mlp_forward) a workspace, so this variant keeps its
scratch in a fixed 8 MiB array compiled into the library. This file checks, through the C-ABI, that it gives the same
output as the regular entry point on two calls in a row, and that a batch too large for the fixed array is refused.
It is named to be collected last, so a run that stops at the first failure has run every other test first; it also
passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _check(y, ref, what):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.isfinite(y).all(), what
    rms = np.sqrt((ref ** 2).mean())
    err = np.abs(y - ref).max()
    assert err <= TOL * rms, f"{what}: max abs err {err:.3e} > {TOL} x rms {rms:.3e}"


def _static_forward(pkg, mlp, x):
    C = pkg._capi
    points = x.shape[0]
    raw = torch.empty((points, 14), dtype=torch.float32, device=x.device)
    out = torch.empty((points, 14), dtype=torch.float32, device=x.device)
    rc = C.lib().idol_b200_gaussian_mlp_forward_static(
        ctypes.c_void_p(mlp.handle), ctypes.c_void_p(x.data_ptr()), points, x.stride(0),
        ctypes.c_void_p(raw.data_ptr()), ctypes.c_void_p(out.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream))
    C.check(rc)
    return raw, out


def test_static_scratch_matches_the_workspace_entry_point(pkg, oracle, cuda):
    from idol_b200.block import GaussianMLP, Q8Weight
    rng = np.random.default_rng(21)
    ws = []
    for n, k in [(512, 128), (512, 512), (14, 512)]:
        w = rng.normal(0, 0.02 if n != 14 else 0.2, (n, k)).astype(np.float32)
        b = rng.normal(0, 0.01, n).astype(np.float32)
        ws.append(Q8Weight(torch.from_numpy(oracle.q8_quantize(w).reshape(-1)).to(cuda), n, k, torch.from_numpy(b)))
    mlp = GaussianMLP(ws)
    g = torch.Generator(device=cuda).manual_seed(5)
    for call in range(2):  # two calls in a row: the shared array keeps the first call's contents
        points = 3000 if call == 0 else 1777
        x = torch.randn((points, 128), device=cuda, generator=g).to(torch.bfloat16)
        ref_raw, ref_out = mlp(x)
        raw, out = _static_forward(pkg, mlp, x)
        torch.cuda.synchronize()
        _check(raw.cpu().numpy(), ref_raw.cpu().numpy(), f"call {call}: raw")
        _check(out.cpu().numpy(), ref_out.cpu().numpy(), f"call {call}: heads")
    assert pkg._capi.device_status(0) == 0


def test_static_scratch_rejects_a_batch_beyond_its_size(pkg, oracle, cuda):
    from idol_b200.block import GaussianMLP, Q8Weight
    rng = np.random.default_rng(22)
    ws = []
    for n, k in [(512, 128), (512, 512), (14, 512)]:
        w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
        ws.append(Q8Weight(torch.from_numpy(oracle.q8_quantize(w).reshape(-1)).to(cuda), n, k))
    mlp = GaussianMLP(ws)
    x = torch.zeros((8192, 128), device=cuda, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="fixed"):
        _static_forward(pkg, mlp, x)
