"""GPU parity of the norms and attention against the CPU oracle (pinned to the reference's norm_rows, rms_heads and
attention in tests/test_oracle.py). One bar for every check, bf16 inputs against the fp32 oracle:
max |y - ref| <= 2e-2 x rms(ref).

Attention is checked twice per case: its fp32 output against the oracle, and its bf16 output, which must be the fp32
output rounded to bf16 bit for bit (the kernel rounds once, at the store). Inputs: the reference's own attention-test
distribution (uniform in [-1, 1], tests/test_kernels.cpp:184-191) and the blocks' distribution (q and k through
rms_heads, so each head has norm 8 and its scores have unit spread), where the bf16 output is also held to the bar
(the rows with one dominant key then carry values near the largest of v, the case the bf16 store can miss; the
measured ratio is printed)."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _check(y, ref, tol=TOL, what=""):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.isfinite(y).all(), what
    rms = np.sqrt((ref ** 2).mean())
    err = np.abs(y - ref).max()
    assert err <= tol * rms, f"{what}: max abs err {err:.3e} > {tol} x rms {rms:.3e}"


def _ratio(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.isfinite(y).all()
    return float(np.abs(y - ref).max() / np.sqrt((ref ** 2).mean()))


def _bf(oracle, a):
    return oracle.f32_to_bf16_round(np.asarray(a, np.float32))


@pytest.mark.parametrize("dim", [256, 1024, 2048])
@pytest.mark.parametrize("mode", ["plain", "affine", "adaln"])
def test_norm_rows(pkg, oracle, cuda, dim, mode):
    from idol_b200 import layers
    rng = np.random.default_rng(dim)
    rows = 77
    x = _bf(oracle, rng.normal(0.3, 2.0, (rows, dim)))
    kw = {}
    if mode == "affine":
        kw = dict(gamma=rng.normal(1, 0.2, dim).astype(np.float32), beta=rng.normal(0, 0.2, dim).astype(np.float32))
    if mode == "adaln":
        kw = dict(shift=rng.normal(0, 0.2, dim).astype(np.float32), scale=rng.normal(0, 0.2, dim).astype(np.float32))
    eps = 1e-6 if mode != "adaln" else 1e-5
    ref = oracle.norm_rows(x, eps, **kw)
    xt = torch.from_numpy(x).to(cuda, torch.bfloat16)
    tkw = {k: torch.from_numpy(v).to(cuda) for k, v in kw.items()}
    y = layers.norm_rows(xt, eps, **tkw)
    _check(y.float().cpu().numpy(), ref, what=f"norm_rows {mode} {dim}")
    # fp32 in, fp32 out, in place
    xf = torch.from_numpy(x).to(cuda)
    layers.norm_rows(xf, eps, out=xf, **tkw)
    np.testing.assert_allclose(xf.cpu().numpy(), ref, rtol=0, atol=2e-5)


def test_norm_rows_golden(pkg, cuda):
    from idol_b200 import layers
    z = np.load(GOLDEN / "ops.npz")
    x = torch.from_numpy(z["x"]).to(cuda)
    y = layers.norm_rows(x, 1e-6, gamma=torch.from_numpy(z["gamma"]).to(cuda), beta=torch.from_numpy(z["beta"]).to(cuda))
    np.testing.assert_allclose(y.cpu().numpy(), z["ln_affine"], rtol=0, atol=2e-5)


def test_rms_heads(pkg, oracle, cuda):
    from idol_b200 import layers
    z = np.load(GOLDEN / "ops.npz")
    rows, dim, heads, hd, lq, lk = (int(v) for v in z["meta"])
    qk = torch.from_numpy(z["qk"]).to(cuda)
    layers.rms_heads_(qk[:, :dim], heads, torch.from_numpy(z["qk_gamma"]).to(cuda))
    np.testing.assert_allclose(qk.cpu().numpy()[:, :dim], z["rms"][:, :dim], rtol=0, atol=2e-6)
    np.testing.assert_array_equal(qk.cpu().numpy()[:, dim:], z["qk"][:, dim:])  # untouched columns
    rng = np.random.default_rng(4)
    x = _bf(oracle, rng.normal(0, 1, (300, 3 * 1024)))
    g = rng.normal(1, 0.1, 1024).astype(np.float32)
    ref = oracle.rms_heads(x, 16, 64, g, col0=1024)
    xt = torch.from_numpy(x).to(cuda, torch.bfloat16)
    layers.rms_heads_(xt[:, 1024:2048], 16, torch.from_numpy(g).to(cuda))
    _check(xt.float().cpu().numpy()[:, 1024:2048], ref[:, 1024:2048], what="rms_heads bf16")


def _draw(oracle, rng, shape, dist, heads=None, qk_cols=0):
    """bf16-representable inputs: 'uniform' = U(-1, 1) as the reference's attention test; 'blocks' = N(0, 1) with the
    first qk_cols columns (q or q,k) normalised per 64-wide head to norm 8, as rms_heads leaves them."""
    if dist == "uniform":
        return _bf(oracle, rng.uniform(-1, 1, shape))
    a = rng.normal(0, 1, shape)
    if qk_cols:
        h = a[:, :qk_cols].reshape(shape[0], qk_cols // 64, 64)
        a[:, :qk_cols] = (h * (8.0 / np.linalg.norm(h, axis=2, keepdims=True))).reshape(shape[0], qk_cols)
    return _bf(oracle, a)


def _attention_case(oracle, cuda, lq, lk, heads, batch=1, packed=True, seed=0, rows=None, dist="uniform"):
    from idol_b200 import layers
    rng = np.random.default_rng(seed)
    dim = heads * 64
    if packed:  # self-attention layout: q, k, v are column blocks of one qkv buffer (src/decoders.cpp:301)
        assert lq == lk
        qkv = _draw(oracle, rng, (batch * lq, 3 * dim), dist, qk_cols=2 * dim)
        t = torch.from_numpy(qkv).to(cuda, torch.bfloat16)
        q, k, v = t[:, :dim], t[:, dim:2 * dim], t[:, 2 * dim:]
        qn, kn, vn = qkv[:, :dim], qkv[:, dim:2 * dim], qkv[:, 2 * dim:]
    else:  # cross-attention layout: q alone (row stride dim + 8), kv packed (src/decoders.cpp:239)
        qn = _draw(oracle, rng, (batch * lq, dim + 8), dist, qk_cols=dim)
        kv = _draw(oracle, rng, (batch * lk, 2 * dim), dist, qk_cols=dim)
        qt = torch.from_numpy(qn).to(cuda, torch.bfloat16)
        kvt = torch.from_numpy(kv).to(cuda, torch.bfloat16)
        q, k, v = qt[:, :dim], kvt[:, :dim], kvt[:, dim:]
        qn, kn, vn = qn[:, :dim], kv[:, :dim], kv[:, dim:]
    out16 = layers.attention(q, k, v, heads, batch=batch)
    out32 = layers.attention(q, k, v, heads, batch=batch,
                             out=torch.empty((batch * lq, dim), dtype=torch.float32, device=cuda))
    torch.cuda.synchronize()
    assert torch.equal(out16, out32.to(torch.bfloat16)), "bf16 output is not the fp32 output rounded once"
    got32, got16 = out32.cpu().numpy(), out16.float().cpu().numpy()
    worst32 = worst16 = 0.0
    for b in range(batch):
        sel = np.arange(lq) if rows is None else rows
        ref = oracle.attention(np.ascontiguousarray(qn[b * lq:(b + 1) * lq][sel]),
                               np.ascontiguousarray(kn[b * lk:(b + 1) * lk]),
                               np.ascontiguousarray(vn[b * lk:(b + 1) * lk]), heads, 64)
        worst32 = max(worst32, _ratio(got32[b * lq:(b + 1) * lq][sel], ref))
        worst16 = max(worst16, _ratio(got16[b * lq:(b + 1) * lq][sel], ref))
    what = f"attention {dist} lq={lq} lk={lk} h={heads} batch={batch}"
    print(f"\n{what}: max|err|/rms fp32 out {worst32:.3e}, bf16 out {worst16:.3e}")
    assert worst32 <= TOL, f"{what}: fp32 output max abs err / rms {worst32:.3e} > {TOL}"
    assert worst16 <= TOL, f"{what}: bf16 output max abs err / rms {worst16:.3e} > {TOL}"


@pytest.mark.parametrize("dist", ["uniform", "blocks"])
@pytest.mark.parametrize("lq,lk,heads", [(37, 53, 2), (3, 16, 1), (70, 130, 2), (128, 128, 1), (129, 257, 3),
                                         (300, 1000, 4)])
def test_attention_ragged_cross(pkg, oracle, cuda, lq, lk, heads, dist):
    """The reference's attention test shapes (tests/test_kernels.cpp:221-228) at head dim 64, strided q and kv."""
    _attention_case(oracle, cuda, lq, lk, heads, packed=False, seed=lq + lk, dist=dist)


@pytest.mark.parametrize("dist", ["uniform", "blocks"])
@pytest.mark.parametrize("l,heads,batch", [(256, 4, 2), (200, 2, 3), (1000, 16, 1)])
def test_attention_self_packed_batched(pkg, oracle, cuda, l, heads, batch, dist):
    _attention_case(oracle, cuda, l, l, heads, batch=batch, packed=True, seed=l, dist=dist)


def test_attention_config3_size_sampled_rows(pkg, oracle, cuda):
    """4096 tokens x 16 heads x 2 images (config 3's self-attention, the blocks' distribution), queries sampled
    across every 128-row tile."""
    rows = np.unique(np.concatenate([np.arange(0, 4096, 97), [0, 127, 128, 4095]]))
    _attention_case(oracle, cuda, 4096, 4096, 16, batch=2, packed=True, seed=3, rows=rows, dist="blocks")


def test_attention_golden(pkg, cuda):
    from idol_b200 import layers
    z = np.load(GOLDEN / "ops.npz")
    rows, dim, heads, hd, lq, lk = (int(v) for v in z["meta"])
    q = torch.from_numpy(z["att_q"]).to(cuda, torch.bfloat16)
    kv = torch.from_numpy(z["att_kv"]).to(cuda, torch.bfloat16)
    out = layers.attention(q[:, :dim], kv[:, :dim], kv[:, dim:2 * dim], heads,
                           out=torch.empty((q.shape[0], dim), dtype=torch.float32, device=cuda))
    r = _ratio(out.cpu().numpy(), z["att_out"])
    print(f"\ngolden attention: max|err|/rms fp32 out {r:.3e}")
    assert r <= TOL, f"golden attention (bf16 inputs): max abs err / rms {r:.3e} > {TOL}"


def test_layers_no_timeout(pkg, cuda):
    torch.cuda.synchronize()
    assert pkg._capi.device_status(0) == 0


@pytest.mark.parametrize("heads", [3, 4, 6, 32])
def test_rms_heads_bf16_head_counts(pkg, oracle, cuda, heads):
    """The vectorised bf16 kernel (head counts divisible by 4) and the per-head one (others), on a column block of a
    wider row as the decoders pass q and k."""
    from idol_b200 import layers
    rng = np.random.default_rng(heads)
    dim = heads * 64
    x = _bf(oracle, rng.normal(0, 1, (131, 3 * dim)))
    g = rng.normal(1, 0.1, dim).astype(np.float32)
    ref = oracle.rms_heads(x, heads, 64, g, col0=dim)
    xt = torch.from_numpy(x).to(cuda, torch.bfloat16)
    layers.rms_heads_(xt[:, dim:2 * dim], heads, torch.from_numpy(g).to(cuda))
    got = xt.float().cpu().numpy()
    _check(got[:, dim:2 * dim], ref[:, dim:2 * dim], what=f"rms_heads bf16 heads={heads}")
    np.testing.assert_array_equal(got[:, :dim], x[:, :dim])
    np.testing.assert_array_equal(got[:, 2 * dim:], x[:, 2 * dim:])
