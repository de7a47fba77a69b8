"""The tcgen05 INT8 GEMMs against exact CPU restatements (config-5 shapes, reduced M).

int8 activations: the s32 accumulators must match an int64 matmul bit for bit.
float32 activations: the three digit-plane accumulators must match a CPU restatement of the
slicing bit for bit, and the result must be within MatVecInt8's tolerance of the oracle's
float32 products (internal/kernels/int8_test.go:53-77 uses 1e-4 absolute at this scale).
"""
import numpy as np
import pytest

from mignon_ai_b200 import _lib

pytestmark = pytest.mark.gpu


def _rng_i8(rng, shape):
    return rng.integers(-127, 128, size=shape, dtype=np.int64).astype(np.int8)


# "pair": 256 x 256 tiles on CTA pairs (cta_group::2 MMAs reading both CTAs' operand halves), the
# default; "single": 128 x 256 tiles, one CTA each (MC_GEMM_I8_SINGLE=1). Row counts that are not a
# multiple of 256 leave the second CTA of a pair with partly or wholly out-of-range rows.
@pytest.mark.parametrize("kernel", ["pair", "single"])
@pytest.mark.parametrize("m,n,k", [(256, 256, 192), (256, 1024, 384), (4096, 256, 1152), (384, 512, 128),
                                   (200, 256, 384), (100, 512, 96), (4500, 2048, 1152)])
def test_gemm_i8_exact(m, n, k, kernel, monkeypatch):
    if kernel == "single":
        monkeypatch.setenv("MC_GEMM_I8_SINGLE", "1")
    else:
        monkeypatch.delenv("MC_GEMM_I8_SINGLE", raising=False)
    rng = np.random.default_rng(5)
    a, w = _rng_i8(rng, (m, k)), _rng_i8(rng, (n, k))
    rs = rng.uniform(0.5, 2, m).astype(np.float32)
    cs = rng.uniform(0.001, 0.01, n).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    c = np.zeros((m, n), np.int32)
    y = np.zeros((m, n), np.float32)
    L = _lib.lib()
    _lib.check(L.mc_gemm_i8(0, _lib.ptr(a), _lib.ptr(w), m, n, k, _lib.ptr(rs), _lib.ptr(cs), _lib.ptr(bias),
                            _lib.ptr(c), _lib.ptr(y)))
    # float64 products and sums of int8 values stay below 2^53 here: exact
    want = (a.astype(np.float64) @ w.astype(np.float64).T).astype(np.int64)
    assert np.array_equal(c.astype(np.int64), want)
    yw = ((want.astype(np.float32) * rs[:, None]) * cs[None, :]) + bias[None, :]
    assert np.array_equal(y, yw.astype(np.float32))


def slice_planes(x):
    """CPU restatement of mc_sm100.cuh slice3 (float32 arithmetic, round half to even)."""
    x = x.astype(np.float32)
    m = np.max(np.abs(x), axis=1)
    inv = np.where(m >= np.float32(1e-30), np.float32(127.0) / np.where(m > 0, m, 1).astype(np.float32),
                   np.float32(0)).astype(np.float32)
    q = (x * inv[:, None]).astype(np.float32)
    d1 = np.rint(q).astype(np.float32)
    t2 = ((q - d1) * np.float32(254)).astype(np.float32)
    d2 = np.rint(t2).astype(np.float32)
    t3 = ((t2 - d2) * np.float32(254)).astype(np.float32)
    d3 = np.rint(t3).astype(np.float32)
    step = np.where(m >= np.float32(1e-30), m * np.float32(1.0 / 127.0), 0).astype(np.float32)
    return d1.astype(np.int64), d2.astype(np.int64), d3.astype(np.int64), step


# K up to 1536 runs the weights-on-M kernel (32 activation rows sliced once per CTA, every weight
# tile streamed past them); K = 2048 the one-output-tile-per-CTA kernel. Both must give the exact
# plane accumulators and the same float32 outputs.
@pytest.mark.parametrize("m,n,k", [(256, 128, 384), (300, 256, 1152), (128, 512, 192), (256, 2048, 128),
                                   (45, 384, 1536), (256, 256, 2048)])
def test_gemm_f32a_slices_exact(m, n, k, oracle):
    import torch
    rng = np.random.default_rng(6)
    x = (rng.standard_normal((m, k)) * rng.uniform(0.1, 3, (m, 1))).astype(np.float32)
    x[0] = 0  # an all-zero row
    w = _rng_i8(rng, (n, k))
    bias = rng.standard_normal(n).astype(np.float32)
    scale = np.float32(0.0123)
    dev = torch.device("cuda:0")
    tx, tw, tb = (torch.from_numpy(v).to(dev) for v in (x, w, bias))
    ty = torch.zeros((m, n), dtype=torch.float32, device=dev)
    ts = torch.zeros((3, m, n), dtype=torch.int32, device=dev)
    tr = torch.zeros(m, dtype=torch.float32, device=dev)
    _lib.check(_lib.lib().mc_gemm_f32a_dev(_lib.ptr(tx), _lib.ptr(tw), m, n, k, float(scale), _lib.ptr(tb),
                                           _lib.ptr(ty), _lib.ptr(ts), _lib.ptr(tr), None))
    torch.cuda.synchronize()
    y, s = ty.cpu().numpy(), ts.cpu().numpy()
    d1, d2, d3, step = slice_planes(x)
    W = w.astype(np.int64).T
    for p, d in enumerate((d1, d2, d3)):
        assert np.array_equal(s[p].astype(np.int64), d @ W), p
    comb = (s[0].astype(np.float64) + (s[1].astype(np.float64) + s[2].astype(np.float64) * (1 / 254.0)) * (1 / 254.0))
    dot = (comb * step.astype(np.float64)[:, None]).astype(np.float32)
    want = ((dot * scale).astype(np.float32) + bias).astype(np.float32)
    assert np.array_equal(y, want)
    # Against the reference's float32 INT8 product (the oracle's MatVecInt8).
    for r in range(0, m, max(1, m // 16)):
        ref = oracle.matvec_i8(w.reshape(-1), n, k, float(scale), x[r], bias)
        assert np.max(np.abs(ref - y[r])) <= 1e-5 * max(1.0, np.max(np.abs(ref))), r
