"""Single-kernel parity on the GPU, through the C ABI, against the C oracle.

Tolerances: Q4_0 dequantisation is bit-exact; Snake within 1e-5 abs (the
reference's own gate for its polynomial sin vs libm); tensor-core convs are
compared with the oracle's GPU-numerics mode (same fp16 operand rounding)
within 2e-4 relative to the output scale -- only the fp32 accumulation order
differs.
"""
import numpy as np
import pytest

import oracle_lib as O
import vxb_synth as S

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def vxb():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import vxb as V

    V.lib()
    return V


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_q4_0_dequant_bit_exact(vxb):
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(32 * 4096) * 0.1).astype(np.float32)
    q = S.quantize_q4_0(x)
    ref = np.zeros(x.size, np.float32)
    O.lib().vo_dequant_q4_0(O.P(q), x.size, O.P(ref))
    out = torch.empty(x.size, dtype=torch.float32, device="cuda")
    vxb.q4_0_dequant(dev(q.reshape(-1)), x.size, out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_snake_matches_oracle(vxb):
    rng = np.random.default_rng(1)
    N, C = 333, 96
    x = (rng.standard_normal((N, C)) * 4).astype(np.float32)
    x[0, :4] = [0.0, 1500.0, -3000.0, 1e-20]
    alpha = rng.uniform(0.5, 1.5, C).astype(np.float16).astype(np.float32)
    ref = np.zeros_like(x)
    O.lib().vo_snake(O.P(x), O.P(alpha), C, N, O.P(ref))
    y = torch.empty((N, C), dtype=torch.float32, device="cuda")
    vxb.snake(dev(x), dev(alpha), C, N, y)
    torch.cuda.synchronize()
    np.testing.assert_allclose(y.cpu().numpy(), ref, rtol=1e-6, atol=1e-5)


def _pw_case(vxb, K, M, N, wt, res, snk, out16, seed):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((M, K)) * (0.5 / np.sqrt(K))).astype(np.float32)
    x = rng.standard_normal((N, K)).astype(np.float32)
    x16 = x.astype(np.float16)
    b = (rng.standard_normal(M) * 0.01).astype(np.float32)
    r = rng.standard_normal((N, M)).astype(np.float32) if res else None
    alpha = rng.uniform(0.5, 1.5, M).astype(np.float32) if snk else None
    if wt == "f16":
        raw = W.astype(np.float16)
        Wf, typ = raw.astype(np.float32), vxb.TYPE_F16
        raw_bytes = raw.view(np.uint8).reshape(-1)
    else:
        raw_bytes = S.quantize_q4_0(W).reshape(-1)
        Wf, typ = S.dequantize_q4_0(raw_bytes).reshape(M, K), vxb.TYPE_Q4_0
    ref = np.zeros((N, M), np.float32)
    O.lib().vo_pointwise(O.P(np.ascontiguousarray(Wf)), O.P(raw_bytes), 1 if wt == "f16" else 2, O.P(b),
                         O.P(r) if res else None, O.P(x16.astype(np.float32)), N, K, M, O.MODE_GPU, O.P(ref))
    if snk:
        tmp = ref.copy()
        O.lib().vo_snake(O.P(tmp), O.P(alpha), M, N, O.P(ref))
    y = torch.empty((N, M), dtype=torch.float16 if out16 else torch.float32, device="cuda")
    vxb.pointwise(dev(raw_bytes), typ, K, M, dev(x16), N, dev(b), y, res=dev(r) if res else None,
                  snake_alpha=dev(alpha) if snk else None, out_f16=out16)
    torch.cuda.synchronize()
    got = y.float().cpu().numpy()
    scale = max(1.0, float(np.abs(ref).max()))
    tol = (2e-3 if out16 else 2e-4) * scale
    err = float(np.abs(got - ref).max())
    assert err <= tol, f"K={K} M={M} N={N} {wt}: max|d| {err:.3e} > {tol:.3e}"


@pytest.mark.parametrize("wt", ["f16", "q4"])
@pytest.mark.parametrize("K,M,N", [(64, 1536, 6), (1536, 128, 16), (768, 768, 48), (384, 384, 384),
                                   (192, 192, 1920), (96, 96, 3840), (96, 96, 77), (384, 192, 5000),
                                   (768, 384, 700)])
def test_pointwise_matches_oracle(vxb, K, M, N, wt):
    _pw_case(vxb, K, M, N, wt, res=False, snk=False, out16=False, seed=K + M + N)


@pytest.mark.parametrize("wt", ["f16", "q4"])
@pytest.mark.parametrize("res,snk,out16", [(True, False, False), (True, True, True), (False, True, True),
                                           (True, True, False)])
def test_pointwise_epilogues(vxb, wt, res, snk, out16):
    _pw_case(vxb, 384, 192, 300, wt, res, snk, out16, seed=7)


@pytest.mark.parametrize("res,snk,out16", [(True, False, False), (False, False, False), (True, True, True)])
def test_pointwise_resident_weight_column(vxb, res, snk, out16):
    """Q4_0 at 384 channels over enough tokens that every CTA keeps its m tile's
    dequantised weight column resident across several n tiles (the resident-A
    kernels: fp32 output with the 4-deep residual ring, fp16 Snake output with
    the staging buffers); 12 871 tokens leave a ragged last tile."""
    _pw_case(vxb, 384, 384, 12871, "q4", res, snk, out16, seed=11)


@pytest.mark.parametrize("wt", ["f16", "q4"])
@pytest.mark.parametrize("Cin,Cout,s,B,T", [(1536, 768, 8, 1, 6), (768, 384, 8, 1, 48), (384, 192, 5, 1, 384),
                                            (192, 96, 2, 1, 1920), (384, 192, 5, 3, 7), (192, 96, 2, 2, 300),
                                            (64, 32, 3, 2, 50), (128, 64, 4, 1, 1),
                                            # enough token tiles for the tokens-as-M kernel (Q4_0), with
                                            # sequence starts inside its 124-token tiles
                                            (384, 192, 5, 8, 400), (192, 96, 2, 5, 2500)])
def test_convt_matches_oracle(vxb, Cin, Cout, s, B, T, wt):
    rng = np.random.default_rng(Cin + s + T)
    K = 2 * s
    Wfold = (rng.standard_normal((Cin, K * Cout)) * (0.5 / np.sqrt(Cin))).astype(np.float32)  # [ci][co*K+k]
    x = rng.standard_normal((B * T, Cin)).astype(np.float32)
    x16 = x.astype(np.float16)
    b = (rng.standard_normal(Cout) * 0.01).astype(np.float32)
    if wt == "f16":
        raw = Wfold.astype(np.float16)
        deq = raw.astype(np.float32)
        raw_bytes, typ = raw.view(np.uint8).reshape(-1), vxb.TYPE_F16
    else:
        raw_bytes = S.quantize_q4_0(Wfold).reshape(-1)
        deq = S.dequantize_q4_0(raw_bytes).reshape(Cin, K * Cout)
        typ = vxb.TYPE_Q4_0
    Wg = np.ascontiguousarray(deq.T)  # [co*K + k][ci]
    ref = np.zeros((B * T * s, Cout), np.float32)
    O.lib().vo_convt(O.P(Wg), 1, 2, O.P(b), O.P(x16.astype(np.float32)), T, B, Cin, Cout, s, O.MODE_GPU, O.P(ref))
    y = torch.empty((B * T * s, Cout), dtype=torch.float32, device="cuda")
    vxb.convt(dev(raw_bytes), typ, Cin, Cout, s, dev(x16), B, T, dev(b), y)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    err = float(np.abs(got - ref).max())
    tol = 2e-4 * max(1.0, float(np.abs(ref).max()))
    assert err <= tol, f"convt {Cin}->{Cout} s={s} B={B} T={T} {wt}: max|d| {err:.3e} > {tol:.3e}"


def test_snake_error_bound_wide_range(vxb):
    """Snake over |alpha * x| up to 2e5 and alpha from 0.05 to 20 against fp64:
    |y - y64| <= inv * 1.2e-6 + |x| * 2^-22 (the bound the kernel's sin^2
    states) plus the fp32 rounding of y."""
    mags = np.logspace(-4, 4, 2001)
    x = np.concatenate([mags, -mags, [0.0, 1e-30, 3.0e4, -9.9e3]]).astype(np.float32)
    alpha = np.array([0.05, 0.5, 1.0, 1.37, 5.0, 20.0], np.float32)
    C, N = alpha.size, x.size
    X = np.repeat(x[:, None], C, axis=1).copy()
    y = torch.empty((N, C), dtype=torch.float32, device="cuda")
    vxb.snake(dev(X), dev(alpha), C, N, y)
    torch.cuda.synchronize()
    inv = (1.0 / (alpha.astype(np.float32) + np.float32(1e-9))).astype(np.float64)
    X64 = X.astype(np.float64)
    y64 = X64 + inv * np.sin(alpha.astype(np.float64) * X64) ** 2
    err = np.abs(y.cpu().numpy().astype(np.float64) - y64)
    bound = inv * 1.2e-6 + np.abs(X64) * 2.0 ** -22 + np.abs(y64) * 2.0 ** -24
    assert np.all(err <= bound), float(np.max(err / bound))


@pytest.mark.parametrize("C,d,B,T,wt,snk,out16", [
    (96, 9, 2, 3000, "q4", False, False),    # fused residual-unit kernel
    (96, 1, 1, 700, "f16", True, False),     # fused, final Snake (fp32)
    (64, 3, 3, 400, "q4", True, True),       # fused, next block's Snake (fp16)
    (192, 3, 2, 9600, "q4", False, False),   # prologue + pointwise-only kernel (150 tiles of 128 tokens)
    (192, 9, 2, 9600, "f16", True, True),    # the same with Snake + fp16 output
    (192, 1, 1, 500, "q4", False, False),    # prologue + pointwise GEMM (few tiles)
    (384, 3, 1, 300, "f16", True, False),    # prologue + pointwise GEMM (wide stage)
])
def test_residual_unit_matches_oracle(vxb, C, d, B, T, wt, snk, out16):
    """vxb_residual_unit (every kernel path the decoder uses for a residual
    unit) against the oracle's snake -> dilated dw -> snake -> pointwise
    (fp16 operand rounding) -> + bias + x [-> Snake] composition."""
    rng = np.random.default_rng(C * 7 + d + T)
    N = B * T
    x = rng.standard_normal((N, C)).astype(np.float32)
    a1 = rng.uniform(0.5, 1.5, C).astype(np.float32)
    a2 = rng.uniform(0.5, 1.5, C).astype(np.float32)
    ao = rng.uniform(0.5, 1.5, C).astype(np.float32) if snk else None
    dw = (rng.standard_normal((C, 7)) * (0.5 / np.sqrt(7))).astype(np.float32)
    db = (rng.standard_normal(C) * 0.01).astype(np.float32)
    pb = (rng.standard_normal(C) * 0.01).astype(np.float32)
    W = (rng.standard_normal((C, C)) * (0.5 / np.sqrt(C))).astype(np.float32)
    if wt == "f16":
        raw = W.astype(np.float16)
        Wf, typ, raw_bytes = raw.astype(np.float32), vxb.TYPE_F16, raw.view(np.uint8).reshape(-1)
    else:
        raw_bytes = S.quantize_q4_0(W).reshape(-1)
        Wf, typ = S.dequantize_q4_0(raw_bytes).reshape(C, C), vxb.TYPE_Q4_0
    L = O.lib()
    h1 = np.zeros_like(x)
    L.vo_snake(O.P(x), O.P(a1), C, N, O.P(h1))
    h2 = np.zeros_like(x)
    L.vo_dwconv(O.P(h1), O.P(dw), O.P(db), C, T, B, d, O.P(h2))
    h3 = np.zeros_like(x)
    L.vo_snake(O.P(h2), O.P(a2), C, N, O.P(h3))
    ref = np.zeros_like(x)
    L.vo_pointwise(O.P(np.ascontiguousarray(Wf)), O.P(raw_bytes), 1 if wt == "f16" else 2, O.P(pb), O.P(x), O.P(h3),
                   N, C, C, O.MODE_GPU, O.P(ref))
    if snk:
        tmp = ref.copy()
        L.vo_snake(O.P(tmp), O.P(ao), C, N, O.P(ref))
    y = torch.empty((N, C), dtype=torch.float16 if out16 else torch.float32, device="cuda")
    vxb.residual_unit(dev(raw_bytes), typ, C, d, dev(x), B, T, dev(a1), dev(dw), dev(db), dev(a2), dev(pb), y,
                      out_alpha=dev(ao) if snk else None, out_f16=out16)
    torch.cuda.synchronize()
    got = y.float().cpu().numpy()
    scale = max(1.0, float(np.abs(ref).max()))
    tol = (2e-3 if out16 else 5e-4) * scale
    err = float(np.abs(got - ref).max())
    assert err <= tol, f"C={C} d={d} B={B} T={T} {wt}: max|d| {err:.3e} > {tol:.3e}"
