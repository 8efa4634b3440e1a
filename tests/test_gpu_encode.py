"""End-to-end encode (waveform -> latent) on the GPU, through the C ABI.

Against the reference's own AudioVAE::encode (golden outputs in tests/golden/)
and against the C oracle in its GPU-numerics mode (fp16 conv operands, fp32
accumulation).  Tolerances are relative to max|latent|: the encoder has 16
conv layers whose inputs are rounded (fp16 here; fp16 or Q8_0 in the
reference), and a 1-ulp accumulation-order difference that straddles a
rounding boundary moves one rounded input by a whole step; compounded over
the layers this reaches about 1e-3 of the latent's scale for F16 weights and
a few per cent against the reference's Q8_0 activations for Q4_0 weights
(see test_oracle_golden.py: the oracle itself sits there too).
"""
import ast
import os

import numpy as np
import pytest

import oracle_lib as O
import vxb_synth as S
from models import model_path

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# relative to max|latent|: vs the reference / vs the oracle's GPU-numerics mode
TOL_REF = {"f16": 5e-3, "q4_0": 6e-2}
TOL_ORACLE = {"f16": 3e-3, "q4_0": 3e-3}


@pytest.fixture(scope="module")
def vxb():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import vxb as V

    V.lib()
    return V


_ctx = {}


def encoder_for(vxb, q, **mk):
    """(Decoder, OracleModel) of the seed-0 encoder model of quant `q`, or of model kwargs mk."""
    mk = mk or dict(quant=q, seed=0, encoder=True)
    key = repr(sorted(mk.items()))
    if key not in _ctx:
        path, _ = model_path(**mk)
        d = vxb.Decoder(0)
        d.load_gguf(path)
        d.prepare()
        _ctx[key] = (d, O.OracleModel(path))
    return _ctx[key]


def rel_err(got, ref):
    return float(np.abs(got - ref).max() / np.abs(ref).max())


@pytest.mark.parametrize("name", ["f16_t6", "q4_t6", "q4_small_rates"])
def test_encode_matches_reference(vxb, name):
    f = np.load(os.path.join(G, f"encode_{name}.npz"))
    mk = ast.literal_eval(str(f["model"]))
    _, sha = model_path(**mk)
    assert sha == str(f["sha"])
    d, m = encoder_for(vxb, mk["quant"], **mk)
    got = d.encode(f["audio"])
    assert got.shape == f["latent"].shape
    err = rel_err(got, f["latent"])
    assert err <= TOL_REF[mk["quant"]], f"{name}: GPU vs reference encode, relative max|d| {err:.3e}"
    err = rel_err(got, m.encode(f["audio"], O.MODE_GPU))
    assert err <= TOL_ORACLE[mk["quant"]], f"{name}: GPU vs oracle (GPU numerics), relative max|d| {err:.3e}"


@pytest.mark.parametrize("quant", ["f16", "q4_0"])
def test_encode_ragged_length_and_single_frame(vxb, quant):
    """A waveform that is not a hop multiple is zero-padded (the reference's
    preprocess); one latent frame is the smallest plan."""
    d, m = encoder_for(vxb, quant)
    for n in (640, 3 * 640 - 211):
        a = S.make_audio(n, 2, seed=21 + n)
        got = d.encode(a)
        assert got.shape == (2, 64, (n + 639) // 640)
        err = rel_err(got, m.encode(a, O.MODE_GPU))
        assert err <= TOL_ORACLE[quant], f"n={n}: relative max|d| {err:.3e}"


def test_encode_batch_equals_single_waveforms(vxb):
    """Waveforms of a batch are independent: a batch of 3 equals three single encodes."""
    d, _ = encoder_for(vxb, "q4_0")
    a = S.make_audio(4 * 640, 3, seed=5)
    batch = d.encode(a)
    single = np.concatenate([d.encode(a[i : i + 1]) for i in range(3)])
    assert np.abs(batch - single).max() <= 1e-5 * np.abs(single).max()


def test_encode_then_decode_shapes(vxb):
    """The latent layout is the decoder's input layout: encode -> decode round trip of shapes."""
    d, _ = encoder_for(vxb, "f16")
    a = S.make_audio(5 * 640, 1, seed=9)
    z = d.encode(a)
    y = d.decode(z)
    assert y.shape == (1, 5 * 640) and np.isfinite(y).all()


def test_encode_device_entry_point(vxb):
    """vxb_encode_device on device buffers equals vxb_encode on host buffers."""
    d, _ = encoder_for(vxb, "f16")
    a = S.make_audio(2 * 640, 2, seed=13)
    host = d.encode(a)
    ad = torch.from_numpy(a).cuda()
    zd = torch.empty((2, 64, 2), device="cuda")
    d.encode_device(ad, zd)
    d.sync()
    assert np.array_equal(zd.cpu().numpy(), host)


def test_encode_placeholder_encoder_is_an_error(vxb):
    path, _ = model_path(quant="f16", seed=0)
    d = vxb.Decoder(0)
    try:
        d.load_gguf(path)
        d.prepare()
        with pytest.raises(vxb.VxbError) as e:
            d.build_encode_plan(1, 2)
        assert e.value.code == vxb.ERR_INVALID_FORMAT
    finally:
        d.close()


def test_chunked_encode_equals_full(vxb):
    """A long waveform encoded in 8-frame windows with the minimal halo (15
    frames for rates 2,5,8,8) equals the one-shot encode."""
    d, _ = encoder_for(vxb, "f16")
    assert d.encoder_config() == {"encoder_dim": 128, "rates": [2, 5, 8, 8]}
    a = S.make_audio(40 * 640 - 123, 1, seed=27)[0]
    full = d.encode(a[None])[0]
    got = d.encode_chunked(a, chunk=8)
    assert got.shape == full.shape
    assert np.abs(got - full).max() <= 1e-5 * np.abs(full).max()
