"""End-to-end decode parity on the GPU, through the C ABI (libvxb).

Against the reference (golden L1 outputs of the reference's own code) with the
stated tolerances: max|d| <= 2e-3 for F16 models and <= 5e-3 for Q4_0-mixed
models; and against the C oracle in its GPU-numerics mode (same fp16 operand
rounding) with a tight 5e-4.
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
DECODES = sorted(n[len("decode_"):-4] for n in os.listdir(G) if n.startswith("decode_"))


@pytest.fixture(scope="module")
def vxb():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import vxb as V

    V.lib()
    return V


_decoders = {}


def decoder_for(vxb, **mk):
    key = repr(sorted(mk.items()))
    if key not in _decoders:
        path, _ = model_path(**mk)
        d = vxb.Decoder(0)
        d.load_gguf(path)
        d.prepare()
        _decoders[key] = d
    return _decoders[key]


@pytest.mark.parametrize("name", DECODES)
def test_decode_matches_reference(vxb, name):
    f = np.load(os.path.join(G, f"decode_{name}.npz"))
    mk = ast.literal_eval(str(f["model"]))
    path, sha = model_path(**mk)
    assert sha == str(f["sha"])
    d = decoder_for(vxb, **mk)
    z = f["z"]
    got = np.stack([d.decode(z[s : s + 1])[0] for s in range(z.shape[0])])
    tol = 2e-3 if mk["quant"] == "f16" else 5e-3
    err = float(np.abs(got - f["l1"]).max())
    assert err <= tol, f"{name}: GPU vs reference L1 max|d| {err:.3e} > {tol}"
    m = O.OracleModel(path)
    ref = np.stack([m.decode(z[s : s + 1], O.MODE_GPU)[0] for s in range(z.shape[0])])
    err2 = float(np.abs(got - ref).max())
    assert err2 <= 5e-4, f"{name}: GPU vs oracle (GPU numerics) max|d| {err2:.3e}"


@pytest.mark.parametrize("quant", ["f16", "q4_0"])
def test_stages_match_oracle(vxb, quant):
    """Every materialised intermediate (transposed conv, residual units 0/1)."""
    mk = dict(quant=quant, seed=0)
    path, _ = model_path(**mk)
    d = decoder_for(vxb, **mk)
    z = S.make_latents(1, 6, seed=21)[:, 0]
    d.decode(z)
    m = O.OracleModel(path)
    for b in range(4):
        for k in range(3):
            st = 2 + 4 * b + k
            ref = m.decode(z, O.MODE_GPU, stage=st)
            got = d.debug_stage(st, ref.size)
            err = float(np.abs(got - ref).max())
            assert err <= 5e-4 * max(1.0, float(np.abs(ref).max())), f"stage {st}: {err:.3e}"


@pytest.mark.parametrize("quant", ["f16", "q4_0"])
def test_batch_equals_independent_decodes(vxb, quant):
    d = decoder_for(vxb, quant=quant, seed=0)
    z = S.make_latents(1, 6, seed=22, batch=5)[0]
    together = d.decode(z)
    apart = np.stack([d.decode(z[i : i + 1])[0] for i in range(5)])
    assert np.abs(together - apart).max() <= 1e-5


def test_graph_and_launch_list_agree(vxb):
    d = decoder_for(vxb, quant="q4_0", seed=0)
    z = S.make_latents(1, 6, seed=23)[:, 0]
    d.build_plan(1, 6, graph=True)
    a = d.decode(z)
    d.build_plan(1, 6, graph=False)
    b = d.decode(z)
    assert np.array_equal(a, b)
    d.build_plan(1, 6, graph=True)


@pytest.mark.parametrize("quant", ["f16", "q4_0"])
def test_causal_prefix_property(vxb, quant):
    """The decoder is causal: decoding the first t frames reproduces the first
    t*hop samples of the full decode (size-independent check at T=300)."""
    d = decoder_for(vxb, quant=quant, seed=0)
    z = S.make_latents(1, 300, seed=24, ar=0.9)[:, 0]
    full = d.decode(z)
    for t in (1, 7, 64, 150):
        part = d.decode(np.ascontiguousarray(z[:, :, :t]))
        assert np.abs(part - full[:, : t * 640]).max() <= 1e-5, t


@pytest.mark.parametrize("quant", ["f16", "q4_0"])
def test_chunked_decode_equals_full(vxb, quant):
    """A long utterance decoded in 64-frame windows with the minimal halo
    (19 frames for rates 8,8,5,2) equals the one-shot decode."""
    d = decoder_for(vxb, quant=quant, seed=0)
    assert d.config() == {"latent_dim": 64, "decoder_dim": 1536, "rates": [8, 8, 5, 2]}
    z = S.make_latents(1, 300, seed=25, ar=0.9)[0, 0]
    full = d.decode(z[None])[0]
    got = d.decode_chunked(z, chunk=64)
    assert np.abs(got - full).max() <= 1e-5


@pytest.mark.parametrize("quant", ["f16", "q4_0"])
def test_streaming_decoder_equals_continuous_decode(vxb, quant):
    """Opt-in stateful streaming: two streams pushed 6 frames at a time (then
    an odd step) emit the continuous decode of each whole stream."""
    d = decoder_for(vxb, quant=quant, seed=0)
    z = S.make_latents(1, 45, seed=31, batch=2)[0]  # [2, 64, 45]
    full = d.decode(z)
    sd = vxb.StreamingDecoder(d, batch=2)
    parts, t = [], 0
    for n in (6,) * 7 + (3,):
        parts.append(sd.push(z[:, :, t:t + n]))
        t += n
    got = np.concatenate(parts, axis=1)
    assert got.shape == full.shape
    assert np.abs(got - full).max() <= 1e-5


def test_decode_rejects_bad_shapes(vxb):
    d = decoder_for(vxb, quant="f16", seed=0)
    with pytest.raises(vxb.VxbError) as e:
        d.build_plan(1, 0)
    assert e.value.code == vxb.ERR_INVALID_ARGUMENT
    with pytest.raises(vxb.VxbError):
        d.build_plan(0, 6)


def test_missing_tensor_reported(vxb, tmp_path):
    path, _ = model_path(quant="f16", seed=0)
    d = vxb.Decoder(0)
    d.set_config(64, 1536, [8, 8, 5, 2])
    with pytest.raises(vxb.VxbError) as e:
        d.prepare()
    assert e.value.code == vxb.ERR_MISSING_TENSOR
    with pytest.raises(vxb.VxbError) as e:
        d.build_plan(1, 6)
    assert e.value.code == vxb.ERR_NOT_READY
    with pytest.raises(vxb.VxbError) as e:
        d.load_gguf(str(tmp_path / "absent.gguf"))
    assert e.value.code == vxb.ERR_FILE_NOT_FOUND
    d.close()


def test_sample_rate_conditioning_refused(vxb):
    """A model carrying the reference's optional sample-rate conditioning
    tensors (src/audio-vae.cpp:389-396) is refused at prepare, not decoded
    without the conditioning."""
    path, _ = model_path(quant="f16", seed=0)
    d = vxb.Decoder(0)
    d.load_gguf(path)
    d.upload("audio_vae.decoder.sr_cond_model.2.scale_embed.weight", vxb.TYPE_F32, [4, 768],
             np.zeros(4 * 768, np.float32).tobytes())
    with pytest.raises(vxb.VxbError) as e:
        d.prepare()
    assert e.value.code == vxb.ERR_INVALID_FORMAT
    d.close()
