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


def big(name):
    """A benchmark-shaped fixture (reference outputs) and its model's decoder."""
    f = np.load(os.path.join(G, f"big_decode_{name}.npz"))
    mk = ast.literal_eval(str(f["model"]))
    _, sha = model_path(**mk)
    assert sha == str(f["sha"])
    return f, mk


def test_long_utterance_matches_reference(vxb):
    """The 60 s utterance of the long-form workload (z=[1,64,1500], AR(1) 0.9,
    F16) against the reference's own L1 decode of it: the one-shot decode,
    the decode in 64-frame windows with the minimal 19-frame halo, and the
    opt-in streaming decoder fed 6 frames at a time, each within 2e-3."""
    f, mk = big("f16_c3_t1500")
    d = decoder_for(vxb, **mk)
    assert d.config() == {"latent_dim": 64, "decoder_dim": 1536, "rates": [8, 8, 5, 2]}
    z, ref = f["z"], f["l1"][0]
    full = d.decode(z)[0]
    err = float(np.abs(full - ref).max())
    assert err <= 2e-3, f"one-shot T=1500 vs reference L1 max|d| {err:.3e}"
    chunked = d.decode_chunked(z[0], chunk=64)
    err = float(np.abs(chunked - ref).max())
    assert err <= 2e-3, f"chunked vs reference L1 max|d| {err:.3e}"
    assert float(np.abs(chunked - full).max()) <= 1e-5
    sd = vxb.StreamingDecoder(d, batch=1)
    got = np.concatenate([sd.push(z[:, :, t:t + 6]) for t in range(0, 1500, 6)], axis=1)[0]
    err = float(np.abs(got - ref).max())
    assert err <= 2e-3, f"streaming decoder vs reference L1 max|d| {err:.3e}"


def test_offline_batch_matches_reference(vxb):
    """Two 30 s utterances of the offline workload (z=[2,64,750], AR(1) 0.9,
    Q4_0-mixed), decoded as one batch.

    The reference's Q4_0 path quantises the input of every pointwise conv to
    Q8_0 blocks (8-bit, one scale per 32 values); at this length that alone
    moves its waveform up to 5.6e-3 away from the exact fp32 arithmetic with
    the same Q4_0 weights (the fixture stores that exact decode, made by the
    oracle), more than the 5e-3 the reference comparison allows.  So the GPU
    (fp16 operands) is held to the exact decode at 5e-4, and to the
    reference at 5e-3 or, where the reference's own distance from the exact
    decode exceeds that, at that distance plus 5e-4.  The reference's HEAD
    decode (transposed-conv weights re-quantised to Q8_0 as well) is held the
    same way."""
    f, mk = big("q4_c5_t750x2")
    d = decoder_for(vxb, **mk)
    got = d.decode(f["z"])
    l1 = f["l1"]
    l2 = l1 + f["l2_minus_l1"].astype(np.float32)
    exact = l1 + f["exact_minus_l1"].astype(np.float32)
    e_exact = float(np.abs(got - exact).max())
    assert e_exact <= 5e-4, f"vs exact fp32 arithmetic max|d| {e_exact:.3e}"
    own_l1 = float(np.abs(l1 - exact).max())
    e_l1 = float(np.abs(got - l1).max())
    assert e_l1 <= max(5e-3, own_l1 + 5e-4), f"vs reference L1 max|d| {e_l1:.3e} (L1 vs exact {own_l1:.3e})"
    own_l2 = float(np.abs(l2 - exact).max())
    e_l2 = float(np.abs(got - l2).max())
    assert e_l2 <= max(5e-3, own_l2 + 5e-4), f"vs reference HEAD max|d| {e_l2:.3e} (HEAD vs exact {own_l2:.3e})"
    print(f"offline batch 2 x 750: vs exact {e_exact:.2e}; vs L1 {e_l1:.2e} (L1 vs exact {own_l1:.2e}); "
          f"vs HEAD {e_l2:.2e} (HEAD vs exact {own_l2:.2e})")


def test_batched_streaming_step_matches_reference(vxb):
    """One step of the batched streaming workload (256 streams, z=[256,64,6],
    Q4_0-mixed) decoded as one batch: 8 sampled streams against the
    reference's L1 decode (5e-3) and the oracle's GPU-numerics decode (5e-4)."""
    f, mk = big("q4_c4_b256")
    lk = ast.literal_eval(str(f["latents"]))
    z = S.make_latents(**lk)[0]
    keep = f["keep"]
    assert np.array_equal(z[keep], f["z"])
    d = decoder_for(vxb, **mk)
    got = d.decode(z)[keep]
    err = float(np.abs(got - f["l1"]).max())
    assert err <= 5e-3, f"256-stream step vs reference L1 max|d| {err:.3e}"
    path, _ = model_path(**mk)
    m = O.OracleModel(path)
    ref = m.decode(f["z"], O.MODE_GPU)
    err2 = float(np.abs(got - ref).max())
    assert err2 <= 5e-4, f"256-stream step vs oracle (GPU numerics) max|d| {err2:.3e}"


@pytest.mark.parametrize("quant", ["f16", "q4_0"])
def test_streaming_decoder_matches_oracle(vxb, quant):
    """Opt-in stateful streaming: two streams pushed 6 frames at a time (then
    an odd step) emit the continuous decode of each whole stream, checked
    against the oracle's GPU-numerics decode of the whole streams."""
    mk = dict(quant=quant, seed=0)
    d = decoder_for(vxb, **mk)
    z = S.make_latents(1, 27, seed=31, batch=2)[0]  # [2, 64, 27]
    sd = vxb.StreamingDecoder(d, batch=2)
    parts, t = [], 0
    for n in (6,) * 4 + (3,):
        parts.append(sd.push(z[:, :, t:t + n]))
        t += n
    got = np.concatenate(parts, axis=1)
    path, _ = model_path(**mk)
    ref = O.OracleModel(path).decode(z, O.MODE_GPU)
    assert got.shape == ref.shape
    err = float(np.abs(got - ref).max())
    assert err <= 5e-4, f"streaming decoder vs oracle max|d| {err:.3e}"


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


def test_q4_fp16_cache_gives_the_same_decode(vxb):
    """The opt-in fp16 copies of Q4_0 weights hold the values the GEMMs'
    in-kernel dequantisation produces, so the decode is bit-identical."""
    path, _ = model_path(quant="q4_0", seed=0)
    d = vxb.Decoder(0)
    d.load_gguf(path)
    d.prepare()
    z = S.make_latents(1, 6, seed=41, batch=3)[0]
    a = d.decode(z)
    d.set_q4_fp16_cache(True)
    d.prepare()
    d.build_plan(3, 6)
    b = d.decode(z)
    d.close()
    assert np.array_equal(a, b)


@pytest.mark.parametrize("quant", ["f16", "q4_0"])
def test_layer_state_stream_equals_continuous_decode(vxb, quant):
    """Stateful streaming with per-layer carried context: a stream pushed 6
    frames at a time emits the continuous decode of the whole stream (the
    GPU's one-shot decode to 1e-5, the oracle to 5e-4); after a reset the
    next pushes start a new stream."""
    mk = dict(quant=quant, seed=0)
    d = decoder_for(vxb, **mk)
    z = S.make_latents(1, 30, seed=33)[0, 0]  # [64, 30]
    full = d.decode(z[None])[0]
    st = vxb.LayerStateStream(d, 6)
    got = np.concatenate([st.push(z[:, t:t + 6]) for t in range(0, 30, 6)])
    assert got.shape == full.shape
    err = float(np.abs(got - full).max())
    assert err <= 1e-5, f"stream vs one-shot decode max|d| {err:.3e}"
    path, _ = model_path(**mk)
    ref = O.OracleModel(path).decode(z[None, :, :], O.MODE_GPU)[0]
    assert float(np.abs(got - ref).max()) <= 5e-4
    st.reset()
    again = np.concatenate([st.push(z[:, t:t + 6]) for t in range(0, 12, 6)])
    assert np.array_equal(again, got[: again.size])
    st.close()


def test_layer_state_stream_long_utterance_matches_reference(vxb):
    """The 60 s utterance pushed 6 frames at a time through the stateful
    stream stays within 2e-3 of the reference's continuous L1 decode."""
    f, mk = big("f16_c3_t1500")
    d = decoder_for(vxb, **mk)
    z = f["z"][0]
    st = vxb.LayerStateStream(d, 6)
    got = np.concatenate([st.push(z[:, t:t + 6]) for t in range(0, 1500, 6)])
    st.close()
    err = float(np.abs(got - f["l1"][0]).max())
    assert err <= 2e-3, f"stateful stream vs reference L1 max|d| {err:.3e}"
