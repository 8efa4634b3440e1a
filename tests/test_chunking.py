"""Time-chunked decode: receptive field, chunk arithmetic, and exactness of
halo chunks checked on the C oracle (CPU, small-width model with the
VoxCPM rates; the receptive field does not depend on the width)."""
import numpy as np
import pytest

import chunking as CH
import oracle_lib as O
import vxb_synth as S
from models import model_path


def test_receptive_field_voxcpm():
    rf = CH.receptive_field_frames((8, 8, 5, 2))
    # 6 + (1 + 78/8) + (1/8 + 78/64) + (1/64 + 78/320) + (1/320 + 78/640) + 6/640
    assert abs(rf - 18.4875) < 1e-12
    assert CH.min_halo((8, 8, 5, 2)) == 19


@pytest.mark.parametrize("T,parts,halo", [(1500, 8, 20), (1500, 3, 19), (7, 8, 20), (1, 1, 0), (64, 5, 19)])
def test_split_covers_every_frame_once(T, parts, halo):
    ch = CH.split(T, parts, halo)
    assert len(ch) == min(T, parts)
    assert ch[0].start == 0 and ch[0].keep == 0 and ch[-1].end == T
    for a, b in zip(ch, ch[1:]):
        assert a.end == b.keep
    for c in ch:
        assert c.keep - c.start == min(halo, c.keep)
    sizes = [c.end - c.keep for c in ch]
    assert max(sizes) - min(sizes) <= 1


def test_chunks_of_and_bad_arguments():
    ch = CH.chunks_of(100, 32, 19)
    assert [(c.start, c.keep, c.end) for c in ch] == [(0, 0, 32), (13, 32, 64), (45, 64, 96), (77, 96, 100)]
    for bad in [(0, 1, 0), (5, 0, 1), (5, 1, -1)]:
        with pytest.raises(ValueError):
            CH.split(*bad)


@pytest.fixture(scope="module")
def small_model():
    path, _ = model_path(quant="f16", seed=3, decoder_dim=128)
    m = O.OracleModel(path)
    yield m
    m.close()


def test_halo_chunks_reproduce_full_decode(small_model):
    """Chunks with the minimal halo (19 frames) reproduce the full decode's
    kept samples exactly; an 18-frame halo does not."""
    m, T, hop = small_model, 72, 640
    z = S.make_latents(1, T, latent_dim=m.latent_dim, seed=9, ar=0.9)[0, 0]
    full = m.decode(z[None], O.MODE_EXACT)
    for halo, exact in ((19, True), (24, True), (18, False)):
        worst = 0.0
        for c in CH.chunks_of(T, 25, halo):
            part = m.decode(z[None, :, c.start:c.end], O.MODE_EXACT)
            kept = part[0, c.halo * hop:]
            worst = max(worst, float(np.abs(kept - full[0, c.keep * hop:c.end * hop]).max()))
        if exact:
            assert worst == 0.0, (halo, worst)
        else:
            assert worst > 0.0, halo


class _OracleDecoder:
    """The oracle behind the StreamingDecoder's duck-typed Decoder interface."""

    def __init__(self, m):
        self.m = m
        self.hop = m.hop

    def config(self):
        return {"latent_dim": self.m.latent_dim, "rates": self.m.rates}

    def decode(self, z):
        return self.m.decode(z, O.MODE_EXACT)


def test_streaming_decoder_equals_continuous_decode(small_model):
    """Stateful streaming (history + new frames, halo >= the receptive field)
    emits exactly the continuous decode of the whole stream, for any step
    sizes; a halo below the receptive field is refused."""
    import vxb

    m, hop = small_model, 640
    z = S.make_latents(1, 40, latent_dim=m.latent_dim, seed=12, ar=0.9)[0]  # [1, L, 40]
    full = m.decode(z, O.MODE_EXACT)
    sd = vxb.StreamingDecoder(_OracleDecoder(m), batch=1)
    assert sd.halo == CH.min_halo(m.rates)
    got, t = [], 0
    for n in (6, 6, 1, 13, 6, 8):
        got.append(sd.push(z[:, :, t:t + n]))
        t += n
    got = np.concatenate(got, axis=1)
    assert got.shape == (1, 40 * hop)
    assert np.array_equal(got, full)
    with pytest.raises(ValueError):
        vxb.StreamingDecoder(_OracleDecoder(m), batch=1, halo=CH.min_halo(m.rates) - 1)


def test_encoder_receptive_field_voxcpm():
    """6 + sum_b r_b (78 + 2 ceil(s_b/2)) + 2 * 640 = 9274 samples = 14.49 frames for rates 2,5,8,8."""
    assert abs(CH.encoder_receptive_field_frames((2, 5, 8, 8)) - 9274 / 640) < 1e-12
    assert CH.min_encoder_halo((2, 5, 8, 8)) == 15


class _OracleEncoder:
    """The oracle behind the Decoder methods encode_chunked uses."""

    def __init__(self, m, rates):
        self.m, self.rates = m, rates
        self.encoder_hop = int(np.prod(rates))

    def encoder_config(self):
        return {"encoder_dim": 0, "rates": list(self.rates)}

    def encode(self, audio):
        return self.m.encode(audio, O.MODE_EXACT)


def test_chunked_encode_equals_full_encode():
    """A waveform encoded in windows with the minimal halo (15 frames) equals
    the one-shot encode; a 14-frame halo does not."""
    import vxb

    rates = (2, 5, 8, 8)
    path, _ = model_path(quant="f16", seed=4, decoder_dim=128, encoder=True, encoder_dim=32)
    m = O.OracleModel(path)
    try:
        a = S.make_audio(29 * 640 - 77, 1, seed=17)[0]
        full = m.encode(a[None], O.MODE_EXACT)[0]
        enc = _OracleEncoder(m, rates)
        got = vxb.Decoder.encode_chunked(enc, a, chunk=10)
        assert got.shape == full.shape == (64, 29)
        assert np.array_equal(got, full)
        with pytest.raises(ValueError):
            vxb.Decoder.encode_chunked(enc, a, chunk=10, halo=14)
        short = vxb.Decoder._encode_windows(enc, a, 10, 14)  # the window loop without the check
        assert not np.array_equal(short, full)
    finally:
        m.close()
