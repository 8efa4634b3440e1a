"""Capture-replay tool (decode_mock.py): manifest, capture and WAV handling on
the CPU; the end-to-end replay on the GPU."""
import json
import os
import struct

import numpy as np
import pytest

import decode_mock as DM
import vxb_synth as S
from models import model_path


def _mock_dir(tmp_path, steps=5, T=6, patch=640, shuffle=True):
    d = tmp_path / "mock"
    (d / "captures").mkdir(parents=True)
    z = S.make_latents(steps, T, seed=31)[:, 0]  # [steps, 64, T]
    calls = []
    for i in range(steps):
        f = f"captures/decoder_input_{i:04d}.npz"
        np.savez(d / f, z=z[i][None])
        calls.append({"index": i, "file": f, "z_shape": [1, 64, T]})
    if shuffle:
        calls = calls[::-1]
    (d / "manifest.json").write_text(json.dumps({"sample_rate": 16000, "patch_len_samples": patch, "calls": calls}))
    return str(d), z


def test_manifest_sorted_and_validated(tmp_path):
    d, _ = _mock_dir(tmp_path)
    m = DM.load_manifest(os.path.join(d, "manifest.json"))
    assert [c["index"] for c in m["calls"]] == list(range(5)) and m["patch_len_samples"] == 640
    bad = tmp_path / "bad.json"
    bad.write_text(json.dumps({"sample_rate": 16000, "calls": [{"index": 0, "file": "x.npz"}]}))
    with pytest.raises(ValueError):
        DM.load_manifest(str(bad))
    bad.write_text(json.dumps({"sample_rate": 16000, "patch_len_samples": 640, "calls": []}))
    with pytest.raises(ValueError):
        DM.load_manifest(str(bad))


def test_capture_shape_checks(tmp_path):
    d, z = _mock_dir(tmp_path, steps=1)
    f = os.path.join(d, "captures/decoder_input_0000.npz")
    assert np.array_equal(DM.read_capture(f, [1, 64, 6]), z[0])
    with pytest.raises(ValueError):
        DM.read_capture(f, [1, 64, 7])
    np.savez(f, z=z[0][None].astype(np.float64))
    with pytest.raises(ValueError):
        DM.read_capture(f)


def test_wav_roundtrip_and_formats(tmp_path):
    x = np.linspace(-1.2, 1.2, 1001).astype(np.float32)
    p = str(tmp_path / "a.wav")
    DM.write_wav_pcm16(p, x, 16000)
    sr, y = DM.read_wav(p)
    assert sr == 16000 and y.size == x.size
    q = np.rint(np.clip(x, -1, 1) * 32767).astype(np.int16)
    assert np.array_equal(y, q.astype(np.float32) / 32768.0)
    # float32 stereo: channels averaged
    st = np.stack([x, -x * 0.5], axis=1).astype("<f4")
    body = st.tobytes()
    hdr = b"RIFF" + struct.pack("<I", 36 + len(body)) + b"WAVE" + b"fmt " + struct.pack("<IHHIIHH", 16, 3, 2, 8000,
                                                                                        64000, 8, 32)
    (tmp_path / "f.wav").write_bytes(hdr + b"data" + struct.pack("<I", len(body)) + body)
    sr, y = DM.read_wav(str(tmp_path / "f.wav"))
    assert sr == 8000 and np.allclose(y, (x - x * 0.5) / 2, atol=1e-7)


def test_compare_max_and_snr():
    b = np.array([1.0, -1.0, 0.5, 0.0], np.float32)
    mx, snr = DM.compare(b, b)
    assert mx == 0.0 and snr == float("inf")
    mx, snr = DM.compare(b, b + np.float32(0.1))
    assert abs(mx - 0.1) < 1e-6 and abs(snr - 10 * np.log10(2.25 / 0.04)) < 1e-4


@pytest.mark.gpu
def test_replay_matches_per_step_decodes(tmp_path):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import vxb

    d, z = _mock_dir(tmp_path, steps=7)
    path, _ = model_path(quant="q4_0", seed=0)
    dec = vxb.Decoder(0)
    dec.load_gguf(path)
    dec.prepare()
    wave, sr, st = DM.replay(dec, d, batch=3)  # batches of 3, 3, 1
    ref = np.concatenate([dec.decode(z[i][None])[0][-640:] for i in range(7)])
    assert sr == 16000 and st["calls"] == 7 and wave.size == 7 * 640
    assert np.abs(wave - ref).max() <= 1e-5
    out = str(tmp_path / "o.wav")
    dec.close()
    rc = DM.main(["--model-path", path, "--mock-dir", d, "--output", out, "--max-steps", "4"])
    assert rc == 0
    _, y = DM.read_wav(out)
    assert y.size == 4 * 640
    assert np.abs(y - np.clip(ref[: 4 * 640], -1, 1)).max() <= 1.0 / 32767 + 1e-5
    # the same replay compared with its own output: identical
    assert DM.main(["--model-path", path, "--mock-dir", d, "--output", str(tmp_path / "p.wav"), "--max-steps", "4",
                    "--compare-wav", out]) == 0
