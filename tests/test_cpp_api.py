"""The voxcpm C++ API over libvxb: callers written like the reference's own
(decode_waveform; AudioVAE::encode with last_input_tensor) compile, link and
-- on a B200 -- decode / encode within the stated tolerances of the reference
(golden outputs of its own code)."""
import os
import subprocess

import numpy as np
import pytest

from cpp_api import build_api_decode, build_api_encode
from models import model_path

G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_cpp_caller_compiles_and_fails_loudly_without_gpu(tmp_path):
    import torch

    exe = build_api_decode(str(tmp_path))
    if torch.cuda.is_available():
        return
    z = np.zeros((1, 64, 6), np.float32)
    z.tofile(tmp_path / "z.f32")
    path, _ = model_path(quant="f16", seed=0)
    r = subprocess.run([exe, path, str(tmp_path / "z.f32"), "6", "1", str(tmp_path / "o.f32")],
                       capture_output=True, text=True)
    assert r.returncode == 7 and "voxcpm::Error" in r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("name,tol", [("f16_full_t6", 2e-3), ("q4_full_t6", 5e-3)])
def test_cpp_caller_decodes_like_the_reference(tmp_path, name, tol):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    exe = build_api_decode(str(tmp_path))
    f = np.load(os.path.join(G, f"decode_{name}.npz"))
    quant = "f16" if name.startswith("f16") else "q4_0"
    path, sha = model_path(quant=quant, seed=0)
    assert sha == str(f["sha"])
    z = np.ascontiguousarray(f["z"], dtype=np.float32)
    steps, _, T = z.shape
    z.tofile(tmp_path / "z.f32")
    r = subprocess.run([exe, path, str(tmp_path / "z.f32"), str(T), str(steps), str(tmp_path / "o.f32")],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    got = np.fromfile(tmp_path / "o.f32", dtype=np.float32).reshape(steps, -1)
    assert np.abs(got - f["l1"]).max() <= tol


@pytest.mark.gpu
def test_cpp_load_from_store_rejects_missing_encoder_names(tmp_path):
    """load_from_store returns false when a required tensor is missing (exit 3)."""
    import torch

    import vxb_synth as S

    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    exe = build_api_decode(str(tmp_path))
    w = S.GGUFWriter()
    w.u32("voxcpm_audio_vae_config_encoder_dim", 128)
    w.u32("voxcpm_audio_vae_config_decoder_dim", 1536)
    w.u32("voxcpm_audio_vae_config_latent_dim", 64)
    w.u32("voxcpm_audio_vae_config_sample_rate", 16000)
    w.i32_array("voxcpm_audio_vae_config_encoder_rates", [2, 5, 8, 8])
    w.i32_array("voxcpm_audio_vae_config_decoder_rates", [8, 8, 5, 2])
    w.tensor("audio_vae.decoder.model.0.bias", (64,), S.GGML_F16, np.zeros(64, np.float16).tobytes())
    (tmp_path / "m.gguf").write_bytes(w.tobytes())
    np.zeros((1, 64, 6), np.float32).tofile(tmp_path / "z.f32")
    r = subprocess.run([exe, str(tmp_path / "m.gguf"), str(tmp_path / "z.f32"), "6", "1", str(tmp_path / "o.f32")],
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 3, (r.returncode, r.stderr)


def test_cpp_encode_caller_compiles_and_fails_loudly_without_gpu(tmp_path):
    """Without a B200 the backend constructor throws voxcpm::Error (exit 7): no CPU fallback."""
    import torch

    exe = build_api_encode(str(tmp_path))
    if torch.cuda.is_available():
        return
    np.zeros((1, 640), np.float32).tofile(tmp_path / "a.f32")
    path, _ = model_path(quant="f16", seed=0)
    r = subprocess.run([exe, path, str(tmp_path / "a.f32"), "640", "1", str(tmp_path / "o.f32")],
                       capture_output=True, text=True)
    assert r.returncode == 7 and "voxcpm::Error" in r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("name,tol", [("f16_t6", 5e-3), ("q4_t6", 6e-2)])
def test_cpp_caller_encodes_like_the_reference(tmp_path, name, tol):
    """Relative to max|latent| (the encoder tolerances of test_gpu_encode.py)."""
    import ast

    import torch

    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    exe = build_api_encode(str(tmp_path))
    f = np.load(os.path.join(G, f"encode_{name}.npz"))
    path, sha = model_path(**ast.literal_eval(str(f["model"])))
    assert sha == str(f["sha"])
    a = np.ascontiguousarray(f["audio"], dtype=np.float32)
    steps, n = a.shape
    a.tofile(tmp_path / "a.f32")
    r = subprocess.run([exe, path, str(tmp_path / "a.f32"), str(n), str(steps), str(tmp_path / "o.f32")],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    got = np.fromfile(tmp_path / "o.f32", dtype=np.float32).reshape(f["latent"].shape)
    ref = f["latent"]
    assert np.abs(got - ref).max() <= tol * np.abs(ref).max()
