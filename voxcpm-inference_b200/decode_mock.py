"""Streaming-capture replay on the GPU decoder (the reference's
vae_decode_mock tool, vae_decode_mock.cpp, on libvxb).

    python voxcpm-inference_b200/decode_mock.py --model-path MODEL.gguf --mock-dir mock \
        [--output out.wav] [--max-steps N] [--compare-wav base.wav] [--batch 256] [--device 0]

Input (the reference's mock-capture layout, vae_decode_mock.cpp:1-23, :415-480):
  mock/manifest.json   {"sample_rate", "patch_len_samples", "calls": [{"index", "file", "z_shape"}]}
  mock/<file>          npz with member z.npy: float32 z [1, latent_dim, T]
  mock/reference_streaming.wav   optional reference for max|delta|
Every capture is decoded independently (full sequence, zero left context)
and the last patch_len_samples samples of each are concatenated
(:1320-1358); captures are decoded `--batch` at a time (the decode has no
batch coupling, so this equals one at a time).  The result is written as
16-bit mono PCM clamped to [-1, 1] (:917-960) and compared with the
reference WAV and --compare-wav (max|delta| and SNR, :1393-1433).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import struct
import sys
import time

import numpy as np


def load_manifest(path: str) -> dict:
    """manifest.json -> {"sample_rate", "patch_len_samples", "calls"} with
    calls sorted by index; raises ValueError on a malformed manifest."""
    with open(path) as f:
        root = json.load(f)
    calls = root.get("calls")
    if not isinstance(calls, list) or not calls:
        raise ValueError(f"manifest has no calls: {path}")
    out = []
    for c in calls:
        if not c.get("file"):
            raise ValueError(f"manifest call without file: {path}")
        out.append({"index": int(c.get("index", 0)), "file": c["file"],
                    "z_shape": [int(v) for v in c.get("z_shape", [])]})
    out.sort(key=lambda c: c["index"])  # stable: equal indices keep file order
    sr, patch = int(root.get("sample_rate", 0)), int(root.get("patch_len_samples", 0))
    if sr <= 0 or patch <= 0:
        raise ValueError(f"manifest missing sample_rate / patch_len_samples: {path}")
    return {"sample_rate": sr, "patch_len_samples": patch, "calls": out}


def read_capture(path: str, z_shape=None) -> np.ndarray:
    """z.npy of a capture npz as float32 [latent_dim, T] (the leading batch of 1 dropped)."""
    with np.load(path) as f:
        if "z" not in f.files:
            raise ValueError(f"npz member not found: z.npy in {path}")
        z = np.asarray(f["z"])
    if z.dtype != np.float32:
        raise ValueError(f"{path}: z must be float32, got {z.dtype}")
    if z_shape and list(z.shape) != list(z_shape):
        raise ValueError(f"capture shape mismatch for {path}: npz {list(z.shape)} vs manifest {list(z_shape)}")
    if z.ndim != 3 or z.shape[0] != 1:
        raise ValueError(f"{path}: z must be [1, latent_dim, T], got {list(z.shape)}")
    return np.ascontiguousarray(z[0])


def write_wav_pcm16(path: str, audio: np.ndarray, sample_rate: int) -> None:
    """Mono 16-bit PCM WAV; samples clamped to [-1, 1], scaled by 32767, rounded to nearest."""
    d = os.path.dirname(path)
    if d:
        os.makedirs(d, exist_ok=True)
    pcm = np.rint(np.clip(np.asarray(audio, np.float32), -1.0, 1.0) * np.float32(32767.0)).astype("<i2")
    data = pcm.tobytes()
    hdr = b"RIFF" + struct.pack("<I", 36 + len(data)) + b"WAVE"
    hdr += b"fmt " + struct.pack("<IHHIIHH", 16, 1, 1, sample_rate, sample_rate * 2, 2, 16)
    hdr += b"data" + struct.pack("<I", len(data))
    with open(path, "wb") as f:
        f.write(hdr + data)


def read_wav(path: str) -> tuple[int, np.ndarray]:
    """(sample_rate, mono float32 samples) of a PCM16 or float32 WAV; channels averaged."""
    with open(path, "rb") as f:
        buf = f.read()
    if buf[:4] != b"RIFF" or buf[8:12] != b"WAVE":
        raise ValueError(f"not a RIFF/WAVE file: {path}")
    pos, fmt, data = 12, None, None
    while pos + 8 <= len(buf):
        cid, size = buf[pos:pos + 4], struct.unpack("<I", buf[pos + 4:pos + 8])[0]
        body = buf[pos + 8:pos + 8 + size]
        if cid == b"fmt ":
            fmt = struct.unpack("<HHIIHH", body[:16])
        elif cid == b"data":
            data = body
        pos += 8 + size + (size & 1)
    if fmt is None or data is None:
        raise ValueError(f"WAV without fmt/data chunk: {path}")
    tag, ch, sr, _, _, bits = fmt
    if tag not in (1, 3) or ch < 1:
        raise ValueError(f"{path}: unsupported WAV format (only PCM / float)")
    bps = bits // 8
    if bps == 0:
        raise ValueError(f"{path}: invalid bits per sample")
    n = len(data) // (bps * ch) * ch  # whole frames
    raw = data[: n * bps]
    if tag == 3 and bits == 32:
        x = np.frombuffer(raw, "<f4").astype(np.float32)
    elif tag == 1 and bits == 16:
        x = np.frombuffer(raw, "<i2").astype(np.float32) / np.float32(32768.0)
    elif tag == 1 and bits == 24:
        b = np.frombuffer(raw, np.uint8).reshape(-1, 3).astype(np.int32)
        v = b[:, 0] | (b[:, 1] << 8) | (b[:, 2] << 16)
        v = np.where(v & 0x800000, v - (1 << 24), v)
        x = v.astype(np.float32) / np.float32(8388608.0)
    elif tag == 1 and bits == 32:
        x = np.frombuffer(raw, "<i4").astype(np.float32) / np.float32(2147483648.0)
    else:
        raise ValueError(f"{path}: unsupported WAV bit depth {bits}")
    if ch > 1:
        x = x.reshape(-1, ch).sum(axis=1, dtype=np.float32) / np.float32(ch)
    return sr, x


def compare(base: np.ndarray, got: np.ndarray) -> tuple[float, float]:
    """(max|delta|, SNR dB) over the common length; SNR = 10 log10(sum base^2 / sum delta^2)."""
    n = min(len(base), len(got))
    b, g = base[:n].astype(np.float64), got[:n].astype(np.float64)
    d = b - g
    err = float(np.sum(d * d))
    snr = 10.0 * math.log10(float(np.sum(b * b)) / err) if err > 0 else math.inf
    return (float(np.abs(d).max()) if n else 0.0), snr


def replay(decoder, mock_dir: str, max_steps: int = 0, batch: int = 256) -> tuple[np.ndarray, int, dict]:
    """Decodes every capture of mock_dir; returns (waveform, sample_rate, stats)."""
    man = load_manifest(os.path.join(mock_dir, "manifest.json"))
    calls = man["calls"][:max_steps] if max_steps > 0 else man["calls"]
    zs = [read_capture(os.path.join(mock_dir, c["file"]), c["z_shape"]) for c in calls]
    patch = man["patch_len_samples"]
    pieces = []
    t0 = time.perf_counter()
    i = 0
    while i < len(zs):
        # one batch of captures of equal shape
        j = i + 1
        while j < len(zs) and j - i < batch and zs[j].shape == zs[i].shape:
            j += 1
        out = decoder.decode(np.stack(zs[i:j]))
        for row in out:
            pieces.append(row[-min(patch, row.size):])
        i = j
    secs = time.perf_counter() - t0
    wave = np.concatenate(pieces) if pieces else np.zeros(0, np.float32)
    return wave, man["sample_rate"], {"calls": len(zs), "seconds": secs}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--model-path", default="models/voxcpm-0.5b-audio-vae-q4_0.gguf")
    ap.add_argument("--mock-dir", default="mock")
    ap.add_argument("--output", "-o", default="assets/out/output_streaming.wav")
    ap.add_argument("--max-steps", type=int, default=0, help="replay only the first N captures (0 = all)")
    ap.add_argument("--compare-wav", default="", help="WAV to compare with (max|delta| and SNR)")
    ap.add_argument("--batch", type=int, default=256, help="captures decoded per call")
    ap.add_argument("--device", type=int, default=0)
    a = ap.parse_args(argv)
    if not os.path.isfile(a.model_path):
        print(f"Error: model GGUF does not exist: {a.model_path}", file=sys.stderr)
        return 1
    if not os.path.isdir(a.mock_dir):
        print(f"Error: mock dir does not exist: {a.mock_dir}", file=sys.stderr)
        return 1
    if a.batch < 1:
        print("Error: --batch must be >= 1", file=sys.stderr)
        return 1
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import vxb

    d = vxb.Decoder(a.device)
    try:
        d.load_gguf(a.model_path)
        d.prepare()
        wave, sr, st = replay(d, a.mock_dir, a.max_steps, a.batch)
    finally:
        d.close()
    audio_s = wave.size / sr
    print(f"Decoded {wave.size} samples ({audio_s:.2f}s) from {st['calls']} captures in {st['seconds']:.3f}s "
          f"(RTF {st['seconds'] / max(audio_s, 1e-9):.4f})", file=sys.stderr)
    write_wav_pcm16(a.output, wave, sr)
    print(f"Saved audio to {a.output}", file=sys.stderr)
    ref = os.path.join(a.mock_dir, "reference_streaming.wav")
    if os.path.isfile(ref):
        rsr, r = read_wav(ref)
        if rsr != sr:
            print(f"Warning: reference sample rate {rsr} != model output sample rate {sr}", file=sys.stderr)
        mx, _ = compare(r, wave)
        print(f"Compare with reference_streaming.wav: length {r.size} vs {wave.size}, max|delta| = {mx:.6e} -> "
              f"{'PASS' if mx == 0.0 else 'DIFF'}", file=sys.stderr)
    else:
        print("No reference_streaming.wav found, skip comparison.", file=sys.stderr)
    if a.compare_wav:
        if not os.path.isfile(a.compare_wav):
            print(f"Error: compare WAV does not exist: {a.compare_wav}", file=sys.stderr)
            return 1
        _, b = read_wav(a.compare_wav)
        mx, snr = compare(b, wave)
        print(f"Compare with {a.compare_wav}: length {b.size} vs {wave.size}, max|delta| = {mx:.6e}, "
              f"SNR = {snr:.1f} dB", file=sys.stderr)
    return 0


if __name__ == "__main__":
    sys.exit(main())
