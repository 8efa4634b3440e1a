"""Seeded synthetic AudioVAE decoder checkpoints and latents.

The real VoxCPM GGUF files and mock captures are not distributed with the
reference, so every benchmark and parity case runs on weights drawn from a
seed and written in the reference's own GGUF layout:

* tensor names, shapes and KV keys as ``AudioVAE::load_from_store`` /
  ``load_decoder_weights`` read them (reference src/audio-vae.cpp:365-463);
* pointwise weights ``[Cin, Cout]`` (k = 1 folded), transposed-conv weights
  folded ``[2s*Cout, Cin]`` with row ``j = cout*2s + k`` (k fastest,
  audio-vae.cpp:127-136), depthwise ``[7, 1, C]``, final ``[7, C, 1]``,
  Snake alpha ``[1, C, 1]``, biases ``[C]``;
* Q4_0 blocks of 32 with an fp16 scale, quantised with the deterministic
  rounding of ggml's ``quantize_row_q4_0_ref`` (ggml-quants.c:113-145);
* encoder tensors present by name only (``load_encoder_weights`` only checks
  that they exist, audio-vae.cpp:331-363), or with ``encoder=True`` the full
  encoder (audio-vae.cpp:553-570, 640-650): head conv ``[7, 1, E]``, per block
  three residual units, Snake alpha and the strided conv ``[2s, Cin, Cout]``
  (F16) or folded ``[2s*Cin, Cout]`` (Q4_0, row ``j = cin*2s + k``,
  audio-vae.cpp:78-88), then ``fc_mu`` ``[3, C, latent]`` / ``[3*C, latent]``.

Weights: N(0, gain^2 / fan_in) for every conv, alpha ~ U(0.5, 1.5), bias ~
N(0, 0.01^2).  gain = 0.5 keeps the waveform well inside tanh's linear range
(at gain 1.0 the output saturates and parity degenerates).
"""
from __future__ import annotations

import hashlib
import struct

import numpy as np

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0 = 0, 1, 2, 8

DEFAULT_RATES = (8, 8, 5, 2)


# --------------------------------------------------------------------- Q4_0 --

def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    """Rows of float32 -> Q4_0 bytes, bit-exact with quantize_row_q4_0_ref.

    x is flattened in memory order; its length must be a multiple of 32.
    Returns uint8 [n/32, 18] blocks (fp16 d little-endian, then 16 nibble bytes).
    """
    v = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, 32)
    idx = np.argmax(np.abs(v), axis=1)  # first index of the absolute max
    mx = v[np.arange(v.shape[0]), idx]
    d = (mx / np.float32(-8.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    q = (v * inv[:, None]).astype(np.float32) + np.float32(8.5)
    q = np.minimum(15, q.astype(np.int8).astype(np.int16)).astype(np.uint8)
    out = np.empty((v.shape[0], 18), dtype=np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return out


def dequantize_q4_0(blocks: np.ndarray) -> np.ndarray:
    """Q4_0 bytes [n, 18] -> float32 [n*32] ((q - 8) * d)."""
    b = np.asarray(blocks, dtype=np.uint8).reshape(-1, 18)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(-1)
    lo = (b[:, 2:] & 0x0F).astype(np.float32) - 8
    hi = (b[:, 2:] >> 4).astype(np.float32) - 8
    return (np.concatenate([lo, hi], axis=1) * d[:, None]).reshape(-1).astype(np.float32)


# --------------------------------------------------------------------- GGUF --

_GGUF_U32, _GGUF_I32, _GGUF_BOOL, _GGUF_STR, _GGUF_ARR = 4, 5, 7, 8, 9


def _gstr(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


class GGUFWriter:
    """Minimal GGUF v3 writer: scalar/array KVs and F32/F16/Q4_0 tensors."""

    def __init__(self, alignment: int = 32):
        self.kv: list[bytes] = []
        self.tensors: list[tuple[str, tuple[int, ...], int, bytes]] = []
        self.alignment = alignment

    def u32(self, key, v):
        self.kv.append(_gstr(key) + struct.pack("<II", _GGUF_U32, v))

    def boolean(self, key, v):
        self.kv.append(_gstr(key) + struct.pack("<IB", _GGUF_BOOL, 1 if v else 0))

    def i32_array(self, key, vals):
        self.kv.append(_gstr(key) + struct.pack("<IIQ", _GGUF_ARR, _GGUF_I32, len(vals))
                       + b"".join(struct.pack("<i", int(x)) for x in vals))

    def string(self, key, v):
        self.kv.append(_gstr(key) + struct.pack("<I", _GGUF_STR) + _gstr(v))

    def tensor(self, name: str, ne: tuple[int, ...], gtype: int, data: bytes):
        self.tensors.append((name, tuple(int(x) for x in ne), gtype, data))

    def tobytes(self) -> bytes:
        out = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(self.tensors), len(self.kv)))
        for kv in self.kv:
            out += kv
        offs, off = [], 0
        for name, ne, gtype, data in self.tensors:
            offs.append(off)
            off += (len(data) + self.alignment - 1) // self.alignment * self.alignment
        for (name, ne, gtype, data), o in zip(self.tensors, offs):
            out += _gstr(name) + struct.pack("<I", len(ne))
            out += b"".join(struct.pack("<Q", x) for x in ne)
            out += struct.pack("<IQ", gtype, o)
        out += b"\0" * ((-len(out)) % self.alignment)
        for name, ne, gtype, data in self.tensors:
            out += data
            out += b"\0" * ((-len(data)) % self.alignment)
        return bytes(out)


# -------------------------------------------------------------------- model --

def decoder_plan(decoder_dim=1536, rates=DEFAULT_RATES):
    """Channel progression: [(Cin, Cout, stride)] per decoder block."""
    plan, c = [], decoder_dim
    for s in rates:
        plan.append((c, c // 2, s))
        c //= 2
    return plan


def make_model(quant: str = "f16", seed: int = 0, gain: float = 0.5, decoder_dim: int = 1536,
               latent_dim: int = 64, rates=DEFAULT_RATES, convt_3d: bool = False, encoder: bool = False,
               encoder_dim: int = 128, encoder_gain: float = 0.85) -> bytes:
    """Returns the bytes of a seeded decoder GGUF.

    quant: "f16" (all tensors F16), "f32" (all F32: a model with no fp16
    rounding anywhere, for pinning the oracle's structure against the
    reference; the GPU path takes F16 / Q4_0 only) or "q4_0" (Q4_0-mixed: model.1, the 4
    transposed convs and the 12 residual pointwise convs as Q4_0, the 17
    encoder matrices likewise, everything else F16).  convt_3d writes F16
    transposed-conv weights as the 3-D [2s, Cout, Cin] tensor the F16
    checkpoints use (same memory order as the folded 2-D layout).
    encoder=True writes a full encoder of width encoder_dim (its weights
    drawn after the decoder's, so the decoder is the same either way; convs
    N(0, encoder_gain^2 / fan_in): the Snake residual units amplify, so the
    latent's scale is steep in the gain -- 0.85 gives a latent of std about
    1.3 on make_audio input, 0.7 about 0.06, 1.0 about 12);
    otherwise the encoder tensors are 32-value placeholders.
    """
    assert quant in ("f16", "q4_0", "f32")
    rng = np.random.default_rng(seed)
    w = GGUFWriter()
    w.u32("voxcpm_audio_vae_config_encoder_dim", encoder_dim)
    w.u32("voxcpm_audio_vae_config_decoder_dim", decoder_dim)
    w.u32("voxcpm_audio_vae_config_latent_dim", latent_dim)
    w.u32("voxcpm_audio_vae_config_sample_rate", 16000)
    w.i32_array("voxcpm_audio_vae_config_encoder_rates", list(reversed(rates)))
    w.i32_array("voxcpm_audio_vae_config_decoder_rates", list(rates))
    w.boolean("voxcpm_audio_vae_config_depthwise", True)

    def add(name, arr_np, q=False, ne=None):
        # arr_np is in numpy (outer..inner) order; ggml ne is the reverse.
        arr = np.ascontiguousarray(arr_np, dtype=np.float32)
        ne = ne if ne is not None else tuple(reversed(arr.shape))
        if q and quant == "q4_0":
            w.tensor(name, ne, GGML_Q4_0, quantize_q4_0(arr).tobytes())
        elif quant == "f32":
            w.tensor(name, ne, GGML_F32, arr.tobytes())
        else:
            w.tensor(name, ne, GGML_F16, arr.astype(np.float16).tobytes())

    def conv_w(shape, fan_in):
        return rng.normal(0.0, gain / np.sqrt(fan_in), shape)

    def alpha(c):
        return rng.uniform(0.5, 1.5, (1, c, 1))

    def bias(c):
        return rng.normal(0.0, 0.01, (c,))

    p = "audio_vae.decoder.model."
    add(p + "0.weight", conv_w((latent_dim, 1, 7), 7))
    add(p + "0.bias", bias(latent_dim))
    add(p + "1.weight", conv_w((decoder_dim, latent_dim), latent_dim), q=True)
    add(p + "1.bias", bias(decoder_dim))
    for bi, (cin, cout, s) in enumerate(decoder_plan(decoder_dim, rates)):
        pre = f"{p}{bi + 2}.block."
        add(pre + "0.alpha", alpha(cin))
        wt = conv_w((cin, 2 * s * cout), cin)  # numpy (Cin, 2s*Cout): ggml ne [2s*Cout, Cin]
        if convt_3d and quant == "f16":
            add(pre + "1.weight", wt, ne=(2 * s, cout, cin))
        else:
            add(pre + "1.weight", wt, q=True)
        add(pre + "1.bias", bias(cout))
        for r in range(3):
            rp = f"{pre}{r + 2}.block."
            add(rp + "0.alpha", alpha(cout))
            add(rp + "1.weight", conv_w((cout, 1, 7), 7))
            add(rp + "1.bias", bias(cout))
            add(rp + "2.alpha", alpha(cout))
            add(rp + "3.weight", conv_w((cout, cout), cout), q=True)
            add(rp + "3.bias", bias(cout))
    c_last = decoder_plan(decoder_dim, rates)[-1][1]
    nb = len(rates)
    add(f"{p}{nb + 2}.alpha", alpha(c_last))
    add(f"{p}{nb + 3}.weight", conv_w((1, c_last, 7), 7 * c_last))
    add(f"{p}{nb + 3}.bias", bias(1))

    e = "audio_vae.encoder."
    if encoder:
        def conv_e(shape, fan_in):
            return rng.normal(0.0, encoder_gain / np.sqrt(fan_in), shape)

        def conv_k(name, cout, cin, k):
            # [Cout][Cin][K] in memory: F16 as the 3-D [K, Cin, Cout] tensor,
            # Q4_0 folded to 2-D [K*Cin, Cout] (blocks need 32 | K*Cin)
            arr = conv_e((cout, cin, k), cin * k)
            if quant == "q4_0":
                add(name, arr.reshape(cout, cin * k), q=True)
            else:
                add(name, arr)

        add(e + "block.0.weight", conv_e((encoder_dim, 1, 7), 7))
        add(e + "block.0.bias", bias(encoder_dim))
        c = encoder_dim
        for b, s in enumerate(reversed(rates), start=1):
            for r in range(3):
                rp = f"{e}block.{b}.block.{r}.block."
                add(rp + "0.alpha", alpha(c))
                add(rp + "1.weight", conv_e((c, 1, 7), 7))
                add(rp + "1.bias", bias(c))
                add(rp + "2.alpha", alpha(c))
                add(rp + "3.weight", conv_e((c, c), c), q=True)
                add(rp + "3.bias", bias(c))
            add(f"{e}block.{b}.block.3.alpha", alpha(c))
            conv_k(f"{e}block.{b}.block.4.weight", 2 * c, c, 2 * s)
            add(f"{e}block.{b}.block.4.bias", bias(2 * c))
            c *= 2
        conv_k(e + "fc_mu.weight", latent_dim, c, 3)
        add(e + "fc_mu.bias", bias(latent_dim))
        return w.tobytes()
    zeros = np.zeros(32, dtype=np.float32)
    add(e + "block.0.weight", zeros)
    add(e + "block.0.bias", zeros)
    add(e + "fc_mu.weight", zeros, q=True)
    add(e + "fc_mu.bias", zeros)
    for b in range(1, len(rates) + 1):
        for r in range(3):
            for n in ["0.alpha", "1.weight", "1.bias", "2.alpha", "3.weight", "3.bias"]:
                add(f"{e}block.{b}.block.{r}.block.{n}", zeros, q=(n == "3.weight"))
        for n in ["3.alpha", "4.weight", "4.bias"]:
            add(f"{e}block.{b}.block.{n}", zeros, q=(n == "4.weight"))
    return w.tobytes()


def write_model(path: str, **kw) -> str:
    """Writes make_model(**kw) to path; returns the sha256 of the bytes."""
    data = make_model(**kw)
    with open(path, "wb") as f:
        f.write(data)
    return hashlib.sha256(data).hexdigest()


def make_audio(n: int, batch: int = 1, seed: int = 7) -> np.ndarray:
    """float32 waveforms [batch, n] at 16 kHz: a few seeded partials (80 Hz - 4 kHz,
    decaying amplitudes, random phases) plus a little noise, peak about 0.5."""
    rng = np.random.default_rng(seed)
    t = np.arange(n, dtype=np.float64) / 16000.0
    out = np.empty((batch, n), dtype=np.float32)
    for b in range(batch):
        f = rng.uniform(80.0, 4000.0, 6)
        a = rng.uniform(0.02, 0.12, 6)
        ph = rng.uniform(0.0, 2 * np.pi, 6)
        x = (a[:, None] * np.sin(2 * np.pi * f[:, None] * t[None, :] + ph[:, None])).sum(0)
        out[b] = (x + rng.normal(0.0, 0.01, n)).astype(np.float32)
    return out


def make_latents(steps: int, T: int, latent_dim: int = 64, seed: int = 1, ar: float | None = None,
                 batch: int = 1) -> np.ndarray:
    """float32 latents [steps, batch, latent_dim, T] (ggml ne=[T, latent_dim] each).

    ar=None: i.i.d. N(0, 1).  ar=rho: AR(1) along time with innovation
    sqrt(1 - rho^2), so every frame is marginally N(0, 1).
    """
    rng = np.random.default_rng(seed)
    if ar is None:
        return rng.standard_normal((steps, batch, latent_dim, T)).astype(np.float32)
    e = rng.standard_normal((steps, batch, latent_dim, T)).astype(np.float32)
    z = np.empty_like(e)
    z[..., 0] = e[..., 0]
    k = np.float32(np.sqrt(1.0 - ar * ar))
    for t in range(1, T):
        z[..., t] = np.float32(ar) * z[..., t - 1] + k * e[..., t]
    return z
