"""ctypes binding of the C oracle (oracle/vae_oracle.c) for the tests.

Test infrastructure only: the oracle is the checker, never the thing tested.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_SO = os.path.join(ROOT, "oracle", "liboracle.so")

MODE_EXACT, MODE_REF, MODE_GPU = 0, 1, 2

_lib = None


def lib():
    global _lib
    if _lib is None:
        src = os.path.join(ROOT, "oracle", "vae_oracle.c")
        if not os.path.exists(ORACLE_SO) or os.path.getmtime(ORACLE_SO) < os.path.getmtime(src):
            subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True)
        L = ctypes.CDLL(ORACLE_SO)
        vp, i, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
        L.vo_open.restype = vp
        L.vo_open.argtypes = [ctypes.c_char_p]
        L.vo_close.argtypes = [vp]
        L.vo_decode.restype = i64
        L.vo_decode.argtypes = [vp, vp, i, i, i, i, vp]
        L.vo_f32_to_f16.restype = ctypes.c_uint16
        L.vo_f32_to_f16.argtypes = [ctypes.c_float]
        L.vo_f16_to_f32.restype = ctypes.c_float
        L.vo_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.vo_dequant_q4_0.argtypes = [vp, i64, vp]
        L.vo_quantize_q4_0.argtypes = [vp, i64, vp]
        L.vo_snake.argtypes = [vp, vp, i, i64, vp]
        L.vo_dwconv.argtypes = [vp, vp, vp, i, i, i, i, vp]
        L.vo_pointwise.argtypes = [vp, vp, i, vp, vp, vp, i64, i, i, i, vp]
        L.vo_convt.argtypes = [vp, i, i, vp, vp, i, i, i, i, i, i, vp]
        L.vo_final.argtypes = [vp, vp, ctypes.c_float, i, i, i, i, vp]
        for f in ("vo_num_blocks", "vo_decoder_dim", "vo_latent_dim"):
            getattr(L, f).restype = i
            getattr(L, f).argtypes = [vp]
        L.vo_rate.restype = i
        L.vo_rate.argtypes = [vp, i]
        L.vo_encode.restype = i64
        L.vo_encode.argtypes = [vp, vp, i64, i, i, vp]
        for f in ("vo_encoder_dim", "vo_encoder_hop"):
            getattr(L, f).restype = i
            getattr(L, f).argtypes = [vp]
        _lib = L
    return _lib


def P(a):
    return a.ctypes.data_as(ctypes.c_void_p)


class OracleModel:
    def __init__(self, path: str):
        self.h = lib().vo_open(path.encode())
        if not self.h:
            raise RuntimeError(f"oracle failed to open {path}")
        L = lib()
        self.rates = [L.vo_rate(self.h, b) for b in range(L.vo_num_blocks(self.h))]
        self.decoder_dim = L.vo_decoder_dim(self.h)
        self.latent_dim = L.vo_latent_dim(self.h)
        self.hop = int(np.prod(self.rates))

    def close(self):
        if self.h:
            lib().vo_close(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def stage_size(self, T: int, B: int, stage: int) -> int:
        """Element count of the activation after `stage` (-1 = waveform)."""
        if stage < 0:
            return B * T * self.hop
        if stage == 0:
            return B * T * self.latent_dim
        if stage == 1:
            return B * T * self.decoder_dim
        b = (stage - 2) // 4
        n = B * T * int(np.prod(self.rates[: b + 1]))
        return n * (self.decoder_dim >> (b + 1))

    def decode(self, z: np.ndarray, mode: int = MODE_REF, stage: int = -1) -> np.ndarray:
        """z: float32 [B, latent, T] -> waveform [B, hop*T] (or a stage activation)."""
        z = np.ascontiguousarray(z, dtype=np.float32)
        B, _, T = z.shape
        out = np.zeros(self.stage_size(T, B, stage), np.float32)
        n = lib().vo_decode(self.h, P(z), T, B, mode, stage, P(out))
        assert n == out.size, (n, out.size)
        return out.reshape(B, -1) if stage < 0 else out

    def encode(self, audio: np.ndarray, mode: int = MODE_REF) -> np.ndarray:
        """audio: float32 [B, n] -> latent [B, latent, T], T = ceil(n / hop)."""
        audio = np.ascontiguousarray(audio, dtype=np.float32)
        B, n = audio.shape
        hop = lib().vo_encoder_hop(self.h)
        T = (n + hop - 1) // hop
        out = np.zeros((B, self.latent_dim, T), np.float32)
        got = lib().vo_encode(self.h, P(audio), n, B, mode, P(out))
        if got < 0:
            raise RuntimeError("the model holds no encoder")
        assert got == T, (got, T)
        return out
