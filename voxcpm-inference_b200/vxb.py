"""Python binding of libvxb (include/vxb.h) over ctypes.

The decode path is the CUDA library; there is no CPU fallback.  Loading the
library or opening a context without a B200 raises VxbError.

Device buffers are passed as raw pointers (ints) or torch CUDA tensors; torch
is only used for device memory and streams.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "lib", "libvxb.so")

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_OUT_OF_MEMORY = 2
ERR_FILE_NOT_FOUND = 3
ERR_INVALID_FORMAT = 4
ERR_BACKEND = 5
ERR_NOT_READY = 6
ERR_TIMEOUT = 7
ERR_DEVICE_STATUS = 8
ERR_MISSING_TENSOR = 9

TYPE_F32, TYPE_F16, TYPE_Q4_0 = 0, 1, 2

# Every exported symbol of include/vxb.h with its ctypes signature.
_vp, _i, _i64, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
SIGNATURES = {
    "vxb_last_error": (ctypes.c_char_p, []),
    "vxb_open": (_i, [_i, ctypes.POINTER(_vp)]),
    "vxb_close": (_i, [_vp]),
    "vxb_set_config": (_i, [_vp, _i, _i, ctypes.POINTER(_i), _i]),
    "vxb_upload_tensor": (_i, [_vp, ctypes.c_char_p, _i, ctypes.POINTER(_i64), _i, _vp, _sz]),
    "vxb_load_gguf": (_i, [_vp, ctypes.c_char_p]),
    "vxb_prepare": (_i, [_vp]),
    "vxb_set_q4_fp16_cache": (_i, [_vp, _i]),
    "vxb_build_plan": (_i, [_vp, _i, _i, _i]),
    "vxb_hop": (_i, [_vp]),
    "vxb_get_config": (_i, [_vp, ctypes.POINTER(_i), ctypes.POINTER(_i), ctypes.POINTER(_i), _i, ctypes.POINTER(_i)]),
    "vxb_decode": (_i, [_vp, _vp, _vp]),
    "vxb_decode_device": (_i, [_vp, _vp, _vp, _vp]),
    "vxb_sync": (_i, [_vp, _i]),
    "vxb_debug_stage": (_i, [_vp, _i, _vp, _sz]),
    "vxb_debug_wait_probe": (_i, [_vp, _i, _vp]),
    "vxb_decode_static": (_i, [_vp, _vp, _vp, _i, _i, _vp]),
    "vxb_plan_num_ops": (_i, [_vp]),
    "vxb_plan_op_info": (_i, [_vp, _i, ctypes.c_char_p, _i, ctypes.c_char_p, _i, ctypes.POINTER(ctypes.c_double),
                              ctypes.POINTER(ctypes.c_double)]),
    "vxb_time_ops": (_i, [_vp, _i, _vp, _sz, ctypes.POINTER(ctypes.c_float)]),
    "vxb_q4_0_dequant": (_i, [_vp, _i64, _vp, _vp]),
    "vxb_snake": (_i, [_vp, _vp, _i, _i64, _vp, _vp]),
    "vxb_pointwise": (_i, [_vp, _i, _i, _i, _vp, _i64, _vp, _vp, _vp, _i, _vp, _vp]),
    "vxb_convt": (_i, [_vp, _i, _i, _i, _i, _vp, _i, _i, _vp, _vp, _vp]),
    "vxb_residual_unit": (_i, [_vp, _i, _i, _i, _vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp, _vp]),
    "vxb_stream_open": (_i, [_vp, _i, ctypes.POINTER(_vp)]),
    "vxb_stream_push": (_i, [_vp, _vp, _vp]),
    "vxb_stream_push_device": (_i, [_vp, _vp, _vp, _vp]),
    "vxb_stream_reset": (_i, [_vp]),
    "vxb_stream_close": (_i, [_vp]),
    "vxb_set_encoder_config": (_i, [_vp, _i, ctypes.POINTER(_i), _i]),
    "vxb_encoder_hop": (_i, [_vp]),
    "vxb_get_encoder_config": (_i, [_vp, ctypes.POINTER(_i), ctypes.POINTER(_i), _i, ctypes.POINTER(_i)]),
    "vxb_build_encode_plan": (_i, [_vp, _i, _i]),
    "vxb_encode": (_i, [_vp, _vp, _vp]),
    "vxb_encode_device": (_i, [_vp, _vp, _vp, _vp]),
    "vxb_encode_num_ops": (_i, [_vp]),
    "vxb_encode_op_info": (_i, [_vp, _i, ctypes.c_char_p, _i, ctypes.c_char_p, _i, ctypes.POINTER(ctypes.c_double),
                                ctypes.POINTER(ctypes.c_double)]),
    "vxb_encode_time_ops": (_i, [_vp, _i, _vp, _sz, ctypes.POINTER(ctypes.c_float)]),
}


class VxbError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"vxb error {code}: {msg}")
        self.code = code


_lib = None


def lib():
    """Loads libvxb.so (fails loudly when it is missing)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise VxbError(ERR_BACKEND, f"{LIB_PATH} not built (run voxcpm-inference_b200/build.py)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc: int):
    if rc != OK:
        raise VxbError(rc, lib().vxb_last_error().decode())


def ptr(x) -> int | None:
    """Device/host pointer of a torch tensor, numpy array or int (None -> NULL)."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    return x.data_ptr()


CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy: the legacy default stream, named explicitly


def _stream(stream) -> int:
    """CUDA stream handle for a launch: the given torch stream / raw handle, or
    torch's current stream.  Handle 0 (torch's legacy default stream) is passed
    as cudaStreamLegacy, because NULL means "the context's own stream" in the
    C ABI."""
    if stream is None:
        import torch

        stream = torch.cuda.current_stream()
    h = stream if isinstance(stream, int) else stream.cuda_stream
    return h if h else CUDA_STREAM_LEGACY


class Decoder:
    """One decoder context on one GPU (mirrors VoxCPMBackend + AudioVAE)."""

    def __init__(self, device: int = 0):
        h = ctypes.c_void_p()
        check(lib().vxb_open(device, ctypes.byref(h)))
        self.h = h
        self.device = device
        self.B = self.T = 0

    def close(self):
        if self.h:
            lib().vxb_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load_gguf(self, path: str):
        check(lib().vxb_load_gguf(self.h, path.encode()))

    def set_config(self, latent_dim: int, decoder_dim: int, rates):
        arr = (ctypes.c_int * len(rates))(*rates)
        check(lib().vxb_set_config(self.h, latent_dim, decoder_dim, arr, len(rates)))

    def upload(self, name: str, gtype: int, ne, data: bytes):
        ne_arr = (ctypes.c_int64 * len(ne))(*ne)
        buf = ctypes.create_string_buffer(data, len(data))
        check(lib().vxb_upload_tensor(self.h, name.encode(), gtype, ne_arr, len(ne), buf, len(data)))

    def prepare(self):
        check(lib().vxb_prepare(self.h))

    def set_q4_fp16_cache(self, enable: bool):
        """Opt-in fp16 copies of Q4_0 conv weights for the plans' GEMMs (next prepare)."""
        check(lib().vxb_set_q4_fp16_cache(self.h, 1 if enable else 0))

    def build_plan(self, batch: int, T: int, graph: bool = True):
        check(lib().vxb_build_plan(self.h, batch, T, 1 if graph else 0))
        self.B, self.T = batch, T

    @property
    def hop(self) -> int:
        return lib().vxb_hop(self.h)

    def config(self) -> dict:
        """{latent_dim, decoder_dim, rates} of the loaded decoder."""
        lat, dec, n = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        rates = (ctypes.c_int * 8)()
        check(lib().vxb_get_config(self.h, ctypes.byref(lat), ctypes.byref(dec), rates, 8, ctypes.byref(n)))
        return {"latent_dim": lat.value, "decoder_dim": dec.value, "rates": list(rates[: n.value])}

    def decode(self, z: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        """Host latents [B, latent, T] -> host waveform [B, hop*T] (copies included)."""
        z = np.ascontiguousarray(z, dtype=np.float32)
        if z.ndim == 2:
            z = z[None]
        B, _, T = z.shape
        if (B, T) != (self.B, self.T):
            self.build_plan(B, T)
        if out is None:
            out = np.empty((B, self.hop * T), np.float32)
        check(lib().vxb_decode(self.h, ptr(z), ptr(out)))
        return out

    def decode_chunked(self, z: np.ndarray, chunk: int, halo: int | None = None) -> np.ndarray:
        """Host latents [latent, T] (or [1, latent, T]) -> waveform [hop*T],
        decoded in windows of at most chunk + halo frames (activation memory
        bounded by the window, not the utterance).  Equal to decode(z): every
        window starts `halo` frames (>= the receptive field) before the frames
        it keeps, and is zero-padded at its end to one plan size -- the decoder
        is causal, so the padding never reaches a kept sample."""
        import chunking

        z = np.asarray(z, dtype=np.float32)
        if z.ndim == 3:
            if z.shape[0] != 1:
                raise ValueError("decode_chunked decodes one utterance")
            z = z[0]
        L, T = z.shape
        if halo is None:
            halo = chunking.min_halo(self.config()["rates"])
        W = min(T, chunk + halo)
        win = np.zeros((1, L, W), np.float32)
        out = np.empty(T * self.hop, np.float32)
        hop = self.hop
        for c in chunking.chunks_of(T, chunk, halo):
            win[0, :, : c.frames] = z[:, c.start:c.end]
            win[0, :, c.frames:] = 0.0
            y = self.decode(win)
            out[c.keep * hop:c.end * hop] = y[0, c.halo * hop:(c.halo + c.end - c.keep) * hop]
        return out

    def decode_host_ptrs(self, z_ptr: int, out_ptr: int):
        check(lib().vxb_decode(self.h, z_ptr, out_ptr))

    def decode_device(self, z_dev, out_dev, stream=None):
        check(lib().vxb_decode_device(self.h, ptr(z_dev), ptr(out_dev), _stream(stream)))

    def decode_static(self, z_dev, out_dev, batch: int, T: int, stream=None):
        """Allocation-free decode (device buffers, static scratch, batch*T <= 8)."""
        check(lib().vxb_decode_static(self.h, ptr(z_dev), ptr(out_dev), batch, T, _stream(stream)))

    def wait_probe(self, limit_us: int, stream=None):
        """Runs a device wait that nothing satisfies, bounded at limit_us: the
        next sync() raises VxbError(ERR_DEVICE_STATUS)."""
        check(lib().vxb_debug_wait_probe(self.h, limit_us, _stream(stream) if stream is not None else None))

    def sync(self, timeout_ms: int = 60000):
        check(lib().vxb_sync(self.h, timeout_ms))

    def ops(self) -> list[dict]:
        """[{name, kernel, flops, bytes}] for every launch of the current plan."""
        out = []
        for i in range(lib().vxb_plan_num_ops(self.h)):
            name, kern = ctypes.create_string_buffer(64), ctypes.create_string_buffer(64)
            fl, by = ctypes.c_double(), ctypes.c_double()
            check(lib().vxb_plan_op_info(self.h, i, name, 64, kern, 64, ctypes.byref(fl), ctypes.byref(by)))
            out.append({"name": name.value.decode(), "kernel": kern.value.decode(), "flops": fl.value,
                        "bytes": by.value})
        return out

    def time_ops(self, reps: int = 10, flush=None, flush_bytes: int = 0) -> list[float]:
        n = lib().vxb_plan_num_ops(self.h)
        ms = (ctypes.c_float * n)()
        check(lib().vxb_time_ops(self.h, reps, ptr(flush), flush_bytes, ms))
        return list(ms)

    # ---------------------------------------------------------- encoder --

    @property
    def encoder_hop(self) -> int:
        return lib().vxb_encoder_hop(self.h)

    def encoder_config(self) -> dict:
        """{encoder_dim, rates} of the loaded encoder (0 and [] without one)."""
        dim, n = ctypes.c_int(), ctypes.c_int()
        rates = (ctypes.c_int * 8)()
        check(lib().vxb_get_encoder_config(self.h, ctypes.byref(dim), rates, 8, ctypes.byref(n)))
        return {"encoder_dim": dim.value, "rates": list(rates[: n.value])}

    def build_encode_plan(self, batch: int, T: int):
        check(lib().vxb_build_encode_plan(self.h, batch, T))
        self.eB, self.eT = batch, T

    def encode(self, audio: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        """Host waveforms [B, n] (16 kHz; zero-padded here to a hop multiple, as
        the reference's preprocess does) -> host latents [B, latent, T], T = ceil(n / hop)."""
        audio = np.asarray(audio, dtype=np.float32)
        if audio.ndim == 1:
            audio = audio[None]
        B, n = audio.shape
        hop = self.encoder_hop
        if hop <= 0:
            raise VxbError(ERR_NOT_READY, "no encoder config")
        T = (n + hop - 1) // hop
        if n != T * hop:
            audio = np.concatenate([audio, np.zeros((B, T * hop - n), np.float32)], axis=1)
        audio = np.ascontiguousarray(audio)
        if (B, T) != (getattr(self, "eB", None), getattr(self, "eT", None)):
            self.build_encode_plan(B, T)
        if out is None:
            out = np.empty((B, self.config()["latent_dim"], T), np.float32)
        check(lib().vxb_encode(self.h, ptr(audio), ptr(out)))
        return out

    def encode_chunked(self, audio: np.ndarray, chunk: int, halo: int | None = None) -> np.ndarray:
        """One waveform [n] (or [1, n]) -> latent [latent, T], encoded in windows
        of at most chunk + halo frames (activation memory bounded by the window,
        not the waveform).  Equal to encode(): the encoder is causal, every window
        starts `halo` frames (>= chunking.min_encoder_halo(rates), 15 for
        VoxCPM) before the frames it keeps, and is zero-padded at its end to one
        plan size, which never reaches a kept frame."""
        import chunking

        a = np.asarray(audio, dtype=np.float32)
        if a.ndim == 2:
            if a.shape[0] != 1:
                raise ValueError("encode_chunked encodes one waveform")
            a = a[0]
        hop = self.encoder_hop
        if hop <= 0:
            raise VxbError(ERR_NOT_READY, "no encoder config")
        need = chunking.min_encoder_halo(self.encoder_config()["rates"])
        halo = need if halo is None else int(halo)
        if halo < need:
            raise ValueError(f"halo {halo} < the encoder's receptive field ({need} frames)")
        return Decoder._encode_windows(self, a, chunk, halo)

    def _encode_windows(self, a: np.ndarray, chunk: int, halo: int) -> np.ndarray:
        """encode_chunked's window loop, without the halo check."""
        import chunking

        hop = self.encoder_hop
        T = (a.size + hop - 1) // hop
        a = np.concatenate([a, np.zeros(T * hop - a.size, np.float32)])
        W = min(T, chunk + halo)
        win = np.zeros((1, W * hop), np.float32)
        out = None
        for c in chunking.chunks_of(T, chunk, halo):
            win[0, : c.frames * hop] = a[c.start * hop:c.end * hop]
            win[0, c.frames * hop:] = 0.0
            z = self.encode(win)[0]
            if out is None:
                out = np.empty((z.shape[0], T), np.float32)
            out[:, c.keep:c.end] = z[:, c.halo:c.halo + c.end - c.keep]
        return out

    def encode_host_ptrs(self, audio_ptr: int, latent_ptr: int):
        check(lib().vxb_encode(self.h, audio_ptr, latent_ptr))

    def encode_device(self, audio_dev, latent_dev, stream=None):
        check(lib().vxb_encode_device(self.h, ptr(audio_dev), ptr(latent_dev), _stream(stream)))

    def encode_ops(self) -> list[dict]:
        """[{name, kernel, flops, bytes}] for every launch of the encode plan."""
        out = []
        for i in range(lib().vxb_encode_num_ops(self.h)):
            name, kern = ctypes.create_string_buffer(64), ctypes.create_string_buffer(64)
            fl, by = ctypes.c_double(), ctypes.c_double()
            check(lib().vxb_encode_op_info(self.h, i, name, 64, kern, 64, ctypes.byref(fl), ctypes.byref(by)))
            out.append({"name": name.value.decode(), "kernel": kern.value.decode(), "flops": fl.value,
                        "bytes": by.value})
        return out

    def encode_time_ops(self, reps: int = 10, flush=None, flush_bytes: int = 0) -> list[float]:
        n = lib().vxb_encode_num_ops(self.h)
        ms = (ctypes.c_float * n)()
        check(lib().vxb_encode_time_ops(self.h, reps, ptr(flush), flush_bytes, ms))
        return list(ms)

    def debug_stage(self, stage: int, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        check(lib().vxb_debug_stage(self.h, stage, ptr(out), n))
        return out


class LayerStateStream:
    """One latent stream decoded n frames per push with every causal layer's
    left context carried from push to push on the device (vxb_stream_*): the
    pushes emit exactly the continuous decode of the stream.  Not the
    reference's streaming behaviour (every window decoded alone)."""

    def __init__(self, decoder: "Decoder", n_frames: int):
        h = ctypes.c_void_p()
        check(lib().vxb_stream_open(decoder.h, n_frames, ctypes.byref(h)))
        self.h, self.n, self.d = h, n_frames, decoder
        self.latent_dim = decoder.config()["latent_dim"]

    def push(self, z_new: np.ndarray) -> np.ndarray:
        """z_new [latent, n] (or [1, latent, n]) -> waveform [n * hop]."""
        z = np.ascontiguousarray(np.asarray(z_new, dtype=np.float32).reshape(self.latent_dim, self.n))
        out = np.empty(self.n * self.d.hop, np.float32)
        check(lib().vxb_stream_push(self.h, ptr(z), ptr(out)))
        return out

    def push_device(self, z_dev, out_dev, stream=None):
        check(lib().vxb_stream_push_device(self.h, ptr(z_dev), ptr(out_dev), _stream(stream)))

    def reset(self):
        check(lib().vxb_stream_reset(self.h))

    def close(self):
        if self.h:
            lib().vxb_stream_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class StreamingDecoder:
    """Opt-in stateful streaming over a Decoder.

    The reference decodes every streaming window on its own, with zero left
    context (vae_decode_mock.cpp:1337-1347), so consecutive windows do not
    join up; this mode is NOT output-equivalent to it.  It keeps each
    stream's last `halo` latent frames and decodes [history + new frames]
    with the sequence start only at the true start of the stream: the
    decoder is causal with a left receptive field of
    chunking.receptive_field_frames(rates) frames (18.49 for VoxCPM), so with
    halo >= chunking.min_halo(rates) every emitted sample equals the
    continuous decode of the whole stream so far -- the quality check this
    mode is tested against.  Each step decodes halo + n frames to emit n
    (the history is re-decoded, not cached as activations); the window
    length settles at halo + n once the stream is halo frames old.  Streams
    of a batch advance together.
    """

    def __init__(self, decoder: "Decoder", batch: int = 1, halo: int | None = None):
        import chunking

        self.d = decoder
        cfg = decoder.config()
        self.latent_dim = cfg["latent_dim"]
        need = chunking.min_halo(cfg["rates"])
        self.halo = need if halo is None else int(halo)
        if self.halo < need:
            raise ValueError(f"halo {self.halo} < the decoder's receptive field ({need} frames)")
        self.batch = batch
        self.reset()

    def reset(self):
        """Forgets every stream's history (the next push starts new streams)."""
        self.history = np.zeros((self.batch, self.latent_dim, 0), np.float32)

    def push(self, z_new: np.ndarray) -> np.ndarray:
        """New latent frames [batch, latent, n] (or [latent, n] for one stream)
        -> their waveform [batch, n * hop]."""
        z_new = np.asarray(z_new, dtype=np.float32)
        if z_new.ndim == 2:
            z_new = z_new[None]
        if z_new.shape[:2] != (self.batch, self.latent_dim) or z_new.shape[2] < 1:
            raise ValueError(f"expected [{self.batch}, {self.latent_dim}, n >= 1] frames, got {list(z_new.shape)}")
        win = np.ascontiguousarray(np.concatenate([self.history, z_new], axis=2))
        n, hop = z_new.shape[2], self.d.hop
        y = self.d.decode(win)
        self.history = win[:, :, -self.halo:].copy()
        return y[:, -n * hop:].copy()


# ---------------------------------------------------------- single kernels --

def q4_0_dequant(blocks, n: int, out, stream=None):
    check(lib().vxb_q4_0_dequant(ptr(blocks), n, ptr(out), _stream(stream)))


def snake(x, alpha, C: int, N: int, y, stream=None):
    check(lib().vxb_snake(ptr(x), ptr(alpha), C, N, ptr(y), _stream(stream)))


def pointwise(w, w_type: int, K: int, M: int, x16, N: int, bias, y, res=None, snake_alpha=None,
              out_f16: bool = False, stream=None):
    check(lib().vxb_pointwise(ptr(w), w_type, K, M, ptr(x16), N, ptr(bias), ptr(res), ptr(snake_alpha),
                              1 if out_f16 else 0, ptr(y), _stream(stream)))


def convt(w, w_type: int, Cin: int, Cout: int, s: int, x16, B: int, T: int, bias, y, stream=None):
    check(lib().vxb_convt(ptr(w), w_type, Cin, Cout, s, ptr(x16), B, T, ptr(bias), ptr(y), _stream(stream)))


def residual_unit(w, w_type: int, C: int, d: int, x, batch: int, T: int, a1, dw, db, a2, pb, y, out_alpha=None,
                  out_f16: bool = False, stream=None):
    check(lib().vxb_residual_unit(ptr(w), w_type, C, d, ptr(x), batch, T, ptr(a1), ptr(dw), ptr(db), ptr(a2), ptr(pb),
                                  ptr(out_alpha), 1 if out_f16 else 0, ptr(y), _stream(stream)))
