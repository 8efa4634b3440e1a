"""Regenerates the golden fixtures in tests/golden/ from the reference itself.

Run in a checkout that has the reference sources and the reference library
built from them (``make -f oracle/Makefile.ref REF=<reference checkout>``):

    python tests/golden/make_golden.py

Every fixture holds inputs drawn from fixed seeds and the outputs of the
reference's own code (oracle/_ref/liboracle_ref.so): ggml's fp16 and Q4_0
conversions, HEAD's fused Snake callback, ggml mul_mat, whole decodes
through the reference's L1 graph functions and (for Q4_0 models) through
HEAD's AudioVAE::decode, and whole encodes through AudioVAE::encode
(``python tests/golden/make_golden.py encode_f16_t6`` regenerates one case), and
the "big_decode_*" fixtures at the benchmark configurations' shapes (a 60 s
utterance, two 30 s utterances of the offline batch, 8 streams of a
256-stream streaming step).  Models are not stored: they are regenerated
bit-identically from their seeds by vxb_synth.make_model, and each fixture
records the sha256 of the model bytes it was made from.
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "voxcpm-inference_b200"))
import vxb_synth as S  # noqa: E402

# Decode fixtures: name -> (model kwargs, latent kwargs, run L2 too)
DECODE_CASES = {
    "f16_full_t6": (dict(quant="f16", seed=0), dict(steps=2, T=6, seed=1), False),
    "f16_3d_full_t6": (dict(quant="f16", seed=0, convt_3d=True), dict(steps=1, T=6, seed=1), False),
    "q4_full_t6": (dict(quant="q4_0", seed=0), dict(steps=2, T=6, seed=1), True),
    "f16_full_t1": (dict(quant="f16", seed=0), dict(steps=1, T=1, seed=3), False),
    "f16_full_t32_ar": (dict(quant="f16", seed=0), dict(steps=1, T=32, seed=4, ar=0.9), False),
    "q4_full_t32_ar": (dict(quant="q4_0", seed=0), dict(steps=1, T=32, seed=4, ar=0.9), True),
    "q4_small_rates": (dict(quant="q4_0", seed=5, decoder_dim=512, rates=(4, 5, 2, 3)),
                       dict(steps=2, T=8, seed=6), True),
    "f16_small_t3": (dict(quant="f16", seed=7, decoder_dim=256, rates=(2, 2, 2, 2)),
                     dict(steps=3, T=3, seed=8), False),
}


# Decode fixtures at the benchmark configurations' own shapes ("big_decode_*"):
# name -> (model kwargs, latent kwargs, run L2 too, stream indices kept,
# exact-arithmetic decode too).  The latents of a batched case are the whole
# batch (regenerated from the seed); `keep` names the streams whose outputs
# are stored.  "Exact" is the C oracle's fp32 decode with the same weights
# and no activation rounding (oracle/vae_oracle.c, pinned to the reference
# by the other fixtures): it measures how far the reference's Q4_0 path,
# which quantises every pointwise conv's input to Q8_0 blocks, is from the
# arithmetic it approximates at this length.
BIG_DECODE_CASES = {
    # 60 s utterance, F16 (z=[1,64,1500], AR(1) 0.9)
    "f16_c3_t1500": (dict(quant="f16", seed=0), dict(steps=1, T=1500, seed=1000, ar=0.9), False, None, False),
    # two 30 s utterances of the offline batch, Q4_0-mixed (z=[2,64,750], AR(1) 0.9)
    "q4_c5_t750x2": (dict(quant="q4_0", seed=0), dict(steps=1, T=750, seed=1000, ar=0.9, batch=2), True, None,
                     True),
    # 8 of the 256 streams of one batched streaming step, Q4_0-mixed (z=[256,64,6])
    "q4_c4_b256": (dict(quant="q4_0", seed=0), dict(steps=1, T=6, seed=1000, batch=256), True,
                   (0, 1, 37, 100, 128, 191, 254, 255), False),
}


def _oracle_exact(args):
    """One exact-arithmetic oracle decode (run in a spawned worker)."""
    path, z = args
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib as O

    return O.OracleModel(path).decode(z[None], O.MODE_EXACT)[0]


# Encode fixtures: name -> (model kwargs, audio kwargs)
ENCODE_CASES = {
    "f32_t2": (dict(quant="f32", seed=0, encoder=True), dict(n=2 * 640 - 37, batch=2, seed=11)),
    "f16_t6": (dict(quant="f16", seed=0, encoder=True), dict(n=6 * 640, batch=2, seed=7)),
    "q4_t6": (dict(quant="q4_0", seed=0, encoder=True), dict(n=6 * 640, batch=2, seed=7)),
    # non-default config: width 64, encoder rates 3,2,5,4 (hop 120; strided-conv kernels 6, 4, 10, 8)
    "q4_small_rates": (dict(quant="q4_0", seed=5, decoder_dim=512, rates=(4, 5, 2, 3), encoder=True, encoder_dim=64),
                       dict(n=9 * 120 - 31, batch=2, seed=19)),
}


def lib():
    path = os.path.join(ROOT, "oracle", "_ref", "liboracle_ref.so")
    L = ctypes.CDLL(path)
    vp, i, ll = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
    L.ref_open.restype = vp
    L.ref_open.argtypes = [ctypes.c_char_p, i]
    L.ref_close.argtypes = [vp]
    for f in ("ref_decode_l1", "ref_decode_l2"):
        getattr(L, f).argtypes = [vp, vp, i, vp]
    L.ref_encode.restype = ll
    L.ref_encode.argtypes = [vp, vp, ll, vp, ll]
    L.ref_dequant_q4_0.argtypes = [vp, ll, vp]
    L.ref_quantize_q4_0.argtypes = [vp, ll, vp]
    L.ref_fp32_to_fp16.argtypes = [ctypes.c_float]
    L.ref_fp32_to_fp16.restype = ctypes.c_ushort
    L.ref_fp16_to_fp32.argtypes = [ctypes.c_ushort]
    L.ref_fp16_to_fp32.restype = ctypes.c_float
    L.ref_snake_fused.argtypes = [vp, vp, vp, i, i, vp]
    L.ref_mul_mat.argtypes = [vp, i, i, i, vp, i, vp, i]
    return L


def P(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def fp16_fixture(L):
    rng = np.random.default_rng(11)
    specials = np.array([0.0, -0.0, 1.0, -1.0, 65504.0, 65520.0, 1e6, -1e6, 6.1e-5, 5.96e-8,
                         2.98e-8, 3e-8, 1e-10, 0.1, 1 / 3, 2049.0, 2051.0, 1.00048828125,
                         1.000732421875, np.inf, -np.inf], dtype=np.float32)
    x = np.concatenate([specials, rng.standard_normal(2000).astype(np.float32) * 10 ** rng.uniform(
        -9, 5, 2000).astype(np.float32)]).astype(np.float32)
    h = np.array([L.ref_fp32_to_fp16(float(v)) for v in x], dtype=np.uint16)
    bits = np.arange(0, 65536, 7, dtype=np.uint16)
    back = np.array([L.ref_fp16_to_fp32(int(b)) for b in bits], dtype=np.float32)
    np.savez_compressed(os.path.join(HERE, "fp16.npz"), x=x, h=h, bits=bits, back=back)


def q4_fixture(L):
    rng = np.random.default_rng(12)
    rows = [rng.standard_normal(32 * 64).astype(np.float32) * 0.05,
            np.zeros(32, np.float32),                                   # all-zero block
            np.full(32, -0.25, np.float32),                             # constant block
            np.linspace(-1, 1, 32, dtype=np.float32),                   # symmetric extremes
            (np.arange(32, dtype=np.float32) - 16) / 8.0,               # exact half steps
            rng.standard_normal(32 * 8).astype(np.float32) * 1e3]
    x = np.concatenate(rows).astype(np.float32)
    q = np.zeros((x.size // 32, 18), np.uint8)
    L.ref_quantize_q4_0(P(x), x.size, P(q))
    # random blocks with finite scales for the dequantiser
    rb = rng.integers(0, 256, (96, 18), dtype=np.uint8)
    rb[:, 0:2] = rng.standard_normal(96).astype(np.float16).view(np.uint8).reshape(-1, 2)
    deq = np.zeros(96 * 32, np.float32)
    L.ref_dequant_q4_0(P(rb), 96 * 32, P(deq))
    np.savez_compressed(os.path.join(HERE, "q4_0.npz"), x=x, q=q, blocks=rb, deq=deq)


def snake_fixture(L):
    rng = np.random.default_rng(13)
    C, T = 96, 40
    x = (rng.standard_normal((T, C)) * 3).astype(np.float32)
    x[0, :8] = [0, -0.0, 1e-30, 800.0, -1000.0, 1100.0, -4000.0, 3.14159265]
    alpha = rng.uniform(0.5, 1.5, C).astype(np.float16).astype(np.float32)
    inv = (np.float32(1.0) / (alpha + np.float32(1e-9))).astype(np.float32)
    y = np.zeros_like(x)
    L.ref_snake_fused(P(x), P(alpha), P(inv), C, T, P(y))
    np.savez_compressed(os.path.join(HERE, "snake.npz"), x=x, alpha=alpha, inv=inv, y=y)


def mulmat_fixture(L):
    rng = np.random.default_rng(14)
    out = {}
    for tag, K, M, N in (("a", 64, 96, 6), ("b", 384, 192, 40), ("c", 96, 96, 17)):
        W = (rng.standard_normal((M, K)) * (0.5 / np.sqrt(K))).astype(np.float32)
        x = rng.standard_normal((N, K)).astype(np.float32)
        for wt, raw in (("f16", W.astype(np.float16)), ("q4", S.quantize_q4_0(W))):
            y = np.zeros((N, M), np.float32)
            L.ref_mul_mat(P(np.ascontiguousarray(raw)), 1 if wt == "f16" else 2, K, M, P(x), N, P(y), 4)
            out[f"{tag}_{wt}_w"] = raw.view(np.uint8).reshape(-1) if wt == "q4" else raw
            out[f"{tag}_{wt}_y"] = y
        out[f"{tag}_x"] = x
        out[f"{tag}_shape"] = np.array([K, M, N])
    np.savez_compressed(os.path.join(HERE, "mulmat.npz"), **out)


def decode_fixture(L, name, mk, lk, do_l2):
    data = S.make_model(**mk)
    sha = hashlib.sha256(data).hexdigest()
    z = S.make_latents(**lk)
    rates = mk.get("rates", S.DEFAULT_RATES)
    hop = int(np.prod(rates))
    T = lk["T"]
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "m.gguf")
        with open(path, "wb") as f:
            f.write(data)
        h = L.ref_open(path.encode(), os.cpu_count() or 4)
        assert h, "reference failed to open the model"
        l1 = np.zeros((z.shape[0], hop * T), np.float32)
        l2 = np.zeros_like(l1)
        for s in range(z.shape[0]):
            zs = np.ascontiguousarray(z[s, 0])
            n = L.ref_decode_l1(h, P(zs), T, P(l1[s]))
            assert n == hop * T, n
            if do_l2:
                n = L.ref_decode_l2(h, P(zs), T, P(l2[s]))
                assert n == hop * T, n
        L.ref_close(h)
    arrs = dict(z=z[:, 0], l1=l1, sha=np.array(sha), model=np.array(repr(mk)),
                latents=np.array(repr(lk)))
    if do_l2:
        arrs["l2"] = l2
    np.savez_compressed(os.path.join(HERE, f"decode_{name}.npz"), **arrs)
    print(name, sha[:12], "max|y| %.3f" % np.abs(l1).max(),
          ("L1 vs L2 %.2e" % np.abs(l1 - l2).max()) if do_l2 else "")


def big_decode_fixture(L, name, mk, lk, do_l2, keep, do_exact):
    """Reference L1 (and HEAD-L2 for Q4_0) outputs of the kept streams of a
    benchmark-shaped batch.  L2 is stored as its difference from L1 in fp16
    (differences of order 1e-3, stored to ~1e-6), keeping the fixture small."""
    data = S.make_model(**mk)
    sha = hashlib.sha256(data).hexdigest()
    z = S.make_latents(**lk)[0]  # [batch, 64, T]
    keep = list(range(z.shape[0])) if keep is None else list(keep)
    T = lk["T"]
    hop = int(np.prod(mk.get("rates", S.DEFAULT_RATES)))
    l1 = np.zeros((len(keep), hop * T), np.float32)
    l2 = np.zeros_like(l1)
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "m.gguf")
        with open(path, "wb") as f:
            f.write(data)
        h = L.ref_open(path.encode(), os.cpu_count() or 4)
        assert h, "reference failed to open the model"
        for i, b in enumerate(keep):
            zs = np.ascontiguousarray(z[b])
            assert L.ref_decode_l1(h, P(zs), T, P(l1[i])) == hop * T
            if do_l2:
                assert L.ref_decode_l2(h, P(zs), T, P(l2[i])) == hop * T
        L.ref_close(h)
        exact = None
        if do_exact:
            import multiprocessing as mp

            with mp.get_context("spawn").Pool(len(keep)) as pool:
                exact = np.stack(pool.map(_oracle_exact, [(path, np.ascontiguousarray(z[b])) for b in keep]))
    arrs = dict(keep=np.array(keep), z=z[keep], l1=l1, sha=np.array(sha), model=np.array(repr(mk)),
                latents=np.array(repr(lk)))
    if do_l2:
        arrs["l2_minus_l1"] = (l2 - l1).astype(np.float16)
    if exact is not None:
        arrs["exact_minus_l1"] = (exact - l1).astype(np.float16)
    np.savez_compressed(os.path.join(HERE, f"big_decode_{name}.npz"), **arrs)
    print("big", name, sha[:12], "max|y| %.3f" % np.abs(l1).max(),
          ("L1 vs L2 %.2e" % np.abs(l1 - l2).max()) if do_l2 else "",
          ("L1 vs exact %.2e" % np.abs(l1 - exact).max()) if exact is not None else "")


def encode_fixture(L, name, mk, ak):
    """The reference's own AudioVAE::encode on each waveform of a seeded batch."""
    data = S.make_model(**mk)
    sha = hashlib.sha256(data).hexdigest()
    audio = S.make_audio(**ak)
    B, n = audio.shape
    hop = int(np.prod(mk.get("rates", S.DEFAULT_RATES)))
    T = (n + hop - 1) // hop
    lat = np.zeros((B, 64, T), np.float32)
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "m.gguf")
        with open(path, "wb") as f:
            f.write(data)
        h = L.ref_open(path.encode(), os.cpu_count() or 4)
        assert h, "reference failed to open the model"
        for b in range(B):
            got = L.ref_encode(h, P(np.ascontiguousarray(audio[b])), n, P(lat[b]), lat[b].size)
            assert got == 64 * T, got
        L.ref_close(h)
    np.savez_compressed(os.path.join(HERE, f"encode_{name}.npz"), audio=audio, latent=lat, sha=np.array(sha),
                        model=np.array(repr(mk)), audio_kw=np.array(repr(ak)))
    print("encode", name, sha[:12], "max|latent| %.3f" % np.abs(lat).max())


def main():
    L = lib()
    only = sys.argv[1:]
    if not only:
        fp16_fixture(L)
        q4_fixture(L)
        snake_fixture(L)
        mulmat_fixture(L)
    for name, (mk, lk, do_l2) in DECODE_CASES.items():
        if not only or name in only:
            decode_fixture(L, name, mk, lk, do_l2)
    for name, (mk, lk, do_l2, keep, do_exact) in BIG_DECODE_CASES.items():
        if not only or "big_decode_" + name in only:
            big_decode_fixture(L, name, mk, lk, do_l2, keep, do_exact)
    for name, (mk, ak) in ENCODE_CASES.items():
        if not only or "encode_" + name in only:
            encode_fixture(L, name, mk, ak)


if __name__ == "__main__":
    main()
