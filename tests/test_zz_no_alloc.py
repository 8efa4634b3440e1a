"""The allocation-free decode entry point (vxb_decode_static).

Some callers cannot allocate device memory once they run -- a real-time
audio thread, where cudaMalloc may stall and synchronise the device, or a
host whose device memory is all owned by another allocator.  For them
vxb_decode_static keeps every intermediate activation in a fixed array
compiled into the library.  This test calls it through the C ABI twice in a
row (the second call reuses the array the first one left behind) and checks
each output against the planned decode (vxb_decode_device) on the same
latent, at the array's exact-fit size (8 frames) and with a batch of two;
and that the second call leaves the device's free memory unchanged.  It
lives in its own file so that pytest collects it last.
"""
import numpy as np
import pytest

import vxb_synth as S
from models import model_path

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.mark.parametrize("B,T", [(1, 6), (1, 8), (2, 4)])
@pytest.mark.parametrize("quant", ["q4_0", "f16"])
def test_static_decode_matches_planned_decode(quant, B, T):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import vxb

    path, _ = model_path(quant=quant, seed=0)
    d = vxb.Decoder(0)
    d.load_gguf(path)
    d.prepare()
    d.build_plan(B, T)
    stream = torch.cuda.current_stream()
    # every device buffer of the test exists before the calls, so a change of
    # the free device memory across a call can only come from the call itself
    zs = [torch.from_numpy(S.make_latents(1, T, seed=seed, batch=B)[0]).cuda() for seed in (31, 32)]
    want = torch.empty((B, d.hop * T), dtype=torch.float32, device="cuda")
    got = torch.empty_like(want)
    for call, z in enumerate(zs):
        got.fill_(float("nan"))
        d.decode_device(z, want, stream)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        d.decode_static(z, got, B, T, stream)
        d.sync()
        torch.cuda.synchronize()
        free_after = torch.cuda.mem_get_info()[0]
        err = float((got - want).abs().max())
        assert np.isfinite(err) and err <= 1e-5, f"call {call}: static vs planned decode max|d| {err:.3e}"
        if call == 1:  # the first call may load kernels; the second must allocate nothing
            assert free_after >= free_before, f"vxb_decode_static took {free_before - free_after} bytes"
    d.close()


def test_static_decode_rejects_oversized_shapes():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import vxb

    path, _ = model_path(quant="q4_0", seed=0)
    d = vxb.Decoder(0)
    d.load_gguf(path)
    d.prepare()
    z = torch.zeros((2, 64, 6), device="cuda")
    out = torch.empty((2, 640 * 6), device="cuda")
    with pytest.raises(vxb.VxbError) as e:
        d.decode_static(z, out, 2, 6)  # 12 frames > the 8-frame limit
    assert e.value.code == vxb.ERR_INVALID_ARGUMENT
    d.close()
