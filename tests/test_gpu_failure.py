"""Failure detection on the GPU without a GPU fault.

Every device wait of the decode kernels is bounded: a wait that runs out
records an error code in the context's status word and the kernel returns,
so the host reports VXB_ERR_DEVICE_STATUS instead of hanging, and the
context keeps working.  The probe entry point makes one such wait run out
(an mbarrier nothing arrives on, a 1 ms limit); the test checks the
reported status and that an ordinary decode on the same context afterwards
still matches the oracle.
"""
import time

import numpy as np
import pytest

import oracle_lib as O
import vxb_synth as S
from models import model_path

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_expired_device_wait_is_reported_and_context_survives():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import vxb

    path, _ = model_path(quant="q4_0", seed=0)
    d = vxb.Decoder(0)
    d.load_gguf(path)
    d.prepare()
    z = S.make_latents(1, 6, seed=51)[:, 0]
    before = d.decode(z)
    t0 = time.perf_counter()
    d.wait_probe(1000)
    with pytest.raises(vxb.VxbError) as e:
        d.sync(5000)
    waited = time.perf_counter() - t0
    assert e.value.code == vxb.ERR_DEVICE_STATUS
    assert waited < 2.0, f"the 1 ms device wait took {waited:.3f} s to be reported"
    after = d.decode(z)  # clears the status word; must decode normally
    d.sync()
    assert np.array_equal(before, after)
    ref = O.OracleModel(path).decode(z, O.MODE_GPU)
    assert float(np.abs(after - ref).max()) <= 5e-4
    d.close()


def test_probe_rejects_bad_limits():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import vxb

    d = vxb.Decoder(0)
    for bad in (0, -5, 2000001):
        with pytest.raises(vxb.VxbError) as e:
            d.wait_probe(bad)
        assert e.value.code == vxb.ERR_INVALID_ARGUMENT
    d.close()
