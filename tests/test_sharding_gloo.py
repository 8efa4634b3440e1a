"""Host-side multi-rank logic of bench.py, on CPU with world_size-2 gloo ranks.

The decode path has no data-path collective: each rank takes its own share of
the streams (strong scaling) or its own streams (weak scaling), seeded by rank;
the only collective is the max over ranks of the timed region.
"""
import os
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import bench

    dist.init_process_group("gloo", rank=rank, world_size=world)
    ws, r, local = bench.dist_env()
    out = {}
    for w in ("c2", "c4", "c5q"):
        quant, streams, T, emit, scaling, ar = bench.WORKLOADS[w]
        per = streams if scaling == "weak" else max(1, streams // ws)
        z = bench.build_inputs(w, r, per, 2) if T <= 750 else None
        out[w] = (per, None if z is None else z[0, :, 0, :4].copy())
    t = torch.tensor([float(rank + 1) * 10.0])
    dist.all_reduce(t, op=dist.ReduceOp.MAX)  # the bench's max-over-ranks of the timed region
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, ws, out, float(t.item())))


@pytest.mark.timeout(300)
def test_two_gloo_ranks_partition_streams_without_exchange():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        rank, ws, out, tmax = q.get(timeout=240)
        res[rank] = (ws, out, tmax)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][0] == res[1][0] == 2
    # strong scaling: 256 streams -> 128 per rank; weak: 1 stream per rank
    assert res[0][1]["c4"][0] == res[1][1]["c4"][0] == 128
    assert res[0][1]["c2"][0] == 1 and res[0][1]["c5q"][0] == 32
    # each rank's latents differ (seeded by rank): no rank duplicates another's work
    assert not np.array_equal(res[0][1]["c2"][1], res[1][1]["c2"][1])
    # every rank reports the max of the per-rank timings
    assert res[0][2] == res[1][2] == 20.0


def _chunk_worker(rank, world, port, model, T, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    sys.path.insert(0, os.path.join(ROOT, "voxcpm-inference_b200"))
    import bench
    import chunking
    import oracle_lib as O

    dist.init_process_group("gloo", rank=rank, world_size=world)
    ws, r, _ = bench.dist_env()
    w = chunking.split(T, ws, bench.C3_HALO)[r]
    z = bench.S.make_latents(1, T, seed=1000, ar=0.9)[0, 0]  # the utterance every rank shares
    m = O.OracleModel(model)
    y = m.decode(z[None, :, w.start:w.end], O.MODE_EXACT)[0]
    kept = y[w.halo * 640:]
    dist.barrier()
    dist.destroy_process_group()
    q.put((r, w.keep, kept))


@pytest.mark.timeout(300)
def test_two_gloo_ranks_time_chunks_reproduce_one_utterance():
    """c3 over ranks: each rank decodes its time window (20-frame halo) of the
    shared utterance with no exchange; the kept samples, placed side by side,
    equal the one-shot decode (oracle, small-width model, CPU)."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    sys.path.insert(0, os.path.join(ROOT, "voxcpm-inference_b200"))
    import oracle_lib as O
    import vxb_synth as S
    from models import model_path

    model, _ = model_path(quant="f16", seed=3, decoder_dim=128)
    T = 50
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + ((os.getpid() + 7) % 1000)
    procs = [ctx.Process(target=_chunk_worker, args=(r, 2, port, model, T, q)) for r in range(2)]
    for p in procs:
        p.start()
    parts = sorted(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    z = S.make_latents(1, T, seed=1000, ar=0.9)[0, 0]
    full = O.OracleModel(model).decode(z[None], O.MODE_EXACT)[0]
    got = np.concatenate([k for _, _, k in parts])
    assert parts[1][1] == 25 and got.size == full.size
    assert np.array_equal(got, full)


def _enc_chunk_worker(rank, world, port, model, T, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    sys.path.insert(0, os.path.join(ROOT, "voxcpm-inference_b200"))
    import bench
    import chunking
    import oracle_lib as O

    dist.init_process_group("gloo", rank=rank, world_size=world)
    ws, r, _ = bench.dist_env()
    halo = chunking.min_encoder_halo((2, 5, 8, 8))
    w = chunking.split(T, ws, halo)[r]
    a = bench.S.make_audio(T * 640, 1, seed=2000)  # the waveform every rank shares
    m = O.OracleModel(model)
    z = m.encode(a[:, w.start * 640:w.end * 640], O.MODE_EXACT)[0]
    dist.barrier()
    dist.destroy_process_group()
    q.put((r, w.keep, z[:, w.halo:]))


@pytest.mark.timeout(300)
def test_two_gloo_ranks_encode_time_chunks_of_one_waveform():
    """The encoder over ranks: each rank encodes its time window (15-frame
    halo) of one shared waveform with no exchange; the kept latent frames,
    placed side by side, equal the one-shot encode (oracle, narrow encoder, CPU)."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    sys.path.insert(0, os.path.join(ROOT, "voxcpm-inference_b200"))
    import oracle_lib as O
    import vxb_synth as S
    from models import model_path

    model, _ = model_path(quant="f16", seed=4, decoder_dim=128, encoder=True, encoder_dim=32)
    T = 40
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + ((os.getpid() + 13) % 1000)
    procs = [ctx.Process(target=_enc_chunk_worker, args=(r, 2, port, model, T, q)) for r in range(2)]
    for p in procs:
        p.start()
    parts = sorted(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    a = S.make_audio(T * 640, 1, seed=2000)
    full = O.OracleModel(model).encode(a, O.MODE_EXACT)[0]
    got = np.concatenate([k for _, _, k in parts], axis=1)
    assert parts[1][1] == 20 and got.shape == full.shape
    assert np.array_equal(got, full)
