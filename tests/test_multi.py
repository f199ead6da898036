"""Chunk sharding across devices and ranks (CPU: gloo ranks, stand-in models).

The synthesizer's chunks are independent (``runtime/pipeline.py:821-829``), so
multi-GPU work is a host-side split with in-order reassembly: these tests pin
the split (``shard`` / ``balance``), the reassembly across ``world_size = 2``
gloo processes (``gather_ordered``) and the one-process device pool
(``SynthPool.decode_batch``) with stand-in device models.
"""

import os
import socket
import tempfile

import numpy as np
import pytest

from rvc_cuda import multi


def test_shard_contiguous_and_complete():
    for n in (0, 1, 7, 32, 256):
        for world in (1, 2, 3, 8):
            parts = [multi.shard(n, world, r) for r in range(world)]
            assert sum(parts, []) == list(range(n))
            sizes = [len(p) for p in parts]
            assert max(sizes) - min(sizes) <= 1


def test_balance_by_cost_is_deterministic_and_even():
    costs = [1000, 300, 300, 1000, 50, 700, 400, 400, 990]
    a = multi.balance(costs, 3)
    assert a == multi.balance(list(costs), 3)
    assert sorted(sum(a, [])) == list(range(len(costs)))
    loads = [sum(costs[i] for i in b) for b in a]
    assert max(loads) - min(loads) <= max(costs)
    assert all(b == sorted(b) for b in a)
    with pytest.raises(ValueError):
        multi.shard(3, 2, 2)


def test_devices_from_env(monkeypatch):
    monkeypatch.setenv("RVC_CUDA_DEVICES", "3, 1")
    assert multi.devices_from_env() == [3, 1]
    monkeypatch.setenv("RVC_CUDA_DEVICES", "1,1")
    with pytest.raises(ValueError):
        multi.devices_from_env()
    monkeypatch.delenv("RVC_CUDA_DEVICES")
    monkeypatch.setenv("RVC_CUDA_DEVICE", "2")
    assert multi.devices_from_env() == [2]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, lengths, out_path):
    import datetime

    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        ids = multi.shard(len(lengths), world, rank, costs=lengths)
        # stand-in for a chunk's synthesis: the chunk's waveform is its index
        res = [np.full(lengths[i] * 4, i, np.float32) for i in ids]
        got = multi.gather_ordered(res, ids, len(lengths))
        if rank == 0:
            np.save(out_path, np.concatenate(got))
        else:
            assert got is None
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_reassemble_in_chunk_order():
    import torch.multiprocessing as tmp

    lengths = [100, 37, 250, 250, 8, 91, 250]
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "wave.npy")
        tmp.spawn(_rank_main, args=(2, _free_port(), lengths, out), nprocs=2, join=True)
        wave = np.load(out)
    expect = np.concatenate([np.full(L * 4, i, np.float32) for i, L in enumerate(lengths)])
    np.testing.assert_array_equal(wave, expect)


class _StandIn:
    """Device model stand-in: records which chunks it decoded."""

    def __init__(self, dev):
        self.dev, self.upp, self.sr, self.hidden, self.seen = dev, 4, 40000, 2, []

    def prep_dec(self, phone, pitch, nsff0, sid, seed=None, skip_head=None, return_length=None, noise=None):
        return {"phone": phone, "head": None, "length": None, "tag": int(sid)}

    def decode_batch(self, preps):
        self.seen += [p["tag"] for p in preps]
        return [np.full((1, 1, p["phone"].shape[1] * self.upp), p["tag"], np.float32) for p in preps]

    def close(self):
        pass


def test_synth_pool_spreads_chunks_and_keeps_order():
    pool = multi.SynthPool(None, devices=[0, 1, 2], factory=_StandIn)
    Ps = [1000, 40, 1000, 600, 1000, 20, 300]
    chunks = [(np.zeros((1, P, 8), np.float32), None, None, i, None, None) for i, P in enumerate(Ps)]
    waves = pool.infer_chunks(chunks)
    assert [int(w.reshape(-1)[0]) for w in waves] == list(range(len(Ps)))
    assert [w.shape[-1] for w in waves] == [P * 4 for P in Ps]
    assert sorted(sum((m.seen for m in pool.models), [])) == list(range(len(Ps)))
    assert all(m.seen for m in pool.models)  # every device got work
    pool.close()
