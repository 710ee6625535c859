"""Host logic of the data-parallel serving runner (fluxvla_b200.serving):
round-robin sharding, percentiles, and the batch sweep across two gloo
ranks on CPU with a stand-in engine (no GPU)."""
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fluxvla_b200.config import PI0Config
from fluxvla_b200.serving import (ReplicaServer, make_request, percentile,
                                  shard, sweep, dist_helpers)


@pytest.mark.parametrize('n', [0, 1, 4, 5, 16, 64])
@pytest.mark.parametrize('world', [1, 2, 4, 8])
def test_shard_round_robin(n, world):
    parts = [shard(n, r, world) for r in range(world)]
    flat = sorted(i for p in parts for i in p)
    assert flat == list(range(n))
    sizes = [len(p) for p in parts]
    assert max(sizes) - min(sizes) <= 1
    for r, p in enumerate(parts):
        assert all(i % world == r for i in p)


def test_shard_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard(4, 2, 2)


def test_percentile_nearest_rank():
    xs = list(range(1, 101))
    assert percentile(xs, 50) == 50
    assert percentile(xs, 99) == 99
    assert percentile(xs, 100) == 100
    assert percentile([7.0], 99) == 7.0
    with pytest.raises(ValueError):
        percentile([], 50)


def test_requests_are_seeded_per_index():
    cfg = PI0Config(vis_layers=1, llm_layers=1, exp_layers=1, vocab=4096)
    a, b, a2 = (make_request(cfg, 48, i, seed_base=7, pin=False) for i in (0, 1, 0))
    assert torch.equal(a.images, a2.images) and torch.equal(a.noise, a2.noise)
    assert not torch.equal(a.images, b.images)
    assert a.images.dtype == torch.uint8 and a.tokens.shape == (1, 48)


class _FakeEngine:
    """predict_action that takes a fixed time and tags its output."""

    def __init__(self, delay_s):
        self.delay_s = delay_s
        self.served = []

    def predict_action(self, images, tokens, state, noise=None):
        time.sleep(self.delay_s)
        self.served.append(int(tokens[0, 0]))
        return torch.zeros(1, 50, 32)


def _rank_main(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    cfg = PI0Config(vis_layers=1, llm_layers=1, exp_layers=1, vocab=4096)
    eng = _FakeEngine(0.005)

    def request_of(i):
        r = make_request(cfg, 4, i, pin=False)
        r.tokens[0, 0] = i  # lets the engine record which request it served
        return r
    barrier, gather = dist_helpers(world)
    res = sweep(ReplicaServer(eng), request_of, [1, 4, 5], rank, world,
                barrier, gather)
    served = gather(eng.served)
    if rank == 0:
        torch.save({'res': res, 'served': served}, out_path)
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def test_sweep_two_gloo_ranks(tmp_path):
    out = str(tmp_path / 'sweep.pt')
    mp.spawn(_rank_main, args=(2, _free_port(), out), nprocs=2, join=True)
    d = torch.load(out)
    res, served = d['res'], d['served']
    # every request of every batch served exactly once, on replica i % 2
    assert sorted(served[0] + served[1]) == sorted([0] + list(range(4)) + list(range(5)))
    assert all(i % 2 == 0 for i in served[0]) and all(i % 2 == 1 for i in served[1])
    for r, b in zip(res, [1, 4, 5]):
        assert r['batch'] == b and r['requests_measured'] == b
        assert r['requests_per_gpu'] == (b + 1) // 2
        assert 0 < r['p50_ms'] <= r['p99_ms']
        # the slowest replica serves ceil(b/2) requests of >= 5 ms each
        assert r['chunks_per_s'] <= b / (r['requests_per_gpu'] * 0.005) + 1e-6
    # queueing: the last request of a replica waits for the earlier ones
    assert res[2]['p99_ms'] >= 3 * 5.0
