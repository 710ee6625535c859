"""Data-parallel serving of independent PI0 / PI0.5 requests.

One engine replica per GPU (one process per GPU), a round-robin dispatcher
that shards a batch of independent requests over the replicas, and the
batch-size sweep of the serving benchmark (aggregate chunks/s and
per-request p50 / p99 latency).  This is the work-distribution part of the
reference's serving runner (fluxvla/serving/zmq_server.py:185-284 receives a
request, calls `vla.predict_action` and replies; fluxvla/serving/serve.py:
40-138 starts one server); the ZMQ / msgpack / protobuf transport is not
part of this library.

A batch-1 request has no profitable intra-request split, so requests are the
unit of parallelism: request i of a batch goes to replica i % world, each
replica serves its share back to back through its own CUDA graph, and a
request's latency runs from the batch's release until its actions are on the
host (queueing behind the replica's earlier requests included).
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence

import torch


@dataclass
class Request:
    idx: int
    images: torch.Tensor   # uint8 [views, H, W, 3]
    tokens: torch.Tensor   # int64 [1, n_tok]
    state: torch.Tensor    # f32 [1, state_dim]
    noise: torch.Tensor    # f32 [1, n_actions, action_dim]


def make_request(cfg, n_tok: int, idx: int, seed_base: int = 0,
                 pin: bool = True) -> Request:
    """Synthetic request `idx`, seeded with seed_base + idx (uint8 images
    U[0,255], token ids U[0,vocab), state and noise ~N(0,1))."""
    g = torch.Generator().manual_seed(seed_base + idx)
    r = Request(
        idx=idx,
        images=torch.randint(0, 256, (cfg.n_views, cfg.image_size,
                                      cfg.image_size, 3), generator=g,
                             dtype=torch.uint8),
        tokens=torch.randint(0, cfg.vocab, (1, n_tok), generator=g),
        state=torch.randn(1, cfg.state_dim, generator=g),
        noise=torch.randn(1, cfg.n_actions, cfg.action_dim, generator=g))
    if pin and torch.cuda.is_available():
        r.images, r.tokens = r.images.pin_memory(), r.tokens.pin_memory()
        r.state, r.noise = r.state.pin_memory(), r.noise.pin_memory()
    return r


def shard(n_requests: int, rank: int, world: int) -> List[int]:
    """Round-robin: request i is served by replica i % world."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f'bad rank {rank} / world {world}')
    return list(range(rank, n_requests, world))


def percentile(values: Sequence[float], q: float) -> float:
    """Nearest-rank percentile (q in (0, 100])."""
    if not values:
        raise ValueError('no values')
    xs = sorted(values)
    k = max(1, math.ceil(q / 100.0 * len(xs)))
    return float(xs[k - 1])


class ReplicaServer:
    """Serves requests back to back on one GPU through an engine whose
    `predict_action(images, lang_tokens, states, noise=...)` returns the
    actions on the host (e.g. `PI0EngineB200`)."""

    def __init__(self, engine):
        self.engine = engine

    def serve(self, requests: Sequence[Request], t_release: float,
              clock: Callable[[], float] = time.perf_counter):
        """Returns [(idx, latency_ms, actions)] in service order."""
        out = []
        for r in requests:
            a = self.engine.predict_action(r.images, r.tokens, r.state,
                                           noise=r.noise)
            out.append((r.idx, (clock() - t_release) * 1e3, a))
        return out


def sweep(server: ReplicaServer, request_of: Callable[[int], Request],
          batch_sizes: Sequence[int], rank: int, world: int,
          barrier: Callable[[], None],
          gather: Callable[[object], List[object]],
          repeats: int = 1) -> List[Dict]:
    """For each batch size b: release b requests at once, each replica
    serves its round-robin share, and the latencies of all replicas are
    gathered.  Returns (on every rank) per batch size: aggregate chunks/s
    (b / the slowest replica's wall time), p50 / p99 request latency, the
    requests per replica and the number of requests measured."""
    results = []
    for b in batch_sizes:
        mine = [request_of(i) for i in shard(b, rank, world)]
        lat: List[float] = []
        walls: List[float] = []
        for _ in range(repeats):
            barrier()
            t0 = time.perf_counter()
            served = server.serve(mine, t0)
            wall = time.perf_counter() - t0
            gathered = gather(([l for _, l, _ in served], wall))
            for ls, wl in gathered:
                lat.extend(ls)
                walls.append(wl)
        per_rep = len(walls) // repeats
        wall_max = [max(walls[k * per_rep:(k + 1) * per_rep])
                    for k in range(repeats)]
        results.append({
            'batch': b,
            'chunks_per_s': b * repeats / sum(wall_max),
            'p50_ms': percentile(lat, 50),
            'p99_ms': percentile(lat, 99),
            'requests_per_gpu': math.ceil(b / world),
            'requests_measured': len(lat),
        })
    return results


def dist_helpers(world: int, device: Optional[torch.device] = None):
    """barrier / gather callables over the default process group (NCCL or
    gloo), or trivial ones for a single process."""
    if world <= 1:
        return (lambda: None), (lambda obj: [obj])
    import torch.distributed as dist

    def barrier():
        dist.barrier()

    def gather(obj):
        objs = [None] * world
        dist.all_gather_object(objs, obj)
        return objs
    return barrier, gather
