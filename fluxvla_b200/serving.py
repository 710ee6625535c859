"""Data-parallel serving of independent PI0 / PI0.5 requests.

One engine replica per GPU (one process per GPU), a round-robin dispatcher
that shards a batch of independent requests over the replicas, and the
batch-size sweep of the serving benchmark (aggregate chunks/s and
per-request p50 / p99 latency).  This is the work-distribution part of the
reference's serving runner (fluxvla/serving/zmq_server.py:185-284 receives a
request, calls `vla.predict_action` and replies; fluxvla/serving/serve.py:
40-138 starts one server).  The transport in front of it (ZMQ REP socket,
msgpack / protobuf codecs) is fluxvla_b200/zmq_server.py and
fluxvla_b200/wire.py; ``ReplicaPool`` below runs one worker process per GPU
with per-request error statuses, a host-side progress timeout and rerouting
of a dead replica's requests.

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


# ---------------------------------------------------------------------------
# Replica pool with failure handling
# ---------------------------------------------------------------------------

def _replica_main(make_policy, rank, inq, outq):
    """Worker process: build one replica, then serve (req_id, kwargs)
    messages until None; every request gets a reply, an exception becomes
    an 'error' reply (the reference catches per request,
    zmq_server.py:101-141)."""
    try:
        policy = make_policy(rank)
    except Exception as e:  # noqa: BLE001
        outq.put((None, rank, 'dead', f'replica {rank} failed to start: {e}'))
        return
    outq.put((None, rank, 'ready', None))
    while True:
        msg = inq.get()
        if msg is None:
            return
        rid, kw = msg
        try:
            a = policy.predict_action(**kw)
            outq.put((rid, rank, 'ok', a))
        except Exception as e:  # noqa: BLE001
            outq.put((rid, rank, 'error', f'{type(e).__name__}: {e}'))


@dataclass
class Result:
    idx: int
    status: str            # 'ok' | 'error'
    actions: Optional[object] = None
    error: str = ''
    replica: int = -1
    latency_ms: float = 0.0
    attempts: int = 1


class ReplicaPool:
    """One worker process per replica (per GPU) behind a host dispatcher.

    ``make_policy(rank)`` runs inside worker ``rank`` and returns an object
    with ``predict_action(**kwargs)`` (an engine on ``cuda:rank``).  A batch
    of requests is spread round-robin over the live replicas.  A replica
    that exits, or makes no progress for ``timeout_s`` while it has work, is
    marked dead (and terminated); its unfinished requests are rerouted to
    the live replicas (at most ``max_attempts`` tries per request).  A
    request whose handler raises gets an 'error' result and is not retried:
    the error is the request's, not the replica's."""

    def __init__(self, make_policy: Callable, n_replicas: int,
                 timeout_s: float = 10.0, max_attempts: int = 2,
                 start_timeout_s: float = 300.0, mp_context: str = 'spawn'):
        import multiprocessing as mp
        ctx = mp.get_context(mp_context)
        self.timeout_s = timeout_s
        self.max_attempts = max_attempts
        self.outq = ctx.Queue()
        self.inqs = [ctx.Queue() for _ in range(n_replicas)]
        self.procs = [ctx.Process(target=_replica_main,
                                  args=(make_policy, r, self.inqs[r],
                                        self.outq), daemon=True)
                      for r in range(n_replicas)]
        for p in self.procs:
            p.start()
        self.alive = [False] * n_replicas
        deadline = time.monotonic() + start_timeout_s
        pending = n_replicas
        import queue
        while pending and time.monotonic() < deadline:
            try:
                _, rank, st, _ = self.outq.get(timeout=0.2)
            except queue.Empty:
                if not any(p.is_alive() for p in self.procs):
                    break
                continue
            self.alive[rank] = st == 'ready'
            pending -= 1
        if not any(self.alive):
            self.close()
            raise RuntimeError('no replica started')

    def _kill(self, r):
        self.alive[r] = False
        p = self.procs[r]
        if p.is_alive():
            p.terminate()
            p.join(timeout=5)

    def serve(self, requests: Sequence[Dict], clock=time.monotonic
              ) -> List[Result]:
        """Serve a batch (request i = keyword arguments of predict_action);
        returns one Result per request, in request order."""
        import queue
        t0 = clock()
        results: Dict[int, Result] = {}
        attempts = {i: 0 for i in range(len(requests))}
        outstanding: Dict[int, List[int]] = {r: [] for r in
                                             range(len(self.procs))}
        progress = {r: t0 for r in range(len(self.procs))}

        def dispatch(i):
            live = [r for r in range(len(self.procs)) if self.alive[r]]
            if not live or attempts[i] >= self.max_attempts:
                why = 'no live replica' if not live else \
                    f'gave up after {attempts[i]} attempts'
                results[i] = Result(i, 'error', error=why,
                                    attempts=attempts[i])
                return
            r = min(live, key=lambda x: (len(outstanding[x]), x))
            if not outstanding[r]:
                progress[r] = clock()
            attempts[i] += 1
            outstanding[r].append(i)
            self.inqs[r].put((i, requests[i]))

        live0 = [r for r in range(len(self.procs)) if self.alive[r]]
        for i in range(len(requests)):
            if live0:
                r = live0[i % len(live0)]
                if not outstanding[r]:
                    progress[r] = clock()
                attempts[i] += 1
                outstanding[r].append(i)
                self.inqs[r].put((i, requests[i]))
            else:
                dispatch(i)
        while len(results) < len(requests):
            try:
                rid, r, st, payload = self.outq.get(timeout=0.05)
            except queue.Empty:
                rid = None
            if rid is not None and rid not in results and \
                    rid in outstanding.get(r, []):
                outstanding[r].remove(rid)
                progress[r] = clock()
                lat = (clock() - t0) * 1e3
                results[rid] = Result(
                    rid, 'ok' if st == 'ok' else 'error',
                    actions=payload if st == 'ok' else None,
                    error='' if st == 'ok' else str(payload), replica=r,
                    latency_ms=lat, attempts=attempts[rid])
            now = clock()
            for r in range(len(self.procs)):
                if not self.alive[r]:
                    continue
                dead = not self.procs[r].is_alive()
                hung = outstanding[r] and now - progress[r] > self.timeout_s
                if dead or hung:
                    self._kill(r)
                    moved, outstanding[r] = outstanding[r], []
                    for i in moved:
                        if i not in results:
                            dispatch(i)
        return [results[i] for i in range(len(requests))]

    def close(self):
        for r, q in enumerate(self.inqs):
            if self.procs[r].is_alive():
                q.put(None)
        for p in self.procs:
            p.join(timeout=5)
            if p.is_alive():
                p.terminate()
