"""Serving transport and failure handling, on CPU with stand-in policies:
the msgpack / protobuf wire formats (round trips and the reference's byte
layout), the ZMQ policy server over a real socket (per-request error
replies), and the replica pool's handling of a replica that raises, exits
or hangs (host processes; no GPU is involved)."""
import os
import threading
import time

import msgpack
import numpy as np
import pytest
import torch

from fluxvla_b200 import wire
from fluxvla_b200.serving import ReplicaPool
from fluxvla_b200.zmq_server import PolicyServer, create_server


def _obs(seed=0):
    rng = np.random.default_rng(seed)
    return {'images': rng.integers(0, 256, (2, 8, 8, 3), dtype=np.uint8),
            'lang_tokens': rng.integers(0, 100, (1, 5)),
            'states': rng.standard_normal((1, 4)).astype(np.float32),
            'task_description': 'pick up the bowl'}


@pytest.mark.parametrize('fmt', ['msgpack', 'protobuf'])
def test_request_round_trip(fmt):
    obs = _obs()
    raw = wire.encode_predict_request(obs, 'libero', fmt=fmt)
    assert (raw[0] == 1) == (fmt == 'protobuf')
    f, got, key = wire.decode_predict_request(raw)
    assert key == 'libero'
    for k in ('images', 'lang_tokens', 'states'):
        assert np.array_equal(got[k], obs[k]) and got[k].dtype == obs[k].dtype
    assert got['task_description'] == obs['task_description']


def test_jpeg_camera_keys_compressed():
    img = np.full((16, 16, 3), 128, np.uint8)
    f, got, _ = wire.decode_predict_request(
        wire.encode_predict_request({'agentview_image': img}))
    assert got['agentview_image'].shape == (16, 16, 3)
    assert np.abs(got['agentview_image'].astype(int) - 128).max() <= 2


def test_msgpack_layout_is_the_reference_layout():
    """The byte layout the reference's clients produce: endpoint/data map,
    obs_data a msgpack map with {'__ndarray__': True, 'data': npy}."""
    a = np.arange(6, dtype=np.float32).reshape(2, 3)
    raw = wire.encode_predict_request({'states': a}, 'k')
    outer = msgpack.unpackb(raw, raw=False)
    assert outer['endpoint'] == 'predict_action'
    inner = msgpack.unpackb(outer['data']['obs_data'], raw=False)
    assert inner['states']['__ndarray__'] is True
    assert np.array_equal(np.load(__import__('io').BytesIO(
        inner['states']['data'])), a)


def test_protobuf_field_numbers():
    """Hand-decoded tags: PredictActionResponse action_data=1 (bytes),
    infer_time=2 (double), error=3 (string)."""
    raw = wire.encode_predict_response(b'xy', 0.5, wire.FORMAT_PROTOBUF)
    body = raw[1:]
    assert body[:4] == bytes([0x0a, 2]) + b'xy'
    assert body[4] == 0x11  # field 2, wire type 1 (64-bit)
    err = wire.encode_predict_response(b'', 0, wire.FORMAT_PROTOBUF, 'bad')
    assert err[1:] == bytes([0x1a, 3]) + b'bad'
    assert wire.decode_predict_response(err) == {'error': 'bad'}


class EchoPolicy:
    """Stand-in policy: actions = states broadcast; raises on bad input."""

    def predict_action(self, images, lang_tokens, states, **kw):
        if states.shape[-1] != 4:
            raise ValueError('state must have 4 entries')
        return states.float()[:, None, :].expand(1, 3, 4).clone()


def _client(port, payload, timeout_ms=10000):
    import zmq
    ctx = zmq.Context()
    s = ctx.socket(zmq.REQ)
    s.setsockopt(zmq.RCVTIMEO, timeout_ms)
    s.setsockopt(zmq.LINGER, 0)
    s.connect(f'tcp://127.0.0.1:{port}')
    s.send(payload)
    out = s.recv()
    s.close()
    ctx.term()
    return out


def test_zmq_server_endpoints_and_errors():
    server = create_server(EchoPolicy(), host='127.0.0.1', port=0)
    server.poll_ms = 20
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    try:
        port = server.port
        assert msgpack.unpackb(_client(port, msgpack.packb(
            {'endpoint': 'ping'})))['status'] == 'ok'
        for fmt in ('msgpack', 'protobuf'):
            obs = _obs(1)
            rep = wire.decode_predict_response(_client(
                port, wire.encode_predict_request(obs, fmt=fmt)))
            a = wire.npy_load(rep['action_data'])
            assert a.shape == (1, 3, 4)
            assert np.allclose(a[0, 0], obs['states'][0])
            # malformed request: an error reply, and the server survives
            bad = dict(obs, states=np.zeros((1, 5), np.float32))
            rep = wire.decode_predict_response(_client(
                port, wire.encode_predict_request(bad, fmt=fmt)))
            assert 'state must have 4' in rep['error']
        rep = msgpack.unpackb(_client(port, msgpack.packb(
            {'endpoint': 'nope'})))
        assert 'Unknown endpoint' in rep['error']
        rep = msgpack.unpackb(_client(port, b'\xc1garbage'))
        assert 'error' in rep
        st = msgpack.unpackb(_client(port, msgpack.packb(
            {'endpoint': 'get_status'})))
        assert st['total_requests'] == 2
        _client(port, msgpack.packb({'endpoint': 'kill'}))
        th.join(timeout=5)
        assert not th.is_alive()
    finally:
        server.close()


# ---------------------------------------------------------------------------
# replica pool (worker processes)
# ---------------------------------------------------------------------------

class ScriptedPolicy:
    """Replica stand-in whose behaviour per request is in the request:
    'ok' returns [rank, x], 'raise' raises, 'exit' kills the process (only
    on the replica named by 'on'), 'hang' sleeps far past the timeout."""

    def __init__(self, rank):
        self.rank = rank

    def predict_action(self, x, mode='ok', on=-1):
        if mode == 'raise':
            raise ValueError(f'malformed request {x}')
        if mode == 'exit' and self.rank == on:
            os._exit(3)
        if mode == 'hang' and self.rank == on:
            time.sleep(60)
        return torch.tensor([float(self.rank), float(x)])


def make_scripted(rank):
    return ScriptedPolicy(rank)


def test_pool_per_request_errors_and_dead_replica_reroute():
    pool = ReplicaPool(make_scripted, 2, timeout_s=2.0, mp_context='spawn')
    try:
        reqs = [dict(x=i) for i in range(6)]
        reqs[2] = dict(x=2, mode='raise')
        res = pool.serve(reqs)
        assert [r.status for r in res] == ['ok'] * 2 + ['error'] + ['ok'] * 3
        assert 'malformed request 2' in res[2].error
        assert {r.replica for r in res} == {0, 1}
        # replica 1 exits on its first request: that request and the rest
        # of its share are rerouted to replica 0
        reqs = [dict(x=i, mode='exit', on=1) for i in range(4)]
        res = pool.serve(reqs)
        assert all(r.status == 'ok' for r in res), [r.error for r in res]
        assert all(r.replica == 0 for r in res)
        assert [float(r.actions[1]) for r in res] == [0., 1., 2., 3.]
        assert pool.alive == [True, False]
    finally:
        pool.close()


def test_pool_hung_replica_times_out_and_reroutes():
    pool = ReplicaPool(make_scripted, 2, timeout_s=1.0, mp_context='spawn')
    try:
        t0 = time.monotonic()
        res = pool.serve([dict(x=i, mode='hang', on=0) for i in range(4)])
        assert time.monotonic() - t0 < 20
        assert all(r.status == 'ok' and r.replica == 1 for r in res)
        assert pool.alive == [False, True]
        # with every replica gone, requests fail with a status, not a hang
        pool._kill(1)
        res = pool.serve([dict(x=0)])
        assert res[0].status == 'error' and 'no live replica' in res[0].error
    finally:
        pool.close()
