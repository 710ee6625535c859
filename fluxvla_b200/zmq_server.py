"""ZMQ policy server in front of the B200 engine (or a replica pool).

Mirrors the reference serving entry point
(fluxvla/engines/runners/serving/zmq_server.py:40-284): a REP socket with
named endpoints (``ping``, ``kill``, ``predict_action``, ``reset``,
``get_status``), msgpack or protobuf requests told apart by their first byte
(``fluxvla_b200.wire``), and a reply for every request — an exception inside
a handler becomes ``{"error": message}`` (protobuf: the ``error`` field), so
one malformed request never takes the server down (zmq_server.py:101-141).

``create_server(policy, transform=...)`` wires a policy object with the
reference's ``predict_action(images, lang_tokens, states, img_masks,
lang_masks, noise)`` contract into the ``predict_action`` endpoint:
observation -> ``transform`` (the reference passes its dataset transform
pipeline here) -> keyword arguments -> actions, returned as ``.npy`` bytes
with the inference time.
"""
from __future__ import annotations

import threading
import time
from dataclasses import dataclass
from typing import Any, Callable, Dict, Optional

import numpy as np
import torch

from . import wire


@dataclass
class Endpoint:
    handler: Callable
    requires_input: bool = True


class PolicyServer:
    """REP-socket event loop with endpoint routing (see module docstring)."""

    def __init__(self, host: str = '*', port: int = 5555,
                 poll_ms: int = 500):
        import zmq
        self._zmq = zmq
        self.running = True
        self.poll_ms = poll_ms
        self.context = zmq.Context()
        self.socket = self.context.socket(zmq.REP)
        if port == 0:
            self.port = self.socket.bind_to_random_port(f'tcp://{host}')
        else:
            self.socket.bind(f'tcp://{host}:{port}')
            self.port = port
        self.endpoints: Dict[str, Endpoint] = {}
        self.register_endpoint('ping', lambda: {'status': 'ok',
                                                'message': 'Server is running'},
                               requires_input=False)
        self.register_endpoint('kill', self._kill, requires_input=False)

    def register_endpoint(self, name: str, handler: Callable,
                          requires_input: bool = True):
        self.endpoints[name] = Endpoint(handler, requires_input)

    def _kill(self):
        self.running = False
        return {'status': 'ok', 'message': 'Server shutting down'}

    def handle(self, message: bytes) -> bytes:
        """One request -> one reply (never raises)."""
        if wire.detect_format(message) == wire.FORMAT_PROTOBUF:
            return self._handle_protobuf(message)
        try:
            req = wire.msg_unpack(message)
            if not isinstance(req, dict):
                raise ValueError('request is not a map')
            name = req.get('endpoint', 'predict_action')
            if name not in self.endpoints:
                raise ValueError(f'Unknown endpoint: {name}')
            ep = self.endpoints[name]
            result = ep.handler(**req.get('data', {})) if ep.requires_input \
                else ep.handler()
            return wire.msg_pack(result)
        except Exception as e:  # noqa: BLE001 - every error becomes a reply
            return wire.msg_pack({'error': f'{type(e).__name__}: {e}'})

    def _handle_protobuf(self, message: bytes) -> bytes:
        fmt = wire.FORMAT_PROTOBUF
        try:
            _, obs, unnorm_key = wire.decode_predict_request(message)
            ep = self.endpoints.get('predict_action')
            if ep is None:
                return wire.encode_predict_response(
                    b'', 0.0, fmt, error='predict_action endpoint not '
                                         'registered')
            res = ep.handler(obs_data=None, unnorm_key=unnorm_key,
                             _obs_dict=obs)
            return wire.encode_predict_response(
                res.get('action_data', b''), res.get('infer_time', 0.0), fmt,
                error=res.get('error', ''))
        except Exception as e:  # noqa: BLE001
            return wire.encode_predict_response(
                b'', 0.0, fmt, error=f'{type(e).__name__}: {e}')

    def run(self):
        """Serve until the ``kill`` endpoint or close() stops the loop."""
        zmq = self._zmq
        poller = zmq.Poller()
        poller.register(self.socket, zmq.POLLIN)
        while self.running:
            if self.socket not in dict(poller.poll(timeout=self.poll_ms)):
                continue
            self.socket.send(self.handle(self.socket.recv()))
        self.socket.setsockopt(zmq.LINGER, 0)
        self.socket.close()
        self.context.term()

    def close(self):
        self.running = False


def obs_to_inputs(obs: Dict[str, Any]) -> Dict[str, Any]:
    """Default observation -> predict_action keyword arguments: ``images``
    (uint8 [V,H,W,3]), ``lang_tokens`` [1,L], ``states`` [1,S] and optional
    ``img_masks``, ``lang_masks``, ``noise`` arrays, as torch tensors."""
    out = {}
    for k in ('images', 'lang_tokens', 'states', 'img_masks', 'lang_masks',
              'noise'):
        if k in obs and obs[k] is not None:
            out[k] = torch.from_numpy(np.ascontiguousarray(obs[k]))
    for k in ('images', 'lang_tokens', 'states'):
        if k not in out:
            raise KeyError(f"observation has no '{k}'")
    if out['images'].dtype != torch.uint8:
        raise TypeError('images must be uint8 [views, H, W, 3]')
    return out


def create_server(policy, transform: Optional[Callable] = None,
                  host: str = '*', port: int = 5555) -> PolicyServer:
    """PolicyServer whose predict_action endpoint runs ``policy``."""
    transform = transform or obs_to_inputs
    lock = threading.Lock()
    stats = {'n': 0, 'infer': 0.0, 'start': time.time()}

    def predict_action(obs_data: bytes = None, unnorm_key: str = '',
                       _obs_dict: dict = None) -> dict:
        obs = _obs_dict if _obs_dict is not None else \
            wire.obs_from_msgpack(obs_data)
        kw = transform(obs)
        t0 = time.perf_counter()
        with lock:   # one request at a time per model (zmq_server.py:251)
            actions = policy.predict_action(**kw)
        dt = time.perf_counter() - t0
        a = actions.detach().float().cpu().numpy() if torch.is_tensor(
            actions) else np.asarray(actions, np.float32)
        with lock:
            stats['n'] += 1
            stats['infer'] += dt
        return {'action_data': wire.npy_bytes(a), 'infer_time': dt}

    def get_status() -> dict:
        n = stats['n']
        return {'status': 'ready', 'uptime_s': time.time() - stats['start'],
                'total_requests': n,
                'avg_infer_time': stats['infer'] / n if n else 0.0}

    server = PolicyServer(host=host, port=port)
    server.register_endpoint('predict_action', predict_action)
    server.register_endpoint('reset', lambda: {'status': 'ok'},
                             requires_input=False)
    server.register_endpoint('get_status', get_status, requires_input=False)
    return server
