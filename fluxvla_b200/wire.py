"""Wire formats of the policy server: msgpack (default) and protobuf.

Byte-compatible with the reference's serving codecs
(fluxvla/engines/runners/serving/serializers.py and proto/vla_service.proto)
so that existing clients talk to this server unchanged:

* a message whose first byte is 0x01 is protobuf, anything else msgpack;
* msgpack requests are ``{"endpoint": name, "data": {...}}``; predict_action
  data carries ``obs_data`` (a msgpack map of the observation) and
  ``unnorm_key``;
* in an observation map, numpy arrays travel as ``{"__ndarray__": True,
  "data": <.npy bytes>}``, JPEG-compressed uint8 HxWx3 camera frames as
  ``{"__jpeg__": True, "data": <jpeg bytes>}``, strings as strings;
* responses are ``{"action_data": <.npy bytes>, "infer_time": seconds}`` or
  ``{"error": message}``;
* protobuf messages follow the schema of vla_service.proto (package
  ``fluxvla``: Observation{images=1, arrays=2, strings=3} maps,
  PredictActionRequest{obs=1, unnorm_key=2},
  PredictActionResponse{action_data=1, infer_time=2, error=3}).  The message
  classes are built at import time from a descriptor written here (no
  generated ``_pb2`` module and no protoc needed).

The field names, numbers and tags are a format contract and therefore equal
to the reference's; the code is this library's own.
"""
from __future__ import annotations

import io
from typing import Any, Dict, Tuple

import msgpack
import numpy as np

FORMAT_MSGPACK = 0x00
FORMAT_PROTOBUF = 0x01
JPEG_QUALITY = 95
# camera keys whose uint8 frames the client side JPEG-compresses
JPEG_KEYS = frozenset({'cam_high', 'cam_left_wrist', 'cam_right_wrist',
                       'agentview_image', 'robot0_eye_in_hand_image'})


def detect_format(raw: bytes) -> int:
    return FORMAT_PROTOBUF if raw[:1] == bytes([FORMAT_PROTOBUF]) \
        else FORMAT_MSGPACK


def npy_bytes(a: np.ndarray) -> bytes:
    buf = io.BytesIO()
    np.save(buf, np.asarray(a), allow_pickle=False)
    return buf.getvalue()


def npy_load(b: bytes) -> np.ndarray:
    return np.load(io.BytesIO(b), allow_pickle=False)


def jpeg_encode(img: np.ndarray) -> bytes:
    import cv2
    ok, buf = cv2.imencode('.jpg', img, [cv2.IMWRITE_JPEG_QUALITY,
                                         JPEG_QUALITY])
    if not ok:
        raise ValueError('JPEG encoding failed')
    return buf.tobytes()


def jpeg_decode(b: bytes) -> np.ndarray:
    import cv2
    img = cv2.imdecode(np.frombuffer(b, np.uint8), cv2.IMREAD_COLOR)
    if img is None:
        raise ValueError('JPEG decoding failed')
    return img


def split_obs(obs: Dict[str, Any], compress: bool = True):
    """Observation -> (jpeg images, npy arrays, strings) byte maps."""
    images, arrays, strings = {}, {}, {}
    for k, v in obs.items():
        if (compress and k in JPEG_KEYS and isinstance(v, np.ndarray)
                and v.ndim == 3 and v.dtype == np.uint8):
            images[k] = jpeg_encode(v)
        elif isinstance(v, np.ndarray):
            arrays[k] = npy_bytes(v)
        elif isinstance(v, str):
            strings[k] = v
    return images, arrays, strings


# ---------------------------------------------------------------------------
# msgpack
# ---------------------------------------------------------------------------

def _pack_default(obj):
    if isinstance(obj, np.ndarray):
        return {'__ndarray__': True, 'data': npy_bytes(obj)}
    if isinstance(obj, np.generic):
        return obj.item()
    raise TypeError(f'cannot serialise {type(obj)}')


def _unpack_hook(d):
    if '__ndarray__' in d:
        return npy_load(d['data'])
    return d


def msg_pack(obj: Any) -> bytes:
    return msgpack.packb(obj, default=_pack_default)


def msg_unpack(raw: bytes) -> Any:
    return msgpack.unpackb(raw, object_hook=_unpack_hook)


def obs_to_msgpack(obs: Dict[str, Any], compress: bool = True) -> bytes:
    images, arrays, strings = split_obs(obs, compress)
    enc = {k: {'__jpeg__': True, 'data': v} for k, v in images.items()}
    enc.update({k: {'__ndarray__': True, 'data': v}
                for k, v in arrays.items()})
    enc.update(strings)
    return msgpack.packb(enc)


def obs_from_msgpack(raw: bytes) -> Dict[str, Any]:
    out = {}
    for k, v in msgpack.unpackb(raw, raw=False).items():
        if isinstance(v, dict) and '__jpeg__' in v:
            out[k] = jpeg_decode(v['data'])
        elif isinstance(v, dict) and '__ndarray__' in v:
            out[k] = npy_load(v['data'])
        elif isinstance(v, bytes):
            out[k] = v.decode()
        else:
            out[k] = v
    return out


# ---------------------------------------------------------------------------
# protobuf (schema of vla_service.proto, built at import)
# ---------------------------------------------------------------------------

def _build_proto():
    from google.protobuf import descriptor_pb2, descriptor_pool
    from google.protobuf import message_factory
    F = descriptor_pb2.FieldDescriptorProto
    fd = descriptor_pb2.FileDescriptorProto(
        name='fluxvla_b200_vla_service.proto', package='fluxvla',
        syntax='proto3')

    def add_field(msg, name, num, typ, label=F.LABEL_OPTIONAL, tname=None):
        f = msg.field.add(name=name, number=num, type=typ, label=label)
        if tname:
            f.type_name = tname

    obs = fd.message_type.add(name='Observation')
    for i, (name, vt) in enumerate((('images', F.TYPE_BYTES),
                                    ('arrays', F.TYPE_BYTES),
                                    ('strings', F.TYPE_STRING)), 1):
        entry_name = name.capitalize() + 'Entry'
        e = obs.nested_type.add(name=entry_name)
        e.options.map_entry = True
        add_field(e, 'key', 1, F.TYPE_STRING)
        add_field(e, 'value', 2, vt)
        add_field(obs, name, i, F.TYPE_MESSAGE, F.LABEL_REPEATED,
                  f'.fluxvla.Observation.{entry_name}')
    req = fd.message_type.add(name='PredictActionRequest')
    add_field(req, 'obs', 1, F.TYPE_MESSAGE, tname='.fluxvla.Observation')
    add_field(req, 'unnorm_key', 2, F.TYPE_STRING)
    resp = fd.message_type.add(name='PredictActionResponse')
    add_field(resp, 'action_data', 1, F.TYPE_BYTES)
    add_field(resp, 'infer_time', 2, F.TYPE_DOUBLE)
    add_field(resp, 'error', 3, F.TYPE_STRING)
    pool = descriptor_pool.DescriptorPool()
    pool.Add(fd)
    get = message_factory.GetMessageClass
    return (get(pool.FindMessageTypeByName('fluxvla.Observation')),
            get(pool.FindMessageTypeByName('fluxvla.PredictActionRequest')),
            get(pool.FindMessageTypeByName('fluxvla.PredictActionResponse')))


_PB = None


def pb():
    """(Observation, PredictActionRequest, PredictActionResponse) classes."""
    global _PB
    if _PB is None:
        _PB = _build_proto()
    return _PB


# ---------------------------------------------------------------------------
# predict_action request / response
# ---------------------------------------------------------------------------

def encode_predict_request(obs: Dict[str, Any], unnorm_key: str = '',
                           fmt: str = 'msgpack', compress: bool = True
                           ) -> bytes:
    if fmt == 'protobuf':
        Obs, Req, _ = pb()
        images, arrays, strings = split_obs(obs, compress)
        r = Req(unnorm_key=unnorm_key)
        r.obs.images.update(images)
        r.obs.arrays.update(arrays)
        r.obs.strings.update(strings)
        return bytes([FORMAT_PROTOBUF]) + r.SerializeToString()
    return msgpack.packb({'endpoint': 'predict_action',
                          'data': {'obs_data': obs_to_msgpack(obs, compress),
                                   'unnorm_key': unnorm_key}})


def decode_predict_request(raw: bytes) -> Tuple[int, Dict[str, Any], str]:
    """-> (format, observation, unnorm_key)."""
    if detect_format(raw) == FORMAT_PROTOBUF:
        _, Req, _ = pb()
        r = Req()
        r.ParseFromString(raw[1:])
        obs = {k: jpeg_decode(v) for k, v in r.obs.images.items()}
        obs.update({k: npy_load(v) for k, v in r.obs.arrays.items()})
        obs.update(dict(r.obs.strings))
        return FORMAT_PROTOBUF, obs, r.unnorm_key
    msg = msgpack.unpackb(raw, raw=False)
    data = msg.get('data', {})
    return FORMAT_MSGPACK, obs_from_msgpack(data['obs_data']), \
        data.get('unnorm_key', '')


def encode_predict_response(action_data: bytes, infer_time: float,
                            fmt: int = FORMAT_MSGPACK, error: str = ''
                            ) -> bytes:
    if fmt == FORMAT_PROTOBUF:
        _, _, Resp = pb()
        r = Resp(error=error) if error else Resp(action_data=action_data,
                                                 infer_time=infer_time)
        return bytes([FORMAT_PROTOBUF]) + r.SerializeToString()
    if error:
        return msgpack.packb({'error': error})
    return msgpack.packb({'action_data': action_data,
                          'infer_time': infer_time})


def decode_predict_response(raw: bytes) -> Dict[str, Any]:
    if detect_format(raw) == FORMAT_PROTOBUF:
        _, _, Resp = pb()
        r = Resp()
        r.ParseFromString(raw[1:])
        if r.error:
            return {'error': r.error}
        return {'action_data': r.action_data, 'infer_time': r.infer_time}
    return msgpack.unpackb(raw, raw=False)
