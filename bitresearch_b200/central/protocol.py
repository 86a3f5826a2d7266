"""Coordinator <-> worker messages of the centralised mode.

Message codes and JSON field names are the reference's (src/distributed/protocol.ts:3-23, :25-112), so
a client written against that protocol can talk to this coordinator. Two encodings:

* JSON text frames (protocol.ts:117-142): typed arrays travel as
  ``{"__typed_array": true, "type": "Float32Array" | "Uint32Array" | "Int32Array", "data": [...]}`` and
  come back as numpy arrays of the matching dtype.
* Binary frames for tensors (protocol.ts:145-166): ``u8 type | u32 step | u32 count`` little-endian,
  the header padded to 12 bytes, then ``count`` float32 values.

Batches are the large payload of this mode (the reference sends them as JSON number lists). Here a
``BATCH_ASSIGN`` may also travel as a binary frame of this module's own layout:
``u8 type | 3 bytes 0 | u32 step | u32 B | u32 T`` (16 bytes), then int32 inputs [B, T] and int32
targets [B, T]. ``decode`` accepts all three forms.
"""
from __future__ import annotations

import json
import struct
from enum import IntEnum

import numpy as np


class MessageType(IntEnum):
    # worker -> coordinator
    WORKER_JOIN = 0x01
    WORKER_HEARTBEAT = 0x02
    GRADIENT_PUSH = 0x03
    WORKER_LEAVE = 0x04
    WORKER_METRICS = 0x05
    # coordinator -> worker
    WELCOME = 0x10
    PARAMS_BROADCAST = 0x11
    BATCH_ASSIGN = 0x12
    TRAIN_STEP = 0x13
    STEP_COMPLETE = 0x14
    CONFIG_UPDATE = 0x15
    KICK = 0x16
    # dashboard
    STATUS_UPDATE = 0x20
    LOSS_UPDATE = 0x21


_TYPED = {"Float32Array": np.float32, "Uint32Array": np.uint32, "Int32Array": np.int32}
_NAMES = {np.dtype(np.float32): "Float32Array", np.dtype(np.uint32): "Uint32Array", np.dtype(np.int32): "Int32Array"}


def _default(v):
    if isinstance(v, np.ndarray):
        name = _NAMES.get(v.dtype)
        if name is None:
            raise TypeError(f"no typed-array encoding for dtype {v.dtype}")
        return {"__typed_array": True, "type": name, "data": v.ravel().tolist()}
    if isinstance(v, (np.integer,)):
        return int(v)
    if isinstance(v, (np.floating,)):
        return float(v)
    raise TypeError(f"cannot encode {type(v).__name__}")


def _hook(d):
    if d.get("__typed_array"):
        return np.asarray(d["data"], dtype=_TYPED.get(d.get("type"), np.int32))
    return d


def encode_json(msg: dict) -> str:
    return json.dumps(msg, default=_default)


def decode_json(text: str | bytes) -> dict:
    return json.loads(text, object_hook=_hook)


_TENSOR_HDR = struct.Struct("<BII")  # 9 bytes, data at offset 12
_TENSOR_OFF = 12


def encode_tensor_message(kind: int, step: int, data: np.ndarray) -> bytes:
    a = np.ascontiguousarray(data, dtype=np.float32).ravel()
    return _TENSOR_HDR.pack(int(kind), int(step), a.size) + b"\0" * (_TENSOR_OFF - _TENSOR_HDR.size) + a.tobytes()


def decode_tensor_message(buf: bytes) -> dict:
    kind, step, n = _TENSOR_HDR.unpack_from(buf, 0)
    data = np.frombuffer(buf, dtype="<f4", count=n, offset=_TENSOR_OFF)
    return {"type": kind, "stepId": step, "data": data}


_BATCH_HDR = struct.Struct("<B3xIII")  # 16 bytes


def encode_batch(step: int, inputs: np.ndarray, targets: np.ndarray) -> bytes:
    x = np.ascontiguousarray(inputs, dtype="<i4")
    y = np.ascontiguousarray(targets, dtype="<i4")
    if x.shape != y.shape or x.ndim != 2:
        raise ValueError("inputs and targets must both be [B, T]")
    B, T = x.shape
    return _BATCH_HDR.pack(int(MessageType.BATCH_ASSIGN), int(step), B, T) + x.tobytes() + y.tobytes()


def decode(frame: str | bytes) -> dict:
    """A JSON text frame, a tensor frame or a batch frame, as a message dict."""
    if isinstance(frame, str):
        return decode_json(frame)
    if frame[:1] in (b"{", b"["):
        return decode_json(frame)
    if frame[0] == MessageType.BATCH_ASSIGN:
        _, step, B, T = _BATCH_HDR.unpack_from(frame, 0)
        n = B * T
        x = np.frombuffer(frame, dtype="<i4", count=n, offset=_BATCH_HDR.size).reshape(B, T)
        y = np.frombuffer(frame, dtype="<i4", count=n, offset=_BATCH_HDR.size + 4 * n).reshape(B, T)
        return {"type": int(MessageType.BATCH_ASSIGN), "stepId": step, "inputIds": x, "targets": y}
    return decode_tensor_message(frame)
