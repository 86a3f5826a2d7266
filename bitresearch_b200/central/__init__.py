"""Centralised mode: a coordinator hands out batches and collects loss statistics from workers that
each train their own replica (the reference's server/index.ts + src/distributed/protocol.ts)."""
from .coordinator import Coordinator, CoordinatorConfig, CoordinatorThread
from .protocol import MessageType, decode, encode_batch, encode_json, encode_tensor_message
from .worker import CentralWorker

__all__ = ["Coordinator", "CoordinatorConfig", "CoordinatorThread", "CentralWorker", "MessageType", "decode",
           "encode_batch", "encode_json", "encode_tensor_message"]
