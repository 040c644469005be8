"""Typed ZeroMQ queues carrying msgpack-encoded messages (reference: python/minisgl/utils/mp.py).

PUSH/PULL carry work between processes, PUB/SUB fans rank-0's raw request bytes out to the other
TP ranks without re-encoding.
"""

from __future__ import annotations

from typing import Callable, Dict, Generic, TypeVar

import msgpack
import zmq
import zmq.asyncio

T = TypeVar("T")


def _pack(obj: Dict) -> bytes:
    return msgpack.packb(obj, use_bin_type=True)


def _unpack(raw: bytes) -> Dict:
    return msgpack.unpackb(raw, raw=False)


class _Socket:
    def __init__(self, addr: str, create: bool, kind: int, asyncio: bool = False):
        self.context = zmq.asyncio.Context() if asyncio else zmq.Context()
        self.socket = self.context.socket(kind)
        if create:
            self.socket.bind(addr)
        else:
            self.socket.connect(addr)

    def stop(self) -> None:
        self.socket.close(linger=0)
        self.context.term()


class ZmqPushQueue(_Socket, Generic[T]):
    def __init__(self, addr: str, create: bool, encoder: Callable[[T], Dict]):
        super().__init__(addr, create, zmq.PUSH)
        self.encoder = encoder

    def put(self, obj: T) -> None:
        self.socket.send(_pack(self.encoder(obj)), copy=False)

    def put_raw(self, raw: bytes) -> None:
        self.socket.send(raw, copy=False)


class ZmqPullQueue(_Socket, Generic[T]):
    def __init__(self, addr: str, create: bool, decoder: Callable[[Dict], T]):
        super().__init__(addr, create, zmq.PULL)
        self.decoder = decoder

    def get(self) -> T:
        return self.decoder(_unpack(self.socket.recv()))

    def get_raw(self) -> bytes:
        return self.socket.recv()

    def decode(self, raw: bytes) -> T:
        return self.decoder(_unpack(raw))

    def empty(self) -> bool:
        return self.socket.poll(timeout=0) == 0

    def poll(self, timeout_ms: int) -> bool:
        return self.socket.poll(timeout=timeout_ms) != 0


class ZmqPubQueue(_Socket, Generic[T]):
    def __init__(self, addr: str, create: bool, encoder: Callable[[T], Dict]):
        super().__init__(addr, create, zmq.PUB)
        self.encoder = encoder

    def put(self, obj: T) -> None:
        self.socket.send(_pack(self.encoder(obj)), copy=False)

    def put_raw(self, raw: bytes) -> None:
        self.socket.send(raw, copy=False)


class ZmqSubQueue(_Socket, Generic[T]):
    def __init__(self, addr: str, create: bool, decoder: Callable[[Dict], T]):
        super().__init__(addr, create, zmq.SUB)
        self.socket.setsockopt_string(zmq.SUBSCRIBE, "")
        self.decoder = decoder

    def get(self) -> T:
        return self.decoder(_unpack(self.socket.recv()))

    def empty(self) -> bool:
        return self.socket.poll(timeout=0) == 0


class ZmqAsyncPushQueue(_Socket, Generic[T]):
    def __init__(self, addr: str, create: bool, encoder: Callable[[T], Dict]):
        super().__init__(addr, create, zmq.PUSH, asyncio=True)
        self.encoder = encoder

    async def put(self, obj: T) -> None:
        await self.socket.send(_pack(self.encoder(obj)), copy=False)


class ZmqAsyncPullQueue(_Socket, Generic[T]):
    def __init__(self, addr: str, create: bool, decoder: Callable[[Dict], T]):
        super().__init__(addr, create, zmq.PULL, asyncio=True)
        self.decoder = decoder

    async def get(self) -> T:
        return self.decoder(_unpack(await self.socket.recv()))
