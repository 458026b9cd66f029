"""Raw-TCP gateway (openmini-server/src/service/server/gateway.rs:86-627).

Frames: [u32 BE length][type u8][session id 36 B][1 unused byte][stream u8][payload]
(decoded by the C++ runtime's GatewayDecoder). Types: 1 chat, 2 image,
3 image-stream, 4 health. A chat frame's payload is the prompt text; the reply
is the generated text as [u32 BE length][bytes]; health replies "OK". A
connection limiter caps concurrent connections; oversized frames close the
connection.
"""
from __future__ import annotations

import asyncio
import struct

from .. import _native
from ..engine.request import SamplingParams

CHAT, IMAGE, IMAGE_STREAM, HEALTH = 1, 2, 3, 4


class Gateway:
    def __init__(self, aengine, tokenizer, max_connections: int = 10000, max_message: int = 16 << 20,
                 max_tokens: int = 256):
        self.aengine = aengine
        self.tok = tokenizer
        self.sem = asyncio.Semaphore(max_connections)
        self.max_message = max_message
        self.max_tokens = max_tokens
        self.stats = {"connections": 0, "requests": 0, "failed": 0, "bytes_in": 0, "bytes_out": 0}
        self.server = None

    async def _reply(self, w, data: bytes):
        w.write(struct.pack(">I", len(data)) + data)
        self.stats["bytes_out"] += 4 + len(data)
        await w.drain()

    async def handle(self, reader, writer):
        if self.sem.locked():
            writer.close()
            return
        async with self.sem:
            self.stats["connections"] += 1
            dec = _native.rt().GatewayDecoder(self.max_message)
            try:
                while True:
                    data = await reader.read(65536)
                    if not data:
                        break
                    self.stats["bytes_in"] += len(data)
                    dec.feed(data)
                    while True:
                        try:
                            fr = dec.next()
                        except ValueError:
                            self.stats["failed"] += 1
                            return
                        if fr is None:
                            break
                        typ, session, stream, payload = fr
                        self.stats["requests"] += 1
                        if typ == HEALTH:
                            await self._reply(writer, b"OK")
                        elif typ == CHAT:
                            ids = self.tok.encode(payload.decode("utf-8", errors="replace"))
                            sp = SamplingParams(temperature=0.0, max_tokens=self.max_tokens)
                            toks = []
                            async for out in self.aengine.generate(ids, sp):
                                toks = out.output_token_ids
                            await self._reply(writer, self.tok.decode(toks).encode())
                        else:
                            self.stats["failed"] += 1
                            await self._reply(writer, b"ERROR: request type not served")
            finally:
                writer.close()

    async def start(self, host="127.0.0.1", port=0):
        self.server = await asyncio.start_server(self.handle, host, port)
        return self.server.sockets[0].getsockname()[1]

    async def stop(self):
        if self.server:
            self.server.close()
            await self.server.wait_closed()
