"""OpenAI-compatible HTTP frontend and interactive shell
(reference: python/minisgl/server/api_server.py:53-452).

Endpoints: ``POST /generate`` (SSE text stream), ``GET|POST /v1`` (health),
``POST /v1/chat/completions`` and ``POST /v1/completions`` (OpenAI shapes, streaming or not),
``GET /v1/models``. A request gets a uid, goes to the tokenizer as a ``TokenizeMsg``, and its
``UserReply`` chunks come back through one listener task that wakes the waiting handler. A client
disconnect aborts the request in the scheduler.
"""

from __future__ import annotations

import asyncio
import json
import time
from contextlib import asynccontextmanager
from dataclasses import dataclass, field
from typing import AsyncIterator, Callable, Dict, List, Literal

from fastapi import FastAPI, Request
from fastapi.responses import StreamingResponse
from pydantic import BaseModel, Field

from minisgl.core import UNBOUNDED_MAX_TOKENS, SamplingParams
from minisgl.env import ENV
from minisgl.message import AbortMsg, BaseFrontendMsg, BaseTokenizerMsg, BatchFrontendMsg, TokenizeMsg, UserReply
from minisgl.utils import init_logger

logger = init_logger(__name__)


class GenerateRequest(BaseModel):
    prompt: str
    max_tokens: int
    ignore_eos: bool = False
    temperature: float = 0.0
    top_k: int = -1
    top_p: float = 1.0


class Message(BaseModel):
    role: Literal["system", "user", "assistant"]
    content: str


class OpenAICompletionRequest(BaseModel):
    model: str = ""
    prompt: str | None = None
    messages: List[Message] | None = None
    max_tokens: int | None = 16  # null: up to the context limit
    temperature: float = 1.0
    top_k: int = -1
    top_p: float = 1.0
    n: int = 1
    stream: bool = False
    stop: List[str] | str | None = None  # one string or several; output ends before the first match
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    ignore_eos: bool = False
    seed: int | None = None
    stream_options: Dict[str, bool] | None = None  # {"include_usage": true}: a final usage chunk

    def stop_list(self) -> List[str]:
        return [self.stop] if isinstance(self.stop, str) else list(self.stop or [])

    def sampling(self) -> SamplingParams:
        # the scheduler clamps max_tokens to what the context leaves after the prompt
        max_tokens = UNBOUNDED_MAX_TOKENS if self.max_tokens is None else self.max_tokens
        return SamplingParams(temperature=self.temperature, top_k=self.top_k, top_p=self.top_p,
                              ignore_eos=self.ignore_eos, max_tokens=max_tokens, seed=self.seed)


class StopMatcher:
    """Cuts a streamed completion at the first occurrence of any stop string (OpenAI ``stop``).

    ``feed`` returns the text that is safe to send: it holds back a tail that could still grow
    into a stop string across chunk boundaries. After a match ``done`` is set and the text before
    the stop string is the last output; ``flush`` releases the held tail at the end of a request.
    (The reference accepts ``stop`` and ignores it.)"""

    def __init__(self, stops: List[str]):
        self.stops = [x for x in stops if x]
        self.buf = ""
        self.done = False

    def feed(self, piece: str) -> str:
        if not self.stops:
            return piece
        self.buf += piece
        hits = [i for i in (self.buf.find(x) for x in self.stops) if i >= 0]
        if hits:
            out, self.buf, self.done = self.buf[: min(hits)], "", True
            return out
        hold = 0
        for x in self.stops:
            for k in range(min(len(x) - 1, len(self.buf)), hold, -1):
                if self.buf.endswith(x[:k]):
                    hold = k
                    break
        out, self.buf = self.buf[: len(self.buf) - hold], self.buf[len(self.buf) - hold:]
        return out

    def flush(self) -> str:
        out, self.buf = self.buf, ""
        return out


class ModelCard(BaseModel):
    id: str
    object: str = "model"
    created: int = Field(default_factory=lambda: int(time.time()))
    owned_by: str = "minisgl"
    root: str


class ModelList(BaseModel):
    object: str = "list"
    data: List[ModelCard] = Field(default_factory=list)


@dataclass
class _Pending:
    replies: List[UserReply] = field(default_factory=list)
    event: asyncio.Event = field(default_factory=asyncio.Event)
    prompt_tokens: int = 0  # reported by the tokenizer worker


@dataclass
class FrontendManager:
    config: object
    send_tokenizer: object
    recv_tokenizer: object
    next_uid: int = 0
    pending: Dict[int, _Pending] = field(default_factory=dict)
    _listener: asyncio.Task | None = None

    def new_user(self) -> int:
        uid = self.next_uid
        self.next_uid += 1
        self.pending[uid] = _Pending()
        return uid

    async def _listen(self) -> None:
        while True:
            msg = await self.recv_tokenizer.get()
            for r in (msg.data if isinstance(msg, BatchFrontendMsg) else [msg]):
                p = self.pending.get(r.uid)
                if p is not None:
                    p.replies.append(r)
                    p.event.set()

    async def send_one(self, msg: BaseTokenizerMsg) -> None:
        if self._listener is None:
            self._listener = asyncio.create_task(self._listen())
        await self.send_tokenizer.put(msg)

    async def replies(self, uid: int) -> AsyncIterator[UserReply]:
        p = self.pending[uid]
        try:
            while True:
                await p.event.wait()
                p.event.clear()
                batch, p.replies = p.replies, []
                for r in batch:
                    if r.num_input_tokens and not r.finished and not r.incremental_output:
                        p.prompt_tokens = r.num_input_tokens  # prompt length, not output
                        continue
                    yield r
                    if r.finished:
                        return
        finally:
            self.pending.pop(uid, None)

    async def abort_user(self, uid: int) -> None:
        self.pending.pop(uid, None)
        logger.warning(f"aborting request {uid}")
        await self.send_one(AbortMsg(uid=uid))

    async def guard(self, gen: AsyncIterator[bytes], request: Request, uid: int) -> AsyncIterator[bytes]:
        """Stream ``gen``; abort the request if the client goes away."""
        finished = False
        try:
            async for chunk in gen:
                if await request.is_disconnected():
                    raise asyncio.CancelledError
                yield chunk
            finished = True
        finally:
            if not finished:
                asyncio.ensure_future(self.abort_user(uid))

    async def stream_text(self, uid: int) -> AsyncIterator[bytes]:
        async for r in self.replies(uid):
            yield f"data: {r.incremental_output}\n".encode()
        yield b"data: [DONE]\n"

    async def stream_chat(self, uid: int, model: str, chat: bool, stop: List[str] = (),
                          include_usage: bool = False) -> AsyncIterator[bytes]:
        first = True
        pend = self.pending.get(uid)
        n_out = 0
        obj = "chat.completion.chunk" if chat else "text_completion"
        matcher = StopMatcher(list(stop))

        def chunk(text: str) -> bytes:
            if chat:
                delta = {"role": "assistant"} if first else {}
                if text:
                    delta["content"] = text
                choice = {"delta": delta, "index": 0, "finish_reason": None}
            else:
                choice = {"text": text, "index": 0, "finish_reason": None}
            return f"data: {json.dumps({'id': f'cmpl-{uid}', 'object': obj, 'model': model, 'choices': [choice]})}\n\n".encode()

        reason = "stop"
        async for r in self.replies(uid):
            n_out += 1
            text = matcher.feed(r.incremental_output)
            if r.finished:
                text += matcher.flush()
                reason = r.finish_reason or "stop"
            yield chunk(text)
            first = False
            if matcher.done:  # stop string reached: the scheduler can drop the request
                await self.abort_user(uid)
                break
        end = {"delta": {}, "index": 0, "finish_reason": reason} if chat else {"text": "", "index": 0, "finish_reason": reason}
        yield f"data: {json.dumps({'id': f'cmpl-{uid}', 'object': obj, 'model': model, 'choices': [end]})}\n\n".encode()
        if include_usage:  # OpenAI stream_options.include_usage: one last chunk with no choices
            p_tok = pend.prompt_tokens if pend is not None else 0
            usage = {"prompt_tokens": p_tok, "completion_tokens": n_out, "total_tokens": p_tok + n_out}
            yield f"data: {json.dumps({'id': f'cmpl-{uid}', 'object': obj, 'model': model, 'choices': [], 'usage': usage})}\n\n".encode()
        yield b"data: [DONE]\n\n"

    def shutdown(self) -> None:
        self.send_tokenizer.stop()
        self.recv_tokenizer.stop()


_STATE: FrontendManager | None = None


def get_global_state() -> FrontendManager:
    if _STATE is None:
        raise RuntimeError("frontend not initialized")
    return _STATE


@asynccontextmanager
async def lifespan(_: FastAPI):
    yield
    if _STATE is not None:
        _STATE.shutdown()


app = FastAPI(title="minisgl API server", version="0.1.0", lifespan=lifespan)


@app.post("/generate")
async def generate(req: GenerateRequest, request: Request):
    st = get_global_state()
    uid = st.new_user()
    sp = SamplingParams(temperature=req.temperature, top_k=req.top_k, top_p=req.top_p,
                        ignore_eos=req.ignore_eos, max_tokens=req.max_tokens)
    await st.send_one(TokenizeMsg(uid=uid, text=req.prompt, sampling_params=sp))
    return StreamingResponse(st.guard(st.stream_text(uid), request, uid), media_type="text/event-stream")


@app.api_route("/v1", methods=["GET", "POST", "HEAD", "OPTIONS"])
async def v1_root():
    return {"status": "ok"}


async def _completion(req: OpenAICompletionRequest, request: Request, chat: bool):
    st = get_global_state()
    if chat and req.messages:
        text = [m.model_dump() for m in req.messages]
    elif req.prompt is not None:
        text = req.prompt
    elif req.messages:
        text = [m.model_dump() for m in req.messages]
    else:
        return {"error": "either 'messages' or 'prompt' is required"}
    n_choices = max(1, req.n)
    if req.stream and n_choices > 1:
        return {"error": "stream with n > 1 is not supported"}
    uids = [st.new_user() for _ in range(n_choices)]
    pend = st.pending[uids[0]]
    for i, u in enumerate(uids):
        sp = req.sampling()
        if sp.seed is not None:
            sp.seed += i  # n choices from one seed: distinct, reproducible draws
        await st.send_one(TokenizeMsg(uid=u, text=text, sampling_params=sp))
    if req.stream:
        uid = uids[0]
        usage = bool((req.stream_options or {}).get("include_usage"))
        return StreamingResponse(st.guard(st.stream_chat(uid, req.model, chat, req.stop_list(), usage), request, uid),
                                 media_type="text/event-stream")

    async def collect(uid: int, index: int):
        content, n, reason = "", 0, "stop"
        matcher = StopMatcher(req.stop_list())
        async for r in st.replies(uid):
            content += matcher.feed(r.incremental_output)
            n += 1
            if r.finished:
                content += matcher.flush()
                reason = r.finish_reason or "stop"
            if matcher.done:
                await st.abort_user(uid)
                break
        choice = ({"index": index, "message": {"role": "assistant", "content": content}, "finish_reason": reason}
                  if chat else {"index": index, "text": content, "finish_reason": reason})
        return choice, n

    results = await asyncio.gather(*[collect(u, i) for i, u in enumerate(uids)])
    n_out = sum(k for _, k in results)
    return {"id": f"{'chat' if chat else ''}cmpl-{uids[0]}", "object": "chat.completion" if chat else "text_completion",
            "created": int(time.time()), "model": req.model, "choices": [c for c, _ in results],
            "usage": {"prompt_tokens": pend.prompt_tokens, "completion_tokens": n_out,
                      "total_tokens": pend.prompt_tokens + n_out}}


@app.post("/v1/chat/completions")
async def v1_chat_completions(req: OpenAICompletionRequest, request: Request):
    return await _completion(req, request, chat=True)


@app.post("/v1/completions")
async def v1_completions(req: OpenAICompletionRequest, request: Request):
    return await _completion(req, request, chat=False)


@app.get("/v1/models")
async def available_models():
    st = get_global_state()
    return ModelList(data=[ModelCard(id=st.config.model_path, root=st.config.model_path)])


# ---------------------------------------------------------------------------------------- shell
async def _read_line(prompt: str) -> str:
    try:
        from prompt_toolkit import PromptSession
        from prompt_toolkit.completion import WordCompleter

        if not hasattr(_read_line, "session"):
            _read_line.session = PromptSession(prompt, completer=WordCompleter(["/exit", "/reset"]))
        return await _read_line.session.prompt_async()
    except ImportError:
        return await asyncio.to_thread(input, prompt)


async def shell() -> None:
    """Chat REPL: keeps the conversation, ``/reset`` clears it, ``/exit`` (or EOF) quits."""
    st = get_global_state()
    history: List[Message] = []
    try:
        while True:
            line = (await _read_line("$ ")).strip()
            if not line:
                continue
            if line == "/exit":
                break
            if line == "/reset":
                history = []
                continue
            if line.startswith("/"):
                print(f"unknown command {line}")
                continue
            msgs = history + [Message(role="user", content=line)]
            sp = SamplingParams(temperature=ENV.SHELL_TEMPERATURE, top_k=ENV.SHELL_TOP_K, top_p=ENV.SHELL_TOP_P,
                                max_tokens=ENV.SHELL_MAX_TOKENS)
            uid = st.new_user()
            await st.send_one(TokenizeMsg(uid=uid, text=[m.model_dump() for m in msgs], sampling_params=sp))
            answer = ""
            try:
                async for r in st.replies(uid):
                    answer += r.incremental_output
                    print(r.incremental_output, end="", flush=True)
            except (KeyboardInterrupt, asyncio.CancelledError):
                await st.abort_user(uid)
            print(flush=True)
            history = msgs + [Message(role="assistant", content=answer)]
    except EOFError:
        pass
    finally:
        print("Exiting shell...")
        st.shutdown()
        import psutil

        for child in psutil.Process().children(recursive=True):
            child.kill()


def run_api_server(config, start_backend: Callable[[], None], run_shell: bool) -> None:
    global _STATE
    import uvicorn

    from minisgl.utils.mp import ZmqAsyncPullQueue, ZmqAsyncPushQueue

    if _STATE is not None:
        raise RuntimeError("frontend already initialized")
    _STATE = FrontendManager(
        config=config,
        recv_tokenizer=ZmqAsyncPullQueue(config.zmq_frontend_addr, create=True, decoder=BaseFrontendMsg.decoder),
        send_tokenizer=ZmqAsyncPushQueue(config.zmq_tokenizer_addr, create=config.frontend_create_tokenizer_link,
                                         encoder=BaseTokenizerMsg.encoder),
    )
    start_backend()
    logger.info(f"API server ready on {config.server_host}:{config.server_port}")
    if run_shell:
        asyncio.run(shell())
    else:
        uvicorn.run(app, host=config.server_host, port=config.server_port, log_level="warning")
