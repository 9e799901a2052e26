"""Wire projections of the engine's event stream.

* OpenAI chat completions (wire/openai_chat.rs): a role chunk, one content chunk per
  visible delta, tool-call chunks, a final chunk with `finish_reason`, `usage`
  (`prompt_tokens_details.cached_tokens`, `completion_tokens_details.reasoning_tokens`)
  and `helexa_timing`; reasoning is dropped unless the caller opted in
  (`x-include-thinking`), in which case it is sent as `reasoning_content`.
* OpenAI Responses (wire/openai_responses.rs): request -> chat translation (rejects
  `previous_response_id`) and the named SSE event family.
* Anthropic Messages (cortex-core/src/translate.rs): request translation (system,
  content blocks, tools, tool_use / tool_result) and the message_* / content_block_*
  stream.
* The OpenAI error envelope (cortex-core/src/error_envelope.rs).
"""
from __future__ import annotations

import json
import time
import uuid

from ..runtime.serving import Finish, ReasoningDelta, Start, TextDelta, ToolCall


def sse(obj) -> str:
    return "data: " + json.dumps(obj, separators=(",", ":")) + "\n\n"


def sse_named(event: str, obj) -> str:
    return f"event: {event}\ndata: " + json.dumps(obj, separators=(",", ":")) + "\n\n"


def error_body(message: str, code: str = "invalid_request_error", typ: str | None = None, param=None) -> dict:
    return {"error": {"message": message, "type": typ or code, "param": param, "code": code}}


def usage_obj(f: Finish) -> dict:
    return {
        "prompt_tokens": f.prompt_tokens, "completion_tokens": f.completion_tokens,
        "total_tokens": f.prompt_tokens + f.completion_tokens,
        "prompt_tokens_details": {"cached_tokens": f.cached_tokens},
        "completion_tokens_details": {"reasoning_tokens": f.reasoning_tokens},
        "helexa_timing": {"prefill_ms": round(f.prefill_ms, 3), "decode_ms": round(f.decode_ms, 3),
                          "prefill_tokens": f.prefill_tokens},
    }


# ---- OpenAI chat ------------------------------------------------------------------
async def chat_sse(events, include_reasoning: bool):
    start = None
    async for ev in events:
        if isinstance(ev, Start):
            start = ev
            yield sse(_chunk(start, {"role": "assistant", "content": ""}, None))
        elif isinstance(ev, TextDelta):
            yield sse(_chunk(start, {"content": ev.text}, None))
        elif isinstance(ev, ReasoningDelta):
            if include_reasoning:
                yield sse(_chunk(start, {"reasoning_content": ev.text}, None))
        elif isinstance(ev, ToolCall):
            yield sse(_chunk(start, {"tool_calls": [{"index": ev.index, "id": ev.id, "type": "function",
                                                     "function": {"name": ev.name, "arguments": ev.arguments}}]},
                             None))
        elif isinstance(ev, Finish):
            c = _chunk(start, {}, ev.reason if ev.reason != "error" else "error")
            c["usage"] = usage_obj(ev)
            if ev.error:
                c["error"] = {"message": ev.error}
            yield sse(c)
    yield "data: [DONE]\n\n"


def _chunk(start: Start, delta: dict, finish) -> dict:
    return {"id": start.id, "object": "chat.completion.chunk", "created": start.created, "model": start.model,
            "choices": [{"index": 0, "delta": delta, "finish_reason": finish}]}


def chat_response(start: Start, text: str, reasoning: str, tools: list[ToolCall], fin: Finish,
                  include_reasoning: bool) -> dict:
    msg = {"role": "assistant", "content": text if (text or not tools) else None}
    if include_reasoning and reasoning:
        msg["reasoning_content"] = reasoning
    if tools:
        msg["tool_calls"] = [{"id": t.id, "type": "function", "function": {"name": t.name, "arguments": t.arguments}}
                             for t in tools]
    return {"id": start.id, "object": "chat.completion", "created": start.created, "model": start.model,
            "choices": [{"index": 0, "message": msg, "finish_reason": fin.reason}], "usage": usage_obj(fin)}


# ---- OpenAI completions -------------------------------------------------------------
async def completion_sse(events):
    start = None
    async for ev in events:
        if isinstance(ev, Start):
            start = ev
        elif isinstance(ev, (TextDelta, ReasoningDelta)):
            yield sse({"id": start.id, "object": "text_completion", "created": start.created, "model": start.model,
                       "choices": [{"index": 0, "text": ev.text, "finish_reason": None}]})
        elif isinstance(ev, Finish):
            yield sse({"id": start.id, "object": "text_completion", "created": start.created, "model": start.model,
                       "choices": [{"index": 0, "text": "", "finish_reason": ev.reason}], "usage": usage_obj(ev)})
    yield "data: [DONE]\n\n"


# ---- OpenAI Responses ---------------------------------------------------------------
def responses_to_chat(req: dict) -> dict:
    if req.get("previous_response_id"):
        raise ValueError("previous_response_id is not supported; send the full conversation in `input`")
    msgs = []
    if req.get("instructions"):
        msgs.append({"role": "system", "content": req["instructions"]})
    inp = req.get("input", "")
    if isinstance(inp, str):
        msgs.append({"role": "user", "content": inp})
    else:
        for item in inp:
            t = item.get("type", "message")
            if t == "message":
                msgs.append({"role": item.get("role", "user"), "content": item.get("content", "")})
            elif t == "function_call":
                msgs.append({"role": "assistant", "content": "", "tool_calls": [{
                    "id": item.get("call_id"), "type": "function",
                    "function": {"name": item.get("name"), "arguments": item.get("arguments", "{}")}}]})
            elif t == "function_call_output":
                msgs.append({"role": "tool", "tool_call_id": item.get("call_id"), "content": item.get("output", "")})
    tools = []
    for t in req.get("tools") or []:
        if t.get("type") == "function":
            tools.append({"type": "function", "function": {k: t[k] for k in ("name", "description", "parameters")
                                                           if k in t}})
    out = {"messages": msgs, "stream": req.get("stream", False)}
    if tools:
        out["tools"] = tools
    for k_src, k_dst in (("max_output_tokens", "max_tokens"), ("temperature", "temperature"), ("top_p", "top_p")):
        if req.get(k_src) is not None:
            out[k_dst] = req[k_src]
    return out


async def responses_sse(events, model: str):
    rid = "resp_" + uuid.uuid4().hex[:24]
    created = int(time.time())
    base = {"id": rid, "object": "response", "created_at": created, "model": model, "status": "in_progress",
            "output": []}
    seq = 0

    def ev(name, obj):
        nonlocal seq
        obj = dict(obj, type=name, sequence_number=seq)
        seq += 1
        return sse_named(name, obj)

    yield ev("response.created", {"response": base})
    msg_id = "msg_" + uuid.uuid4().hex[:24]
    text_open = False
    text = []
    out_items = []
    async for e in events:
        if isinstance(e, TextDelta):
            if not text_open:
                text_open = True
                yield ev("response.output_item.added", {"output_index": len(out_items), "item": {
                    "id": msg_id, "type": "message", "role": "assistant", "status": "in_progress", "content": []}})
                yield ev("response.content_part.added", {"item_id": msg_id, "output_index": len(out_items),
                                                         "content_index": 0,
                                                         "part": {"type": "output_text", "text": ""}})
            text.append(e.text)
            yield ev("response.output_text.delta", {"item_id": msg_id, "output_index": len(out_items),
                                                    "content_index": 0, "delta": e.text})
        elif isinstance(e, ToolCall):
            item = {"id": "fc_" + uuid.uuid4().hex[:20], "type": "function_call", "call_id": e.id, "name": e.name,
                    "arguments": e.arguments, "status": "completed"}
            idx = len(out_items) + (1 if text_open else 0)
            yield ev("response.output_item.added", {"output_index": idx, "item": dict(item, arguments="")})
            yield ev("response.function_call_arguments.delta", {"item_id": item["id"], "output_index": idx,
                                                                "delta": e.arguments})
            yield ev("response.function_call_arguments.done", {"item_id": item["id"], "output_index": idx,
                                                               "arguments": e.arguments})
            yield ev("response.output_item.done", {"output_index": idx, "item": item})
            out_items.append(item)
        elif isinstance(e, Finish):
            if text_open:
                full = "".join(text)
                yield ev("response.output_text.done", {"item_id": msg_id, "output_index": 0, "content_index": 0,
                                                       "text": full})
                part = {"type": "output_text", "text": full, "annotations": []}
                yield ev("response.content_part.done", {"item_id": msg_id, "output_index": 0, "content_index": 0,
                                                        "part": part})
                item = {"id": msg_id, "type": "message", "role": "assistant", "status": "completed",
                        "content": [part]}
                yield ev("response.output_item.done", {"output_index": 0, "item": item})
                out_items.insert(0, item)
            done = dict(base, status="completed" if e.reason != "error" else "failed", output=out_items,
                        usage={"input_tokens": e.prompt_tokens, "output_tokens": e.completion_tokens,
                               "total_tokens": e.prompt_tokens + e.completion_tokens,
                               "input_tokens_details": {"cached_tokens": e.cached_tokens},
                               "output_tokens_details": {"reasoning_tokens": e.reasoning_tokens}})
            yield ev("response.completed", {"response": done})


def responses_object(model: str, text: str, tools: list[ToolCall], fin: Finish) -> dict:
    out = []
    if text:
        out.append({"id": "msg_" + uuid.uuid4().hex[:24], "type": "message", "role": "assistant",
                    "status": "completed", "content": [{"type": "output_text", "text": text, "annotations": []}]})
    for t in tools:
        out.append({"id": "fc_" + uuid.uuid4().hex[:20], "type": "function_call", "call_id": t.id, "name": t.name,
                    "arguments": t.arguments, "status": "completed"})
    return {"id": "resp_" + uuid.uuid4().hex[:24], "object": "response", "created_at": int(time.time()),
            "model": model, "status": "completed", "output": out, "output_text": text,
            "usage": {"input_tokens": fin.prompt_tokens, "output_tokens": fin.completion_tokens,
                      "total_tokens": fin.prompt_tokens + fin.completion_tokens}}


# ---- Anthropic Messages ---------------------------------------------------------------
def anthropic_to_openai(req: dict) -> dict:
    msgs = []
    sys = req.get("system")
    if sys:
        msgs.append({"role": "system", "content": sys if isinstance(sys, str) else
                     "".join(b.get("text", "") for b in sys if b.get("type") == "text")})
    for m in req.get("messages", []):
        content = m.get("content")
        if isinstance(content, str):
            msgs.append({"role": m["role"], "content": content})
            continue
        texts, calls = [], []
        for b in content or []:
            t = b.get("type")
            if t == "text":
                texts.append(b.get("text", ""))
            elif t == "tool_use":
                calls.append({"id": b.get("id"), "type": "function",
                              "function": {"name": b.get("name"), "arguments": json.dumps(b.get("input", {}))}})
            elif t == "tool_result":
                c = b.get("content")
                if isinstance(c, list):
                    c = "".join(x.get("text", "") for x in c if x.get("type") == "text")
                msgs.append({"role": "tool", "tool_call_id": b.get("tool_use_id"), "content": c or ""})
        if texts or calls:
            mm = {"role": m["role"], "content": "".join(texts)}
            if calls:
                mm["tool_calls"] = calls
            msgs.append(mm)
    out = {"messages": msgs, "max_tokens": req.get("max_tokens", 1024), "stream": req.get("stream", False)}
    for k in ("temperature", "top_p", "top_k"):
        if req.get(k) is not None:
            out[k] = req[k]
    if req.get("stop_sequences"):
        out["stop"] = req["stop_sequences"]
    if req.get("tools"):
        out["tools"] = [{"type": "function", "function": {"name": t["name"], "description": t.get("description", ""),
                                                          "parameters": t.get("input_schema", {})}}
                        for t in req["tools"]]
    th = req.get("thinking")
    if isinstance(th, dict):
        out["chat_template_kwargs"] = {"enable_thinking": th.get("type") == "enabled"}
    return out


_STOP = {"stop": "end_turn", "length": "max_tokens", "tool_calls": "tool_use", "cancelled": "end_turn",
         "error": "end_turn"}


async def anthropic_sse(events, model: str, include_thinking: bool):
    mid = "msg_" + uuid.uuid4().hex[:24]
    idx = -1
    open_kind = None
    yield sse_named("message_start", {"type": "message_start", "message": {
        "id": mid, "type": "message", "role": "assistant", "model": model, "content": [], "stop_reason": None,
        "stop_sequence": None, "usage": {"input_tokens": 0, "output_tokens": 0}}})

    def close():
        return sse_named("content_block_stop", {"type": "content_block_stop", "index": idx})

    async for e in events:
        if isinstance(e, ReasoningDelta) and include_thinking:
            if open_kind != "thinking":
                if open_kind:
                    yield close()
                idx += 1
                open_kind = "thinking"
                yield sse_named("content_block_start", {"type": "content_block_start", "index": idx,
                                                        "content_block": {"type": "thinking", "thinking": ""}})
            yield sse_named("content_block_delta", {"type": "content_block_delta", "index": idx,
                                                    "delta": {"type": "thinking_delta", "thinking": e.text}})
        elif isinstance(e, TextDelta):
            if open_kind != "text":
                if open_kind:
                    yield close()
                idx += 1
                open_kind = "text"
                yield sse_named("content_block_start", {"type": "content_block_start", "index": idx,
                                                        "content_block": {"type": "text", "text": ""}})
            yield sse_named("content_block_delta", {"type": "content_block_delta", "index": idx,
                                                    "delta": {"type": "text_delta", "text": e.text}})
        elif isinstance(e, ToolCall):
            if open_kind:
                yield close()
            idx += 1
            open_kind = None
            yield sse_named("content_block_start", {"type": "content_block_start", "index": idx, "content_block": {
                "type": "tool_use", "id": e.id, "name": e.name, "input": {}}})
            yield sse_named("content_block_delta", {"type": "content_block_delta", "index": idx,
                                                    "delta": {"type": "input_json_delta",
                                                              "partial_json": e.arguments}})
            yield close()
        elif isinstance(e, Finish):
            if open_kind:
                yield close()
            yield sse_named("message_delta", {"type": "message_delta", "delta": {
                "stop_reason": _STOP.get(e.reason, "end_turn"), "stop_sequence": None},
                "usage": {"input_tokens": e.prompt_tokens, "output_tokens": e.completion_tokens,
                          "cache_read_input_tokens": e.cached_tokens}})
            yield sse_named("message_stop", {"type": "message_stop"})


def anthropic_message(model: str, text: str, reasoning: str, tools: list[ToolCall], fin: Finish,
                      include_thinking: bool) -> dict:
    content = []
    if include_thinking and reasoning:
        content.append({"type": "thinking", "thinking": reasoning})
    if text:
        content.append({"type": "text", "text": text})
    for t in tools:
        try:
            inp = json.loads(t.arguments)
        except ValueError:
            inp = {"_raw": t.arguments}
        content.append({"type": "tool_use", "id": t.id, "name": t.name, "input": inp})
    return {"id": "msg_" + uuid.uuid4().hex[:24], "type": "message", "role": "assistant", "model": model,
            "content": content, "stop_reason": _STOP.get(fin.reason, "end_turn"), "stop_sequence": None,
            "usage": {"input_tokens": fin.prompt_tokens, "output_tokens": fin.completion_tokens,
                      "cache_read_input_tokens": fin.cached_tokens}}
