"""Tokenizers and chat-prompt rendering.

* `HFTokenizer` wraps a model directory's `tokenizer.json` (HF `tokenizers`), with the
  model's own Jinja chat template when `tokenizer_config.json` carries one
  (harness/chat_template.rs:1-768 renders it with minijinja; here transformers'
  Jinja environment does), including `tools`, `enable_thinking` and arbitrary
  `chat_template_kwargs`.
* `ByteTokenizer` is a self-contained byte-level tokenizer with the Qwen special tokens,
  for random-init models that ship no tokenizer (no network on the serving hosts).
* `render_chatml` is the fallback prompt format (`format_qwen3_prompt`,
  harness/candle.rs:6860), used when no template is available or
  HELEXA_USE_CHAT_TEMPLATE=0 (the reference's NEURON_USE_CHAT_TEMPLATE kill switch).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass

SPECIALS = ["<|endoftext|>", "<|im_start|>", "<|im_end|>", "<think>", "</think>", "<tool_call>", "</tool_call>",
            "<|vision_start|>", "<|image_pad|>", "<|vision_end|>"]
IMAGE_PART_TYPES = ("image_url", "input_image", "image")


def _content_text(content) -> str:
    if content is None:
        return ""
    if isinstance(content, str):
        return content
    parts = []
    for p in content:
        if isinstance(p, dict) and p.get("type") in ("text", "input_text", "output_text"):
            parts.append(p.get("text", ""))
        elif isinstance(p, dict) and p.get("type") in IMAGE_PART_TYPES:
            # one pad per image; the vision front end expands it to the image's tokens
            parts.append("<|vision_start|><|image_pad|><|vision_end|>")
    return "".join(parts)


def render_chatml(messages: list[dict], add_generation_prompt: bool = True, enable_thinking: bool = True,
                  tools: list | None = None) -> str:
    out = []
    if tools:
        sys_extra = ("# Tools\n\nYou may call one or more functions to assist with the user query.\n\n"
                     "<tools>\n" + "\n".join(json.dumps(t) for t in tools) + "\n</tools>\n\n"
                     "For each function call, return a json object with function name and arguments within "
                     "<tool_call></tool_call> XML tags.")
        if messages and messages[0].get("role") == "system":
            messages = [dict(messages[0], content=_content_text(messages[0]["content"]) + "\n\n" + sys_extra)] + \
                list(messages[1:])
        else:
            messages = [{"role": "system", "content": sys_extra}] + list(messages)
    for m in messages:
        role = m.get("role", "user")
        if role == "tool":
            out.append(f"<|im_start|>user\n<tool_response>\n{_content_text(m.get('content'))}\n</tool_response>"
                       "<|im_end|>\n")
            continue
        text = _content_text(m.get("content"))
        if role == "assistant" and m.get("tool_calls"):
            for tc in m["tool_calls"]:
                fn = tc.get("function", tc)
                args = fn.get("arguments", {})
                if isinstance(args, str):
                    try:
                        args = json.loads(args)
                    except ValueError:
                        pass
                text += "\n<tool_call>\n" + json.dumps({"name": fn.get("name"), "arguments": args}) + \
                        "\n</tool_call>"
        out.append(f"<|im_start|>{role}\n{text}<|im_end|>\n")
    if add_generation_prompt:
        out.append("<|im_start|>assistant\n")
        if not enable_thinking:
            out.append("<think>\n\n</think>\n\n")
    return "".join(out)


class ByteTokenizer:
    """Bytes 0..255 map to ids 0..255; specials follow; ids past that decode to ''."""

    def __init__(self, vocab_size: int = 151936):
        self.vocab_size = vocab_size
        self.special_ids = {s: 256 + i for i, s in enumerate(SPECIALS)}
        self.id_to_special = {v: k for k, v in self.special_ids.items()}
        self.chat_template = None

    @property
    def eos_ids(self) -> list[int]:
        return [self.special_ids["<|im_end|>"], self.special_ids["<|endoftext|>"]]

    def token_id(self, s: str) -> int | None:
        return self.special_ids.get(s)

    def encode(self, text: str) -> list[int]:
        ids: list[int] = []
        i = 0
        while i < len(text):
            for sp, sid in self.special_ids.items():
                if text.startswith(sp, i):
                    ids.append(sid)
                    i += len(sp)
                    break
            else:
                ids.extend(text[i].encode("utf-8"))
                i += 1
        return ids

    def decode(self, ids: list[int]) -> str:
        buf = bytearray()
        out = []
        for t in ids:
            if t < 256:
                buf.append(t)
                continue
            if buf:
                out.append(buf.decode("utf-8", errors="replace"))
                buf = bytearray()
            out.append(self.id_to_special.get(t, ""))
        if buf:
            out.append(buf.decode("utf-8", errors="replace"))
        return "".join(out)

    def apply_chat_template(self, messages, add_generation_prompt=True, enable_thinking=True, tools=None, **kw):
        return render_chatml(messages, add_generation_prompt, enable_thinking, tools)


class HFTokenizer:
    def __init__(self, path: str):
        from tokenizers import Tokenizer

        self.tok = Tokenizer.from_file(os.path.join(path, "tokenizer.json"))
        self.vocab_size = self.tok.get_vocab_size()
        self.chat_template = None
        cfg_path = os.path.join(path, "tokenizer_config.json")
        if os.path.exists(cfg_path):
            with open(cfg_path) as f:
                tc = json.load(f)
            self.chat_template = tc.get("chat_template")
        tmpl = os.path.join(path, "chat_template.jinja")
        if self.chat_template is None and os.path.exists(tmpl):
            with open(tmpl) as f:
                self.chat_template = f.read()

    @property
    def eos_ids(self) -> list[int]:
        return [i for i in (self.token_id("<|im_end|>"), self.token_id("<|endoftext|>")) if i is not None]

    def token_id(self, s: str) -> int | None:
        return self.tok.token_to_id(s)

    def encode(self, text: str) -> list[int]:
        return self.tok.encode(text, add_special_tokens=False).ids

    def decode(self, ids: list[int]) -> str:
        return self.tok.decode(ids, skip_special_tokens=False)

    def apply_chat_template(self, messages, add_generation_prompt=True, enable_thinking=True, tools=None, **kw):
        if self.chat_template is None or os.environ.get("HELEXA_USE_CHAT_TEMPLATE", "1") == "0":
            return render_chatml(messages, add_generation_prompt, enable_thinking, tools)
        from transformers.utils.chat_template_utils import _compile_jinja_template

        tmpl = _compile_jinja_template(self.chat_template)
        return tmpl.render(messages=messages, add_generation_prompt=add_generation_prompt,
                           enable_thinking=enable_thinking, tools=tools, **kw)


def load_tokenizer(path: str | None, vocab_size: int):
    if path and os.path.exists(os.path.join(path, "tokenizer.json")):
        return HFTokenizer(path)
    return ByteTokenizer(vocab_size)


class IncrementalDetokenizer:
    """Token-by-token text deltas that never split a multi-byte character."""

    def __init__(self, tok):
        self.tok = tok
        self.ids: list[int] = []
        self.emitted = ""

    def push(self, new_ids: list[int]) -> str:
        self.ids.extend(new_ids)
        text = self.tok.decode(self.ids)
        if text.endswith("�"):
            return ""
        delta = text[len(self.emitted):]
        self.emitted = text
        return delta


@dataclass
class ParsedDelta:
    kind: str   # "text" | "reasoning" | "tool_call"
    text: str


class StreamParser:
    """Splits streamed text into visible content, reasoning and tool calls.

    `<think>...</think>` becomes reasoning (handle_reasoning_marker, harness/candle.rs:6131);
    `<tool_call>...</tool_call>` bodies become tool calls (handle_tool_call_marker,
    candle.rs:6191) with JSON or Qwen XML bodies (parse_tool_call_body, candle.rs:6274).
    A model whose template opens the assistant turn inside a think block starts in
    reasoning mode (`start_in_reasoning`).
    """

    TAGS = ("<think>", "</think>", "<tool_call>", "</tool_call>")

    def __init__(self, start_in_reasoning: bool = False):
        self.mode = "reasoning" if start_in_reasoning else "text"
        self.buf = ""
        self.tool_buf = ""

    def _flush_safe(self) -> tuple[str, str]:
        # keep a possible partial tag at the end of the buffer
        keep = 0
        for t in self.TAGS:
            for n in range(1, len(t)):
                if self.buf.endswith(t[:n]):
                    keep = max(keep, n)
        out, self.buf = (self.buf[:-keep], self.buf[-keep:]) if keep else (self.buf, "")
        return out, self.buf

    def feed(self, text: str, final: bool = False) -> list[ParsedDelta]:
        self.buf += text
        out: list[ParsedDelta] = []
        while True:
            idx, tag = min(((self.buf.find(t), t) for t in self.TAGS if self.buf.find(t) >= 0),
                           default=(-1, None))
            if tag is None:
                break
            before, self.buf = self.buf[:idx], self.buf[idx + len(tag):]
            self._emit(before, out)
            if tag == "<think>":
                self.mode = "reasoning"
            elif tag == "</think>":
                self.mode = "text"
            elif tag == "<tool_call>":
                self.mode = "tool"
                self.tool_buf = ""
            else:
                out.append(ParsedDelta("tool_call", self.tool_buf.strip()))
                self.mode = "text"
        if final:
            rest, self.buf = self.buf, ""
        else:
            rest, _ = self._flush_safe()
        self._emit(rest, out)
        if final and self.mode == "tool" and self.tool_buf.strip():
            out.append(ParsedDelta("tool_call", self.tool_buf.strip()))
            self.tool_buf = ""
        return out

    def _emit(self, s: str, out: list[ParsedDelta]):
        if not s:
            return
        if self.mode == "tool":
            self.tool_buf += s
        elif self.mode == "reasoning":
            out.append(ParsedDelta("reasoning", s))
        else:
            out.append(ParsedDelta("text", s))


def parse_tool_call_body(body: str) -> tuple[str, dict]:
    """JSON {"name", "arguments"} or Qwen XML <function=name><parameter=k>v</parameter>."""
    body = body.strip()
    try:
        obj = json.loads(body)
        args = obj.get("arguments", obj.get("parameters", {}))
        if isinstance(args, str):
            try:
                args = json.loads(args)
            except ValueError:
                args = {"_raw": args}
        return obj.get("name", ""), args
    except ValueError:
        pass
    import re
    m = re.search(r"<function=([^>\s]+)>(.*?)(</function>|$)", body, re.S)
    if not m:
        return "", {"_raw": body}
    name, inner = m.group(1), m.group(2)
    args = {}
    for pm in re.finditer(r"<parameter=([^>\s]+)>(.*?)</parameter>", inner, re.S):
        v = pm.group(2).strip()
        try:
            args[pm.group(1)] = json.loads(v)
        except ValueError:
            args[pm.group(1)] = v
    return name, args
