"""Reasoning and tool-call output parsers for the Qwen3 family.

* reasoning parser ``qwen3``: text before ``</think>`` (after an optional ``<think>``) is
  ``reasoning_content``; with thinking disabled by the chat template everything is content
  (reference: ``--reasoning-parser qwen3``, thinking on/off agreement ``patch_qwen3_thinkoff.py``).
* tool parsers: ``hermes`` / ``qwen3_json`` (``<tool_call>{json}</tool_call>``) and
  ``qwen3_xml`` / ``qwen3_coder`` (``<tool_call><function=NAME><parameter=K>V</parameter>...``)
  (reference: ``--tool-call-parser qwen3_xml``, ``patch_qwen3_toolparse.py``).
"""
from __future__ import annotations

import json
import re
import uuid
from typing import Optional


class ReasoningParser:
    START, END = "<think>", "</think>"

    def __init__(self, name: str = "qwen3", thinking: bool = True):
        if name not in ("qwen3", "deepseek_r1"):
            raise ValueError(f"unknown reasoning parser {name!r}")
        self.thinking = thinking
        self.buf = ""
        self.sent_r = 0
        self.sent_c = 0
        self.content = ""

    def split(self, text: str):
        if not self.thinking:
            t = text.replace(self.START, "").replace(self.END, "")
            return None, t.lstrip("\n")
        t = text
        if t.startswith(self.START):
            t = t[len(self.START):]
        i = t.find(self.END)
        if i < 0:
            return t.strip("\n"), ""
        return t[:i].strip("\n"), t[i + len(self.END):].lstrip("\n")

    def stream(self, delta: str):
        """Incremental split: returns (reasoning delta, content delta)."""
        self.buf += delta
        r, c = self.split(self.buf)
        if r is not None and self.END not in self.buf and self.thinking:
            # hold back a partial end tag
            for k in range(len(self.END) - 1, 0, -1):
                if r.endswith(self.END[:k]):
                    r = r[:-k]
                    break
        r = r or ""
        dr, dc = r[self.sent_r:], c[self.sent_c:]
        self.sent_r, self.sent_c = len(r), len(c)
        self.content = c
        return dr, dc


_JSON_CALL = re.compile(r"<tool_call>\s*(\{.*?\})\s*</tool_call>", re.S)
_XML_CALL = re.compile(r"<tool_call>\s*<function=([^>\s]+)>(.*?)</function>\s*</tool_call>", re.S)
_XML_PARAM = re.compile(r"<parameter=([^>\s]+)>(.*?)</parameter>", re.S)


def _coerce(v: str):
    v = v.strip("\n")
    try:
        return json.loads(v)
    except (ValueError, TypeError):
        return v


class ToolParser:
    def __init__(self, name: str = "qwen3_xml"):
        if name not in ("hermes", "qwen3_json", "qwen3_xml", "qwen3_coder"):
            raise ValueError(f"unknown tool parser {name!r}")
        self.name = name

    def parse(self, text: str):
        """-> (list of OpenAI tool_call dicts, remaining content)."""
        calls = []
        rest = text
        if self.name in ("qwen3_xml", "qwen3_coder"):
            for m in _XML_CALL.finditer(text):
                args = {k: _coerce(v) for k, v in _XML_PARAM.findall(m.group(2))}
                calls.append(self._call(m.group(1), args))
            rest = _XML_CALL.sub("", text)
        if not calls:
            for m in _JSON_CALL.finditer(text):
                try:
                    obj = json.loads(m.group(1))
                except ValueError:
                    continue
                calls.append(self._call(obj.get("name", ""), obj.get("arguments", {})))
            if calls:
                rest = _JSON_CALL.sub("", text)
        return calls, rest.strip()

    @staticmethod
    def _call(name, args):
        return {"id": f"call_{uuid.uuid4().hex[:24]}", "type": "function",
                "function": {"name": name,
                             "arguments": args if isinstance(args, str) else json.dumps(args)}}
