"""Tool-call extraction from model output.

Dialects (the same set crates/cascadia-api/src/lib.rs:1380-1480 accepts):
* Qwen/Hermes JSON inside ``<tool_call>...</tool_call>`` (brace-balanced scan, so
  a literal close tag inside an argument string cannot truncate the block);
* Qwen3-MoE XML ``<function=name><parameter=k>v</parameter></function>``;
* GLM bare name + ``<arg_key>k</arg_key><arg_value>v</arg_value>``;
* Llama-3.1 ``<|python_tag|>`` JSON, or a bare whole-output JSON object/array
  that carries ``arguments``/``parameters`` (so plain JSON data answers are
  not misread as calls).
"""
from __future__ import annotations

import json
import re
import uuid
from dataclasses import dataclass
from typing import List, Optional


@dataclass
class ToolCall:
    id: str
    name: str
    arguments: str  # JSON text
    type: str = "function"

    def to_openai(self, index: Optional[int] = None) -> dict:
        d = {"id": self.id, "type": self.type,
             "function": {"name": self.name, "arguments": self.arguments}}
        if index is not None:
            d["index"] = index
        return d


def _new_id() -> str:
    return "call_" + uuid.uuid4().hex[:24]


def balanced_json_end(s: str) -> Optional[int]:
    if not s or s[0] not in "{[":
        return None
    open_c, close_c = ("{", "}") if s[0] == "{" else ("[", "]")
    depth, in_str, esc = 0, False, False
    for i, ch in enumerate(s):
        if in_str:
            if esc:
                esc = False
            elif ch == "\\":
                esc = True
            elif ch == '"':
                in_str = False
            continue
        if ch == '"':
            in_str = True
        elif ch == open_c:
            depth += 1
        elif ch == close_c:
            depth -= 1
            if depth == 0:
                return i + 1
    return None


def _call_from_value(v) -> Optional[ToolCall]:
    if not isinstance(v, dict):
        return None
    name = v.get("name")
    if name is None and isinstance(v.get("function"), dict):
        fn = v["function"]
        name, args = fn.get("name"), fn.get("arguments", fn.get("parameters", {}))
    else:
        args = v.get("arguments", v.get("parameters", {}))
    if not isinstance(name, str):
        return None
    if not isinstance(args, str):
        args = json.dumps(args, separators=(",", ":"))
    return ToolCall(_new_id(), name, args)


def _coerce(v: str):
    s = v.strip()
    try:
        return json.loads(s)
    except (ValueError, TypeError):
        return s


_XML_FN = re.compile(r"<function=([^>\s]+)>(.*?)(?:</function>|$)", re.S)
_XML_PARAM = re.compile(r"<parameter=([^>\s]+)>(.*?)</parameter>", re.S)
_GLM_KV = re.compile(r"<arg_key>(.*?)</arg_key>\s*<arg_value>(.*?)</arg_value>", re.S)


def _call_from_xml_function(block: str) -> Optional[ToolCall]:
    m = _XML_FN.search(block)
    if not m:
        return None
    args = {k.strip(): _coerce(v) for k, v in _XML_PARAM.findall(m.group(2))}
    return ToolCall(_new_id(), m.group(1).strip(), json.dumps(args, separators=(",", ":")))


def _call_from_glm(block: str) -> Optional[ToolCall]:
    if "<arg_key>" not in block:
        name = block.strip()
        if name and re.fullmatch(r"[\w.\-]+", name):
            return ToolCall(_new_id(), name, "{}")
        return None
    name = block.split("<arg_key>", 1)[0].strip()
    if not name:
        return None
    args = {k.strip(): _coerce(v) for k, v in _GLM_KV.findall(block)}
    return ToolCall(_new_id(), name, json.dumps(args, separators=(",", ":")))


def parse_tool_calls(text: str) -> Optional[List[ToolCall]]:
    calls: List[ToolCall] = []
    if "<tool_call>" in text:
        rest = text
        while "<tool_call>" in rest:
            after = rest[rest.index("<tool_call>") + len("<tool_call>"):]
            inner = after.lstrip()
            if inner[:1] in ("{", "["):
                off = len(after) - len(inner)
                n = balanced_json_end(after[off:])
                if n is not None:
                    try:
                        v = json.loads(after[off:off + n])
                        vals = v if isinstance(v, list) else [v]
                        for x in vals:
                            c = _call_from_value(x)
                            if c:
                                calls.append(c)
                    except ValueError:
                        pass
                    tail = after[off + n:]
                    e = tail.find("</tool_call>")
                    rest = tail[e + len("</tool_call>"):] if e >= 0 else tail
                    continue
            end = after.find("</tool_call>")
            if end < 0:
                break
            c = _call_from_xml_function(after[:end]) or _call_from_glm(after[:end])
            if c:
                calls.append(c)
            rest = after[end + len("</tool_call>"):]
    else:
        t = text.strip()
        explicit = t.startswith("<|python_tag|>")
        cand = t[len("<|python_tag|>"):].strip() if explicit else t
        if explicit or cand[:1] in ("{", "["):
            try:
                v = json.loads(cand)
            except ValueError:
                v = None
            vals = v if isinstance(v, list) else ([v] if v is not None else [])
            for x in vals:
                if isinstance(x, dict) and (explicit or "arguments" in x or "parameters" in x):
                    c = _call_from_value(x)
                    if c:
                        calls.append(c)
    return calls or None


def tool_call_scan_text(text: str, enable_thinking: bool) -> str:
    """Ignore tool-call-looking text inside a reasoning block."""
    if enable_thinking and "</think>" in text:
        return text.split("</think>", 1)[1]
    return text
