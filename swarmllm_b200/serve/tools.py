"""Tool calling for local models: the prompt that declares the tools, and the
parser that turns the model's text back into structured tool calls.

A local GGUF model emits tool calls as text.  The server asks for one flat
JSON shape (``{"tool_calls": [{"name", "arguments"}]}``) in a system prompt,
and parses that first; instruction-tuned models often answer in the format
they were trained on instead, so the native families are parsed too, each by
its own small function tried in a fixed order:

  generic   {"tool_calls": [{"name", "arguments"}]} (also the nested
            {"function": {"name", "arguments"}} wire shape)
  hermes    <tool_call>{"name", "arguments"}</tool_call>, one block per call
  qwen-xml  <tool_call><function=NAME><parameter=P>V</parameter></function></tool_call>
  mistral   [TOOL_CALLS][{"name", "arguments"}]  or  [TOOL_CALLS]NAME[ARGS]{...}
  phi       functools[{...}]  or  <|tool_calls|>[...]<|/tool_calls|>
  llama3    <|python_tag|>{"name", "parameters"} or a bare such object (last:
            it accepts a bare object and would swallow the other shapes)

Only calls that name a declared tool are accepted, and truncated JSON is
reported as text rather than repaired (a call with invented arguments is
worse than the raw output).  While streaming, ``content_prefix_len`` says how
much of the text so far is certainly content (before anything that could
start a call), so plain answers still stream token by token.

Reference behaviour: src/api/tool_parse.rs (format_tool_prompt:77,
parse_tool_calls:299, content_prefix_len:432, per-family try_* parsers).
"""
from __future__ import annotations

import json
import re
import uuid
from dataclasses import dataclass, field

_DEC = json.JSONDecoder()

# strings that may open a tool call; text before the first one streams as content
MARKERS = ("<tool_call>", "<tools>", "[TOOL_CALLS]", "functools[", "<|tool_calls|>",
           "<|python_tag|>", "<function=", "```", "{")


@dataclass
class ToolCall:
    name: str
    arguments: str                      # JSON object text
    id: str = field(default_factory=lambda: "call_" + uuid.uuid4().hex[:24])

    def openai(self) -> dict:
        return {"id": self.id, "type": "function",
                "function": {"name": self.name, "arguments": self.arguments}}

    def anthropic(self) -> dict:
        try:
            inp = json.loads(self.arguments)
        except ValueError:
            inp = {}
        return {"type": "tool_use", "id": "toolu_" + self.id[5:], "name": self.name, "input": inp}


@dataclass
class ToolSpec:
    name: str
    description: str = ""
    parameters: dict | None = None


def tools_from_openai(tools) -> list[ToolSpec]:
    """OpenAI chat ({"type": "function", "function": {...}}) or Responses
    ({"type": "function", "name": ...}) tool definitions."""
    out = []
    for t in tools or []:
        f = t.get("function", t) if isinstance(t, dict) else {}
        if t.get("type", "function") != "function" or not f.get("name"):
            raise ValueError(f"unsupported tool type {t.get('type')!r} (local models take function tools)")
        out.append(ToolSpec(f["name"], f.get("description", "") or "", f.get("parameters")))
    return out


def tools_from_anthropic(tools) -> list[ToolSpec]:
    return [ToolSpec(t["name"], t.get("description", "") or "", t.get("input_schema"))
            for t in tools or [] if isinstance(t, dict) and t.get("name")]


def tool_choice_forbids(choice) -> bool:
    """tool_choice "none" (OpenAI) or {"type": "none"} (Anthropic)."""
    if choice == "none":
        return True
    return isinstance(choice, dict) and choice.get("type") == "none"


def format_tool_prompt(tools: list[ToolSpec], choice=None) -> str:
    lines = ["You have access to the following tools. To call one or more tools, reply with "
             "ONLY a JSON object of this form and nothing else:",
             '{"tool_calls": [{"name": "<tool name>", "arguments": {<argument name>: <value>}}]}',
             "If no tool is needed, answer normally in plain text.", "", "Tools:"]
    for t in tools:
        lines.append(f"- {t.name}: {t.description}".rstrip(": "))
        props = (t.parameters or {}).get("properties") or {}
        req = set((t.parameters or {}).get("required") or [])
        for pname, ps in props.items():
            typ = ps.get("type", "any") if isinstance(ps, dict) else "any"
            desc = ps.get("description", "") if isinstance(ps, dict) else ""
            lines.append(f"    {pname} ({typ}{', required' if pname in req else ''})"
                         + (f": {desc}" if desc else ""))
    if choice == "required" or (isinstance(choice, dict) and choice.get("type") in ("any", "tool", "function")):
        forced = None
        if isinstance(choice, dict):
            forced = choice.get("name") or (choice.get("function") or {}).get("name")
        lines.append("")
        lines.append(f"You MUST call the tool {forced}." if forced else "You MUST call a tool.")
    return "\n".join(lines)


# --------------------------------------------------------------------------- parsing
def _json_at(text: str, i: int):
    """(value, end) of the JSON value starting at text[i], or (None, i)."""
    try:
        return _DEC.raw_decode(text, i)
    except ValueError:
        return None, i


def _args_text(v) -> str:
    if v is None:
        return "{}"
    if isinstance(v, str):
        try:
            v = json.loads(v)
        except ValueError:
            return json.dumps({"input": v})
    return json.dumps(v, ensure_ascii=False)


def _call_of(obj, names) -> ToolCall | None:
    if not isinstance(obj, dict):
        return None
    if isinstance(obj.get("function"), dict):
        obj = obj["function"]
    name = obj.get("name")
    if not isinstance(name, str) or (names and name not in names):
        return None
    if "parameters" in obj and "arguments" not in obj:
        args = obj["parameters"]
    else:
        args = obj.get("arguments", obj.get("input"))
    # a definition echoed back ({"name", "description", "parameters": {"type": "object"...}})
    if isinstance(args, dict) and args.get("type") == "object" and "properties" in args:
        return None
    return ToolCall(name, _args_text(args))


def _calls_of(items, names) -> list[ToolCall] | None:
    if isinstance(items, dict):
        items = [items]
    if not isinstance(items, list) or not items:
        return None
    calls = [_call_of(x, names) for x in items]
    return calls if all(c is not None for c in calls) else None


def _strip_fences(text: str) -> str:
    m = re.search(r"```(?:json|tool_call|tool_calls)?\s*\n?(.*?)```", text, re.S)
    return m.group(1) if m else text


def _try_generic(text, names):
    i = text.find("{")
    while i >= 0:
        v, end = _json_at(text, i)
        if isinstance(v, dict) and isinstance(v.get("tool_calls"), list):
            calls = _calls_of(v["tool_calls"], names)
            if calls:
                return i, calls
        i = text.find("{", i + 1)
    return None


def _try_hermes(text, names):
    start = None
    calls = []
    for tag in ("tool_call", "tools"):
        for m in re.finditer(rf"<{tag}>\s*(.*?)\s*(?:</{tag}>|$)", text, re.S):
            body = m.group(1).strip()
            if body.startswith("<function="):
                return None  # qwen-xml body
            v, end = _json_at(body, 0)
            c = _calls_of(v, names) if v is not None else None
            if not c:
                return None
            calls += c
            start = m.start() if start is None else start
        if calls:
            return start, calls
    return None


def _typed(raw: str, schema) -> object:
    typ = (schema or {}).get("type") if isinstance(schema, dict) else None
    s = raw.strip()
    if typ in ("integer", "number", "boolean", "array", "object", "null") or typ is None:
        try:
            v = json.loads(s)
            if typ is None or typ in ("array", "object", "null") or \
                    (typ == "boolean" and isinstance(v, bool)) or \
                    (typ in ("integer", "number") and isinstance(v, (int, float)) and not isinstance(v, bool)):
                return v
        except ValueError:
            pass
    return s


def _try_qwen_xml(text, names, schemas):
    ms = list(re.finditer(r"<function=([^>\s]+)>(.*?)(?:</function>|$)", text, re.S))
    if not ms:
        return None
    calls = []
    for m in ms:
        name = m.group(1)
        if names and name not in names:
            return None
        props = ((schemas.get(name) or {}).get("properties") or {})
        args = {}
        for p in re.finditer(r"<parameter=([^>\s]+)>(.*?)</parameter>", m.group(2), re.S):
            args[p.group(1)] = _typed(p.group(2).strip("\n"), props.get(p.group(1)))
        calls.append(ToolCall(name, json.dumps(args, ensure_ascii=False)))
    head = text.rfind("<tool_call>", 0, ms[0].start())
    return (head if head >= 0 else ms[0].start()), calls


def _try_mistral(text, names):
    i = text.find("[TOOL_CALLS]")
    if i < 0:
        return None
    rest = text[i + len("[TOOL_CALLS]"):].lstrip()
    if rest.startswith("["):
        v, _ = _json_at(rest, 0)
        c = _calls_of(v, names)
        return (i, c) if c else None
    calls = []
    for m in re.finditer(r"([A-Za-z0-9_.\-]+)\[ARGS\]", rest):
        v, _ = _json_at(rest, m.end())
        if v is None or (names and m.group(1) not in names):
            return None
        calls.append(ToolCall(m.group(1), _args_text(v)))
    return (i, calls) if calls else None


def _try_phi(text, names):
    for open_, skip in (("functools[", len("functools")), ("<|tool_calls|>", len("<|tool_calls|>"))):
        i = text.find(open_)
        if i >= 0:
            j = text.find("[", i + skip) if open_[0] == "<" else i + skip
            if j < 0:
                return None
            v, _ = _json_at(text, j)
            c = _calls_of(v, names)
            return (i, c) if c else None
    return None


def _try_llama3(text, names):
    i = text.find("<|python_tag|>")
    body_at = i + len("<|python_tag|>") if i >= 0 else None
    if body_at is None:
        s = text.lstrip()
        if not s.startswith("{"):
            return None
        body_at, i = len(text) - len(s), len(text) - len(s)
    v, end = _json_at(text, body_at)
    if not isinstance(v, dict) or "name" not in v or not ("parameters" in v or "arguments" in v):
        return None
    if text[end:].strip() and body_at == i:
        return None  # a bare object followed by more text is content
    c = _call_of(v, names)
    return (i, [c]) if c else None


def parse_tool_calls(text: str, tools: list[ToolSpec]) -> tuple[str, list[ToolCall]] | None:
    """(content before the calls, calls) if the text holds tool calls, else None."""
    if not tools or not text:
        return None
    names = {t.name for t in tools}
    schemas = {t.name: t.parameters for t in tools}
    for src in (text, _strip_fences(text)):
        for fn in (_try_generic, _try_hermes):
            r = fn(src, names)
            if r:
                break
        else:
            r = _try_qwen_xml(src, names, schemas) or _try_mistral(src, names) or \
                _try_phi(src, names) or _try_llama3(src, names)
        if r:
            start, calls = r
            lead = src[:start] if src is text else text[:text.find("```")]
            lead = re.sub(r"```[A-Za-z_]*\s*$", "", lead)   # an opened code fence
            seen = set()
            for c in calls:   # ids unique within the reply
                while c.id in seen:
                    c.id = "call_" + uuid.uuid4().hex[:24]
                seen.add(c.id)
            return lead.strip(), calls
    return None


def content_prefix_len(text: str) -> int:
    """Length of the prefix of `text` that is certainly content: before any
    marker that could open a tool call, and before a trailing partial marker."""
    cut = len(text)
    for m in MARKERS:
        k = text.find(m)
        if 0 <= k < cut:
            cut = k
    if cut < len(text):
        return cut
    # a marker may be arriving token by token: hold back a suffix that is a prefix of one
    hold = 0
    for m in MARKERS:
        for n in range(min(len(m) - 1, cut), hold, -1):
            if text.endswith(m[:n]):
                hold = n
                break
    return cut - hold
