"""Model chat templates (the Jinja dialect of Hugging Face ``chat_template``
strings, as shipped in ``tokenizer_config.json`` and in GGUF metadata under
``tokenizer.chat_template``) and tool calls.

* ``JinjaChatTemplate``  renders a template in a sandboxed jinja2
  environment with the variables such templates expect (``messages``,
  ``tools``, ``add_generation_prompt``, ``bos_token``, ``eos_token``,
  ``raise_exception``, the ``tojson`` filter); messages keep every field
  (``tool_calls``, ``tool_call_id``, ``name``), so tool-use conversations
  render as the model was trained on them.
* ``parse_tool_calls``   finds ``<tool_call>{json}</tool_call>`` blocks (the
  Qwen2.5 / Hermes convention) in generated text and returns the remaining
  text and OpenAI ``tool_calls`` entries, each rendered with the native
  ``aether_tool_render_call``.

The reference implements a subset (variables, ``for m in messages``, ``if``)
in its C ABI (runtime/src/lib.rs:5304-5530) plus ``aether_tool_render_call``
(lib.rs:9712); that subset is ``runtime.render_template`` here.
"""
from __future__ import annotations

import json
import re
import uuid

_TOOL_RE = re.compile(r"<tool_call>\s*(\{.*?\})\s*</tool_call>", re.S)


class TemplateError(ValueError):
    pass


class JinjaChatTemplate:
    def __init__(self, source: str, bos_token: str = "", eos_token: str = ""):
        from jinja2.sandbox import ImmutableSandboxedEnvironment

        def raise_exception(msg):
            raise TemplateError(msg)

        env = ImmutableSandboxedEnvironment(trim_blocks=True, lstrip_blocks=True)
        env.filters["tojson"] = lambda x, indent=None, **kw: json.dumps(x, ensure_ascii=False, indent=indent)
        env.globals["raise_exception"] = raise_exception
        self.template = env.from_string(source)
        self.source = source
        self.bos_token, self.eos_token = bos_token, eos_token

    def render(self, messages: list, tools: list | None = None, add_generation_prompt: bool = True, **extra) -> str:
        return self.template.render(messages=messages, tools=tools, add_generation_prompt=add_generation_prompt,
                                    bos_token=self.bos_token, eos_token=self.eos_token, **extra)

    @staticmethod
    def from_hf_dir(path: str) -> "JinjaChatTemplate | None":
        import os

        f = os.path.join(path, "tokenizer_config.json")
        if not os.path.exists(f):
            return None
        with open(f) as fh:
            cfg = json.load(fh)
        src = cfg.get("chat_template")
        if isinstance(src, list):  # named templates: take "default"
            src = next((t["template"] for t in src if t.get("name") == "default"), None)
        if not src:
            return None

        def tok(v):
            return v.get("content", "") if isinstance(v, dict) else (v or "")

        return JinjaChatTemplate(src, tok(cfg.get("bos_token")), tok(cfg.get("eos_token")))

    @staticmethod
    def from_gguf(g) -> "JinjaChatTemplate | None":
        src = g.meta.get("tokenizer.chat_template")
        if not src:
            return None
        toks = g.meta.get("tokenizer.ggml.tokens") or []

        def tok(key):
            i = g.meta.get(key)
            return toks[int(i)] if i is not None and 0 <= int(i) < len(toks) else ""

        return JinjaChatTemplate(src, tok("tokenizer.ggml.bos_token_id"), tok("tokenizer.ggml.eos_token_id"))


def parse_tool_calls(text: str):
    """-> (content without the tool-call blocks, [OpenAI tool_call dicts])."""
    from ..runtime import render_tool_call

    calls = []
    for m in _TOOL_RE.finditer(text):
        try:
            obj = json.loads(m.group(1))
        except ValueError:
            continue
        name = obj.get("name")
        if not isinstance(name, str):
            continue
        args = obj.get("arguments", {})
        args_s = args if isinstance(args, str) else json.dumps(args, ensure_ascii=False)
        call = json.loads(render_tool_call(name, args_s))
        call["id"] = f"call_{uuid.uuid4().hex[:24]}"
        calls.append(call)
    content = _TOOL_RE.sub("", text).strip() if calls else text
    return content, calls
