"""Chat templates: the GGUF's own Jinja template when it has one
(``tokenizer.chat_template``), else a built-in format per architecture.

Reference: src/inference/chat_template/mod.rs:53 (minijinja + pycompat),
harmony channels for gpt-oss (src/inference/harmony.rs:78).
"""
from __future__ import annotations

BUILTIN = {
    # Llama-3 header format
    "llama": ("{% for m in messages %}<|start_header_id|>{{ m['role'] }}<|end_header_id|>\n\n"
              "{{ m['content'] }}<|eot_id|>{% endfor %}"
              "{% if add_generation_prompt %}<|start_header_id|>assistant<|end_header_id|>\n\n{% endif %}"),
    # ChatML (Qwen family)
    "qwen3next": ("{% for m in messages %}<|im_start|>{{ m['role'] }}\n{{ m['content'] }}<|im_end|>\n"
                  "{% endfor %}{% if add_generation_prompt %}<|im_start|>assistant\n{% endif %}"),
    # harmony (gpt-oss): final channel only
    "gpt-oss": ("{% for m in messages %}<|start|>{{ m['role'] }}<|message|>{{ m['content'] }}<|end|>"
                "{% endfor %}{% if add_generation_prompt %}<|start|>assistant<|channel|>final<|message|>{% endif %}"),
    # Gemma turns (no system role: a system message is sent as a user turn)
    "gemma": ("{% for m in messages %}<start_of_turn>{{ 'model' if m['role'] == 'assistant' else 'user' }}\n"
              "{{ m['content'] }}<end_of_turn>\n{% endfor %}"
              "{% if add_generation_prompt %}<start_of_turn>model\n{% endif %}"),
}
for _fam in ("qwen2", "qwen3", "qwen2moe", "qwen3moe", "qwen35", "qwen35moe"):
    BUILTIN[_fam] = BUILTIN["qwen3next"]
for _fam in ("gemma2", "gemma3"):
    BUILTIN[_fam] = BUILTIN["gemma"]


def render(messages: list[dict], arch: str = "llama", template: str | None = None,
           add_generation_prompt: bool = True) -> str:
    import jinja2
    env = jinja2.Environment(trim_blocks=False, lstrip_blocks=False,
                             undefined=jinja2.ChainableUndefined)
    env.globals["raise_exception"] = lambda msg: (_ for _ in ()).throw(ValueError(msg))
    tpl = env.from_string(template or BUILTIN.get(arch, BUILTIN["llama"]))
    norm = []
    for m in messages:
        c = m.get("content", "")
        if isinstance(c, list):  # OpenAI content parts
            c = "".join(p.get("text", "") for p in c if isinstance(p, dict))
        norm.append({"role": m.get("role", "user"), "content": c or ""})
    return tpl.render(messages=norm, add_generation_prompt=add_generation_prompt,
                      bos_token="", eos_token="")
