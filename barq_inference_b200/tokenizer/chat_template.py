"""Chat templates: built-in presets plus the GGUF ``tokenizer.chat_template`` (Jinja).

Parity: ``ChatTemplate`` (``vocab/src/chat_template.rs:18-291``) with presets Llama / Mistral
(``[INST]`` + ``<<SYS>>``), Qwen / ChatML (``<|im_start|>``) and Generic, roles system / user /
assistant / tool / developer, and ``for_arch`` selection.  The role marker strings are the public
prompt formats of those model families, so they are necessarily the same text.  The reference only
*tries* to read the GGUF template (``cli/src/main.rs:475-482`` calls a method that does not exist);
here it is rendered with a sandboxed Jinja environment when present, and Llama-3's header format
is added as a preset.
"""
from __future__ import annotations

from dataclasses import dataclass

ROLES = ("system", "user", "assistant", "tool", "developer")


def parse_role(role: str) -> str:
    """Lenient role parsing (``cli/src/server.rs:960``): unknown roles are treated as user."""
    r = (role or "").strip().lower()
    return r if r in ROLES else "user"


@dataclass(frozen=True)
class Markers:
    prefix: dict
    suffix: dict
    bos: str = ""
    generation_prompt: str = ""


_LLAMA2 = Markers(
    prefix={"system": "<<SYS>>\n", "user": "[INST] ", "assistant": "", "tool": "[TOOL] ", "developer": "[DEV] "},
    suffix={"system": "\n<</SYS>>\n\n", "user": " [/INST]\n", "assistant": "</s>\n", "tool": "\n", "developer": "\n"},
)
_CHATML = Markers(
    prefix={r: f"<|im_start|>{r}\n" for r in ROLES},
    suffix={r: "<|im_end|>\n" for r in ROLES},
    generation_prompt="<|im_start|>assistant\n",
)
_GENERIC = Markers(
    prefix={"system": "[SYSTEM] ", "user": "[USER] ", "assistant": "[ASSISTANT] ", "tool": "[TOOL] ",
            "developer": "[DEVELOPER] "},
    suffix={r: "\n" for r in ROLES},
    generation_prompt="[ASSISTANT] ",
)
_LLAMA3 = Markers(
    prefix={r: f"<|start_header_id|>{'ipython' if r == 'tool' else r}<|end_header_id|>\n\n" for r in ROLES},
    suffix={r: "<|eot_id|>" for r in ROLES},
    bos="<|begin_of_text|>",
    generation_prompt="<|start_header_id|>assistant<|end_header_id|>\n\n",
)

PRESETS = {"llama": _LLAMA2, "mistral": _LLAMA2, "qwen": _CHATML, "chatml": _CHATML, "generic": _GENERIC,
           "llama3": _LLAMA3}

ARCH_PRESET = {"llama": "llama", "mistral": "mistral", "mixtral": "mistral", "qwen": "qwen", "qwen2": "qwen",
               "qwen2moe": "qwen", "qwen3": "qwen", "qwen3moe": "qwen", "deepseek": "chatml", "deepseek2": "chatml"}


class ChatTemplate:
    def __init__(self, preset: str = "generic", jinja_source: str | None = None, bos_token: str = "",
                 eos_token: str = ""):
        if preset not in PRESETS:
            raise ValueError(f"unknown chat template preset {preset!r}; known: {sorted(PRESETS)}")
        self.preset = preset
        self.markers = PRESETS[preset]
        self.jinja_source = jinja_source
        self.bos_token, self.eos_token = bos_token, eos_token
        self._jinja = None
        if jinja_source:
            try:
                from jinja2.sandbox import ImmutableSandboxedEnvironment

                env = ImmutableSandboxedEnvironment(trim_blocks=True, lstrip_blocks=True)

                def raise_exception(msg):
                    raise ValueError(msg)

                env.globals["raise_exception"] = raise_exception
                self._jinja = env.from_string(jinja_source)
            except Exception:  # malformed template: fall back to the preset
                self._jinja = None

    @staticmethod
    def for_arch(arch: str, metadata: dict | None = None) -> "ChatTemplate":
        md = metadata or {}
        src = md.get("tokenizer.chat_template")
        preset = ARCH_PRESET.get(arch, "generic")
        toks = md.get("tokenizer.ggml.tokens")
        if toks is not None and "<|start_header_id|>" in set(toks):
            preset = "llama3"
        bos = eos = ""
        if toks is not None:
            b, e = md.get("tokenizer.ggml.bos_token_id"), md.get("tokenizer.ggml.eos_token_id")
            bos = toks[b] if b is not None and b < len(toks) else ""
            eos = toks[e] if e is not None and e < len(toks) else ""
        return ChatTemplate(preset, src, bos, eos)

    def render(self, messages: list[dict], add_generation_prompt: bool = True) -> str:
        msgs = [{"role": parse_role(m.get("role", "user")), "content": _content(m.get("content", ""))} for m in messages]
        if self._jinja is not None:
            try:
                return self._jinja.render(messages=msgs, add_generation_prompt=add_generation_prompt,
                                          bos_token=self.bos_token, eos_token=self.eos_token)
            except Exception:
                pass
        mk = self.markers
        out = [mk.bos]
        if self.preset in ("llama", "mistral"):
            # Llama-2 folds the system prompt into the first user turn.
            sys_txt = "\n".join(m["content"] for m in msgs if m["role"] == "system")
            first_user = True
            for m in msgs:
                if m["role"] == "system":
                    continue
                c = m["content"]
                if m["role"] == "user" and first_user and sys_txt:
                    c = mk.prefix["system"] + sys_txt + mk.suffix["system"] + c
                    first_user = False
                out.append(mk.prefix[m["role"]] + c + mk.suffix[m["role"]])
            return "".join(out)
        for m in msgs:
            out.append(mk.prefix[m["role"]] + m["content"] + mk.suffix[m["role"]])
        if add_generation_prompt:
            out.append(mk.generation_prompt)
        return "".join(out)


def _content(c) -> str:
    if isinstance(c, str):
        return c
    if isinstance(c, list):  # OpenAI content parts
        return "".join(p.get("text", "") for p in c if isinstance(p, dict))
    return str(c)
