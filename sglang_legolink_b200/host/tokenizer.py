"""Tokenizers for the host pipeline.

* :class:`RegexTokenizer` -- dependency-free *estimate* (string pieces).  Its
  counts never decide compile eligibility or runtime layout.
* :class:`HashTokenizer` -- deterministic integer ids (regex pieces hashed into
  a vocabulary) with a ChatML-style template; the tokenizer of the CPU fake
  runtime and of random-init benchmark models, whose checkpoints ship no
  tokenizer files.
* :class:`HFTokenizer` -- the model's own ``tokenizer.json`` + Jinja chat
  template through ``transformers``.
* :class:`RuntimeTokenizer` -- the runtime's authoritative ``/v1/tokenize``
  (prompt or messages + chat template), LRU-cached (reference
  ``noc_context_manager/tokenizer.py:330-445``).

Every tokenizer has a ``fingerprint`` that enters cache keys, and a
``token_unit`` ("model" or "estimated").
"""

from __future__ import annotations

import functools
import hashlib
import json
import re
import urllib.request
from typing import Any, Optional, Sequence

TOKEN_PATTERN = re.compile(r"[A-Za-z]+|[0-9]|[一-鿿]|\s+|[^\sA-Za-z0-9]", re.UNICODE)


class RegexTokenizer:
    token_unit = "estimated"
    fingerprint = "regex-ascii-cjk-punct-v1"

    def tokenize(self, text: str) -> tuple:
        return tuple(TOKEN_PATTERN.findall(text))

    def count(self, text: str) -> int:
        return len(TOKEN_PATTERN.findall(text))


class HashTokenizer:
    """Integer-id tokenizer: each regex piece maps to ``2 + sha1(piece) % (V-8)``.
    Ids 0..1 and the last 6 ids are reserved for the chat template."""

    token_unit = "model"

    def __init__(self, vocab_size: int = 1024, name: str = "hash"):
        self.vocab_size = vocab_size
        self.name = name
        v = vocab_size
        self.special = {"<|im_start|>": v - 6, "<|im_end|>": v - 5, "<|endoftext|>": v - 4}
        self.fingerprint = f"hash-tokenizer-v1:{name}:{vocab_size}"
        self.chat_template_sha256 = hashlib.sha256(b"chatml:<|im_start|>{role}\\n{content}<|im_end|>\\n").hexdigest()
        self.eos_token_id = self.special["<|im_end|>"]

    @functools.lru_cache(maxsize=65536)
    def _piece(self, p: str) -> int:
        return 2 + int(hashlib.sha1(p.encode()).hexdigest(), 16) % (self.vocab_size - 8)

    def tokenize(self, text: str) -> tuple[int, ...]:
        return tuple(self._piece(p) for p in TOKEN_PATTERN.findall(text))

    def count(self, text: str) -> int:
        return len(TOKEN_PATTERN.findall(text))

    def tokenize_messages(self, messages: Sequence[dict], *, tools=None, tool_choice=None, reasoning_effort=None,
                          continue_final_message=False, chat_template_kwargs=None, add_generation_prompt=True):
        ids: list[int] = []
        s, e = self.special["<|im_start|>"], self.special["<|im_end|>"]
        if tools:
            ids += [s] + list(self.tokenize("system\n" + json.dumps(tools, sort_keys=True))) + [e] + list(
                self.tokenize("\n"))
        for i, m in enumerate(messages):
            ids += [s] + list(self.tokenize(f"{m.get('role', 'user')}\n")) + list(self.tokenize(m.get("content") or ""))
            last = i == len(messages) - 1
            if not (continue_final_message and last):
                ids += [e] + list(self.tokenize("\n"))
        if add_generation_prompt and not continue_final_message:
            ids += [s] + list(self.tokenize("assistant\n"))
        return tuple(ids)

    def decode(self, ids: Sequence[int]) -> str:
        return " ".join(f"<{int(i)}>" for i in ids)


class HFTokenizer:
    token_unit = "model"

    def __init__(self, path_or_name: str):
        from transformers import AutoTokenizer

        self.tok = AutoTokenizer.from_pretrained(path_or_name)
        tmpl = getattr(self.tok, "chat_template", None) or ""
        self.chat_template_sha256 = hashlib.sha256(str(tmpl).encode()).hexdigest()
        self.fingerprint = f"hf:{path_or_name}:{len(self.tok)}:{self.chat_template_sha256[:12]}"
        self.eos_token_id = self.tok.eos_token_id
        self.vocab_size = len(self.tok)

    def tokenize(self, text: str) -> tuple[int, ...]:
        return tuple(self.tok.encode(text, add_special_tokens=False))

    def count(self, text: str) -> int:
        return len(self.tokenize(text))

    def tokenize_messages(self, messages, *, tools=None, tool_choice=None, reasoning_effort=None,
                          continue_final_message=False, chat_template_kwargs=None, add_generation_prompt=True):
        kw = dict(chat_template_kwargs or {})
        if reasoning_effort is not None:
            kw["reasoning_effort"] = reasoning_effort
        ids = self.tok.apply_chat_template(list(messages), tools=tools, tokenize=True,
                                           add_generation_prompt=add_generation_prompt and not continue_final_message,
                                           continue_final_message=continue_final_message, **kw)
        if isinstance(ids, dict):
            ids = ids["input_ids"]
        return tuple(int(i) for i in ids)

    def decode(self, ids) -> str:
        return self.tok.decode(list(ids), skip_special_tokens=True)


class RuntimeTokenizer:
    """The runtime's ``/v1/tokenize`` (authoritative)."""

    token_unit = "model"

    def __init__(self, api_base: str, model: str = "default", timeout: float = 60.0, cache_size: int = 4096):
        self.api_base = api_base.rstrip("/")
        self.model = model
        self.timeout = timeout
        self._cached = functools.lru_cache(maxsize=cache_size)(self._tokenize_serialized)
        info = self._get("/model_info")
        self.fingerprint = str(info.get("tokenizer_fingerprint") or f"runtime:{self.api_base}:{model}")
        self.chat_template_sha256 = str(info.get("chat_template_sha256") or "0" * 64)
        self.eos_token_id = info.get("eos_token_id")

    def _url(self, path: str) -> str:
        base = self.api_base[:-3] if self.api_base.endswith("/v1") else self.api_base
        return base + path

    def _get(self, path: str) -> dict:
        try:
            with urllib.request.urlopen(self._url(path), timeout=self.timeout) as r:
                return json.loads(r.read())
        except Exception:
            return {}

    def _post(self, payload: dict) -> dict:
        req = urllib.request.Request(self.api_base + "/tokenize", data=json.dumps(payload).encode(),
                                     headers={"Content-Type": "application/json"})
        with urllib.request.urlopen(req, timeout=self.timeout) as r:
            return json.loads(r.read())

    def _tokenize_serialized(self, payload: str) -> tuple[int, ...]:
        body = self._post(json.loads(payload))
        ids = body.get("tokens", body.get("input_ids"))
        if not isinstance(ids, list):
            raise ValueError(f"/v1/tokenize returned no token list: {body!r}")
        return tuple(int(i) for i in ids)

    def tokenize(self, text: str) -> tuple[int, ...]:
        return self._cached(json.dumps({"model": self.model, "prompt": text, "add_special_tokens": False},
                                       sort_keys=True))

    def count(self, text: str) -> int:
        return len(self.tokenize(text))

    def tokenize_messages(self, messages, *, tools=None, tool_choice=None, reasoning_effort=None,
                          continue_final_message=False, chat_template_kwargs=None, add_generation_prompt=True):
        p = {"model": self.model, "messages": list(messages), "add_generation_prompt": add_generation_prompt,
             "continue_final_message": continue_final_message}
        if tools:
            p["tools"] = list(tools)
        if chat_template_kwargs:
            p["chat_template_kwargs"] = dict(chat_template_kwargs)
        return self._cached(json.dumps(p, sort_keys=True))


def count_tokens(text: str, tokenizer=None) -> int:
    return (tokenizer or RegexTokenizer()).count(text)


def require_model_tokens(tokenizer, purpose: str) -> None:
    """Refuse to compare estimated counts against a model-token floor."""
    if getattr(tokenizer, "token_unit", "estimated") != "model":
        raise ValueError(f"{purpose} needs an authoritative (model) tokenizer, got an estimate")


def load_tokenizer(spec: Optional[str], *, vocab_size: int = 1024, api_base: Optional[str] = None):
    if spec in (None, "", "regex"):
        return RegexTokenizer()
    if spec.startswith("hash"):
        return HashTokenizer(vocab_size)
    if spec == "runtime":
        if not api_base:
            raise ValueError("runtime tokenizer needs api_base")
        return RuntimeTokenizer(api_base)
    return HFTokenizer(spec)
