"""Process-wide token-mode selector.

Mirrors the reference's runtime switch (``src/base_model/encoding/encoding.py:33-112``):
``Message_Tokenizer`` and ``Vocab`` are proxies that forward attribute access
and construction to the active mode, so names imported before a switch still
see it.  The default mode is 26tok, as in the reference.
"""
from __future__ import annotations

from typing import Any

from .tokenizer import MODES, get_tokenizer

SUPPORTED_TOKEN_MODES = ("22tok", "23tok", "24tok", "26tok")
DEFAULT_TOKEN_MODE = "26tok"
_active = DEFAULT_TOKEN_MODE


def get_token_mode() -> str:
    return _active


def supported_token_modes() -> tuple:
    return SUPPORTED_TOKEN_MODES


def set_token_mode(mode: str) -> None:
    """Point every proxy at ``mode``.  Call once, before building data or models."""
    global _active
    get_tokenizer(mode)  # validates first, so a bad name leaves no half state
    _active = mode


def active_tokenizer():
    return get_tokenizer(_active)


class _Proxy(type):
    _target = ""

    def __getattr__(cls, name: str) -> Any:
        tok = get_tokenizer(_active)
        impl = tok if cls._target == "Message_Tokenizer" else tok.vocab
        try:
            return getattr(impl, name)
        except AttributeError:
            raise AttributeError(f"{cls._target} of {_active} has no {name!r}") from None

    def __call__(cls, *a, **k):
        tok = get_tokenizer(_active)
        return tok if cls._target == "Message_Tokenizer" else tok.vocab

    def __repr__(cls) -> str:
        return f"<{cls._target} of {_active}>"


class Message_Tokenizer(metaclass=_Proxy):
    _target = "Message_Tokenizer"


class Vocab(metaclass=_Proxy):
    _target = "Vocab"


def encode_msgs(msgs):
    return get_tokenizer(_active).encode_msgs(msgs)


def decode_msgs(toks):
    return get_tokenizer(_active).decode_msgs(toks)
