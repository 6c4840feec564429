"""Request/response contract of the reference engine, for the b200 mode.

``PreparedRequest`` keeps the field layout of
``src/laya_blackwell/protocol.py:22-29`` so prepared requests move between the
modes unchanged.  ``prepare_request`` (tokenisation, ``protocol.py:37-100``) and
``format_response`` (calibrated answers, ``protocol.py:103-180``) are CPU work
outside the device path: both need the Laya SDK (``laya==0.3.9``: ``Agent``,
``laya.common``), which is imported when they are called and is not bundled.
With the SDK installed they delegate to the reference implementation when it
is importable, so the b200 mode formats answers byte-for-byte like the
balanced mode.
"""
from dataclasses import dataclass
from typing import Any


@dataclass
class PreparedRequest:
    """Ordered questions and unpadded model inputs, before any device work."""

    ids: list[str]
    questions: list[dict[str, Any]]
    items: list[dict[str, Any]]
    input_tokens: int


def _reference_protocol():
    try:
        from laya_blackwell import protocol  # noqa: PLC0415 - optional reference install
    except ImportError as exc:
        raise RuntimeError("request tokenisation and answer formatting need the Laya SDK (laya==0.3.9) and the "
                           "reference package laya_blackwell; the b200 device path itself does not") from exc
    return protocol


def prepare_request(tok, cfg, state, questions, **kwargs):
    return _reference_protocol().prepare_request(tok, cfg, state, questions, **kwargs)


def format_response(prepared, logits, act_logits, temperature, temperature_by_options):
    proto = _reference_protocol()
    ref = proto.PreparedRequest(prepared.ids, prepared.questions, prepared.items, prepared.input_tokens)
    return proto.format_response(ref, logits, act_logits, temperature, temperature_by_options)
